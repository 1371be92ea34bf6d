// Sparse lightning-indexer KL-loss gradient for sm_100a (tcgen05).
//
// Replaces the reference core `_sparse_lightning_indexer_grad_kl_loss_core` and its
// kernels `_gather_kv_kernel`, `_indexer_grad_kl_loss_kernel`, `_scatter_dkey_index_kernel`,
// `_cast_dkey_index_kernel` (sparse_lightning_indexer_grad_kl_loss_triton.py:39-327, :355-464).
// Per query row with window n = min(topK, max(act_k - act_q + s1 + 1, 0)) (first n index
// entries, ids clamped to [0, S2-1]; rows with s1 >= act_q contribute nothing):
//   p[k]   = (1/N1) sum_h exp(scale (q_h.k + qr_h.kr) - max_h) / (sum_h + 1e-8)
//   I[k]   = sum_g w_g ReLU(qi_g . ki_k);  sI = exp(I - max I) / (sum + 1e-8);  dI = sI - p
//   loss  += sum_k max(p,1e-8) (log max(p,1e-8) - log max(sI,1e-8))
//   dW_g   = sum_k dI_k ReLU_gk;  C_kg = dI_k w_g [ReLU_gk > 0]
//   dQI    = C^T KI;  dKI[idx_k] += C_k QI  (scatter-add)
//
// No gathered copies are materialised (the reference writes [rows, topK, 512] gathers and a
// [rows, Nidx1, topK] ReLU cache, :396-429).  Two kernels:
//   teacher : CTA pair per row.  2-SM UMMA with M = 256 keys (128 per CTA) and N = 128
//             query heads (Q split 64/64 across the pair), so each thread of the epilogue
//             owns one key and all 128 head scores of it: p[k] is a per-thread sum.
//             Keys stream through a ring of 64-dim chunks (TMA gather4, 2-SM form, issued
//             by 8 warps).
//   index   : one CTA per row.  Pass A: I = KI QI^T (UMMA, keys as M) -> softmax, dI, loss.
//             Pass B: recompute ReLU(KI QI^T), form C in shared memory, then dQI^T += KI^T C
//             and dKI_tile = C QI on tcgen05; dKI rows are scatter-added in fp32 with
//             coalesced vector reductions, dW is reduced in registers.  C is stored as a
//             sum of two 16-bit parts (hi + lo) and both are multiplied, so the products
//             keep ~16 significant bits as the reference's fp32 products do.

#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_b200.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace dsa {
namespace sli {

constexpr float kEps = 1e-8f;
constexpr float kLog2e = 1.4426950408889634f;

struct Args {
  const void* q;
  const void* qr;
  const void* k;
  const void* kr;
  const void* qi;
  const void* ki;
  const void* w;
  const int32_t* idx;
  const float* smax;
  const float* ssum;
  const int32_t* act_q;
  const int32_t* act_k;
  float* p;          // [rows][topk] teacher distribution (scratch)
  void* dqi;         // [rows][Ni][128]
  float* dki_acc;    // [B*S2][128]
  void* dw;          // [rows][Ni]
  float* loss;       // [1]
  int* err;
  int rows, S1, S2, N1, Ni, topk, w_dtype;
  float scale;
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bar.sync is the aligned form: the whole warp must arrive converged, so converge it first
// (a lane that left a wait early, e.g. after a timeout, rejoins here)
__device__ __forceinline__ void named_bar(int id, int n) {
  __syncwarp();
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// window of a query row; b / s1 from the BSND row index
__device__ __forceinline__ int row_window(const Args& a, int row, int* b_out) {
  const int b = row / a.S1, s1 = row % a.S1;
  *b_out = b;
  const int aq = __ldg(a.act_q + b), ak = __ldg(a.act_k + b);
  if (s1 >= aq) return 0;
  return min(a.topk, max(ak - aq + s1 + 1, 0));
}

__device__ __forceinline__ int key_row_of(const Args& a, int b, int row, int e) {
  const int id = __ldg(a.idx + (size_t)row * a.topk + e);
  return b * a.S2 + min(max(id, 0), a.S2 - 1);   // clamp (:63, :300)
}

// =====================================================================================
// teacher distribution p
// =====================================================================================
constexpr int kTKeys = 128;        // keys per CTA per tile (pair tile: 256)
constexpr int kTStages = 6;        // ring of 64-dim key chunks
constexpr int kTGather0 = 6;
constexpr int kTGathers = 8;       // a thread issues one gather4 every ~100 cycles and the
                                   // lanes of a warp take turns: 4 gathers per warp
constexpr int kTThreads = 32 * (kTGather0 + kTGathers);   // 0: Q/stats, 1: MMA,
                                                          // 2-5: epilogue, 6-13: key gathers

template <int D>
struct TCfg {
  static constexpr int kNope = D / 64;
  static constexpr int kChunks = kNope + 1;
  static constexpr int kQBytes = kChunks * 64 * 128;      // 64 heads of this CTA
  static constexpr int kStage = kTKeys * 128;             // 128 keys x 64 dims
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kQBytes;
  static constexpr int kOffBars = kOffK + kTStages * kStage;
};

struct TMaps {
  CUtensorMap q, qr, k, kr;   // k / kr: box 64 x 1 (gather4 rows)
};

struct __align__(16) TBars {
  uint64_t q_full, full[kTStages], empty[kTStages], tfull[2], tfree[2];
  uint32_t tmem_slot;
  float mxl[128];
  float inv[128];
};

template <int D, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTThreads, 1)
    sli_teacher_kernel(const __grid_constant__ TMaps maps, const Args a) {
  using C = TCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TBars& bars = *reinterpret_cast<TBars*>(smem_raw + C::kOffBars);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sQ = sbase + C::kOffQ, sK = sbase + C::kOffK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const uint32_t cta = cluster_ctarank();
  const int row = blockIdx.x >> 1;
  int b;
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const int n = abort ? 0 : row_window(a, row, &b);
  const int ntiles = (n + 2 * kTKeys - 1) / (2 * kTKeys);
  const int nsteps = ntiles * C::kChunks;

  for (int h = threadIdx.x; h < 128; h += kTThreads) {
    if (h < a.N1) {
      bars.mxl[h] = __ldg(a.smax + (size_t)row * a.N1 + h) * kLog2e;
      bars.inv[h] = 1.f / (__ldg(a.ssum + (size_t)row * a.N1 + h) + kEps);
    } else {   // padded heads: exp2(s - inf) = 0, so they add nothing
      bars.mxl[h] = INFINITY;
      bars.inv[h] = 0.f;
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars.q_full), 1);
    for (int s = 0; s < kTStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);   // bytes of both CTAs' gathers
      mbar_init(smem_u32(&bars.empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars.tfull[s]), 1);
      mbar_init(smem_u32(&bars.tfree[s]), 2);
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(smem_u32(&bars.tmem_slot), 256);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool failed = false;

  if (warp == 0) {
    if (ntiles > 0) {
      const uint32_t lead = mapa_shared(smem_u32(&bars.q_full), 0);
      if (cta == 0 && lane == 0) mbar_arrive_expect_tx(smem_u32(&bars.q_full), 2 * C::kQBytes);
      __syncwarp();
      const int qrow0 = row * a.N1 + 64 * (int)cta;
      if (lane < C::kChunks)
        tma_load_2d_pair(sQ + lane * 64 * 128, lane < C::kNope ? &maps.q : &maps.qr, lead,
                         lane < C::kNope ? 64 * lane : 0, qrow0);
    }
  } else if (warp >= kTGather0) {
    // the CTA's 128 keys of each tile, chunk by chunk, by TMA gather4 in the 2-SM form:
    // warp w gathers keys [16w, 16w+16) (4 gathers of 4 rows), and the bytes of both CTAs
    // are counted on the leader's barrier, so no thread waits for the data
    const int w = warp - kTGather0;
    const int filler = n > 0 ? key_row_of(a, b, row, 0) : 0;
    int r4[4] = {0, 0, 0, 0};
    for (int j = 0; j < nsteps && !failed; ++j) {
      const int t = j / C::kChunks, c = j % C::kChunks, s = j % kTStages;
      if (c == 0) {
        const int e = 2 * kTKeys * t + kTKeys * (int)cta + 16 * w + (lane & 15);
        const int my_row = e < n ? key_row_of(a, b, row, e) : filler;
#pragma unroll
        for (int q = 0; q < 4; ++q) r4[q] = __shfl_sync(0xffffffffu, my_row, 4 * (lane & 3) + q);
      }
      mbar_wait(smem_u32(&bars.empty[s]), ((j / kTStages) & 1) ^ 1, a.err, &failed);
      if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
      const uint32_t full = smem_u32(&bars.full[s]);
      if (cta == 0 && w == 0 && lane == 0) mbar_arrive_expect_tx(full, 2 * C::kStage);
      if (lane < 4)
        tma_gather4_pair(sK + s * C::kStage + (16 * w + 4 * lane) * 128,
                         c < C::kNope ? &maps.k : &maps.kr, mapa_shared(full, 0),
                         c < C::kNope ? 64 * c : 0, r4[0], r4[1], r4[2], r4[3]);
      __syncwarp();
    }
  } else if (warp == 1) {
    // The whole warp runs the loop (waits included); one elected lane issues each tcgen05
    // instruction (a lone lane issues MMAs much more slowly).
    if (cta == 0 && ntiles > 0) {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id = idesc_f16(256, 128, bf16, false, false);
      const uint64_t dq = smem_desc_sw128(sQ, 16, 1024);
      const uint64_t dk = smem_desc_sw128(sK, 16, 1024);
      mbar_wait_spin(smem_u32(&bars.q_full), 0, a.err, &failed);
      for (int t = 0; t < ntiles && !failed; ++t) {
        const int buf = t & 1;
        if (t >= 2) mbar_wait_spin(smem_u32(&bars.tfree[buf]), ((t >> 1) - 1) & 1, a.err, &failed, true);
        for (int c = 0; c < C::kChunks; ++c) {
          const int j = t * C::kChunks + c, s = j % kTStages;
          mbar_wait_spin(smem_u32(&bars.full[s]), (j / kTStages) & 1, a.err, &failed, true);
          if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              umma_f16<2>(tmem + 128 * buf, dk + (uint64_t)((s * C::kStage + u * 32) >> 4),
                          dq + (uint64_t)((c * 64 * 128 + u * 32) >> 4), id, (c | u) != 0);
            umma_commit_pair(smem_u32(&bars.empty[s]), 3);
          }
          __syncwarp();
        }
        if (failed) break;
        if (elect_one()) umma_commit_pair(smem_u32(&bars.tfull[buf]), 3);
        __syncwarp();
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread = key; p = (1/N1) sum_h softmax_h[key] ----
    const int qd = warp & 3;
    const int kk = 32 * qd + lane;
    const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
    const float c2 = a.scale * kLog2e;
    const float invn = 1.f / (float)a.N1;
    const uint32_t lead_f0 = mapa_shared(smem_u32(&bars.tfree[0]), 0);
    const uint32_t lead_f1 = mapa_shared(smem_u32(&bars.tfree[1]), 0);
    float* prow = a.p + (size_t)row * a.topk;
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      mbar_wait(smem_u32(&bars.tfull[buf]), (t >> 1) & 1, a.err, &failed);
      const bool wfail = __any_sync(0xffffffffu, failed);
      tc_fence_after();
      float acc = 0.f;
      if (!wfail) {
        for (int h0 = 0; h0 < 128; h0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_addr + 128 * buf + h0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            acc = fmaf(ex2f(fmaf(__uint_as_float(r[i]), c2, -bars.mxl[h0 + i])), bars.inv[h0 + i], acc);
        }
      }
      tc_fence_before();
      named_bar(1, 128);
      if (warp == 2 && lane == 0) mbar_arrive_cluster(buf ? lead_f1 : lead_f0);
      const int e = 2 * kTKeys * t + kTKeys * (int)cta + kk;
      if (e < n) prow[e] = acc * invn;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, 256);
}

// =====================================================================================
// index part: I, softmax/KL, dI, dW, dQI, dKI
// =====================================================================================
constexpr int kIKeys = 128;      // keys per tile (UMMA M)
constexpr int kNip = 64;         // index heads padded to 64
constexpr int kDi = 128;         // index head dim
constexpr int kIDrain0 = 6;      // first dKI drain warp
constexpr int kIDrainWarps = 8;  // two per TMEM lane quadrant, 64 columns each
constexpr int kIGather1 = kIDrain0 + kIDrainWarps;   // extra gather warps after the drains
constexpr int kIGathers = 3;     // warp 0 + 2: a thread issues one gather4 every ~100 cycles
                                 // and the lanes of a warp take turns (16 warps keep the
                                 // 128-register budget)
constexpr int kIThreads = 32 * (kIGather1 + kIGathers - 1);   // 0, 14-16: gathers, 1: MMA,
                                                               // 2-5: epilogue, 6-13: drains

template <int STG>
struct ICfg {
  static constexpr int kQiBytes = 2 * kNip * 128;           // [dim chunk][64 heads][128 B]
  static constexpr int kStage = 2 * kIKeys * 128;           // [dim chunk][128 keys][128 B]
  static constexpr int kCBytes = 2 * kIKeys * 128;          // C = hi + lo: 2 x [128 keys][64 heads]
  static constexpr int kOffQi = 0;
  static constexpr int kOffK = kQiBytes;
  static constexpr int kOffC = kOffK + STG * kStage;
  static constexpr int kOffStage = kOffC + 2 * kCBytes;       // drain staging, 32 x 33 floats per drain warp
  // dW column sums (128 x 65 floats) reuse the key ring: they are formed after the last
  // tile's MMAs, when no gather or MMA touches the ring any more
  static constexpr int kOffRed = kOffK;
  static_assert(128 * 65 * 4 <= STG * kStage, "dW sums fit the key ring");
  static constexpr int kOffI = kOffStage + kIDrainWarps * 32 * 33 * 4;   // I then dI: topk floats
};

struct IMaps {
  CUtensorMap ki;
};

template <int STG>
struct __align__(16) IBars {
  uint64_t full[STG], empty[STG], rfull[2], rfree[2], cready[2], cfree[2], dfull[2], dfree[2], qdone;
  uint32_t tmem_slot;
  float w[kNip];
  float red[8];
  float stat[4];
};

template <typename T, int STG>
__global__ void __launch_bounds__(kIThreads, 1)
    sli_index_kernel(const __grid_constant__ IMaps maps, const Args a) {
  using C = ICfg<STG>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int topk_pad = (a.topk + 3) & ~3;
  IBars<STG>& bars = *reinterpret_cast<IBars<STG>*>(smem_raw + C::kOffI + topk_pad * 4);
  float* Ibuf = reinterpret_cast<float*>(smem_raw + C::kOffI);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sQi = sbase + C::kOffQi, sK = sbase + C::kOffK, sC = sbase + C::kOffC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const int row = blockIdx.x;
  int b;
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const int n = abort ? 0 : row_window(a, row, &b);
  const int ntiles = (n + kIKeys - 1) / kIKeys;

  // ---- QI (zero-padded to 64 heads) and w into shared memory ----
  const T* qi = static_cast<const T*>(a.qi) + (size_t)row * a.Ni * kDi;
  uint8_t* gQi = smem_raw + C::kOffQi;
  for (int i = threadIdx.x; i < kNip * (kDi / 8); i += kIThreads) {
    const int g = i / (kDi / 8), d0 = (i % (kDi / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (g < a.Ni) v = *reinterpret_cast<const uint4*>(qi + (size_t)g * kDi + d0);
    *reinterpret_cast<uint4*>(gQi + (d0 / 64) * kNip * 128 + sw128_offset(g, (d0 % 64) / 8)) = v;
  }
  for (int g = threadIdx.x; g < kNip; g += kIThreads) {
    float wv = 0.f;
    if (g < a.Ni) {
      const size_t wi = (size_t)row * a.Ni + g;
      wv = a.w_dtype == DSA_DTYPE_FP32 ? __ldg(static_cast<const float*>(a.w) + wi)
           : a.w_dtype == DSA_DTYPE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.w)[wi])
                                          : __half2float(static_cast<const __half*>(a.w)[wi]);
    }
    bars.w[g] = wv;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars.rfull[s]), 1);
      mbar_init(smem_u32(&bars.rfree[s]), 4);
      mbar_init(smem_u32(&bars.cready[s]), 1);
      mbar_init(smem_u32(&bars.cfree[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars.dfull[s]), 1);
      mbar_init(smem_u32(&bars.dfree[s]), kIDrainWarps);
    }
    mbar_init(smem_u32(&bars.qdone), 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(&bars.tmem_slot), 512);
    tmem_relinquish<1>();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  // TMEM: R[2] at cols 0 / 64, dQI^T at 128, dKI tiles (double buffer) at 256 / 384
  const uint32_t tR = tmem, tQ = tmem + 128, tD = tmem + 256;
  bool failed = false;
  const int nsteps = 2 * ntiles;   // pass A then pass B, one KI tile per step

  if (warp == 0 || warp >= kIGather1) {
    // ---- KI tiles (TMA gather4), for both passes: 64 gathers per step (2 dim chunks x
    // 32 key groups), item i on gather warp i % 3, lane i / 3 ----
    const int lw = warp == 0 ? 0 : warp - kIGather1 + 1;
    const int item = lw + kIGathers * lane;
    const bool issuer = item < 2 * (kIKeys / 4);
    const int c = item / (kIKeys / 4), g = item % (kIKeys / 4);
    const int filler = key_row_of(a, b, row, 0);
    for (int j = 0; j < nsteps && !failed; ++j) {
      const int t = j % ntiles, s = j % STG;
      const int e0 = kIKeys * t + 4 * g;
      int rr[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        rr[e] = issuer && e0 + e < n ? key_row_of(a, b, row, e0 + e) : filler;
      mbar_wait(smem_u32(&bars.empty[s]), ((j / STG) & 1) ^ 1, a.err, &failed);
      failed = __any_sync(0xffffffffu, failed);
      if (failed) break;
      const uint32_t fb = smem_u32(&bars.full[s]);
      if (lw == 0 && lane == 0) mbar_arrive_expect_tx(fb, C::kStage);
      if (issuer)
        tma_gather4(sK + s * C::kStage + c * kIKeys * 128 + g * 512, &maps.ki, fb, 64 * c, rr[0],
                    rr[1], rr[2], rr[3]);
      __syncwarp();
    }
  } else if (warp == 1) {
    // (whole warp runs the loop, one elected lane issues; see the teacher kernel)
    if (ntiles > 0) {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id_r = idesc_f16(128, kNip, bf16, false, false);   // R = KI QI^T
      const uint32_t id_q = idesc_f16(128, kNip, bf16, true, true);     // dQI^T += KI^T C
      const uint32_t id_d = idesc_f16(128, kDi, bf16, false, true);     // dKI = C QI
      const uint64_t dqi_k = smem_desc_sw128(sQi, 16, 1024);
      const uint64_t dqi_mn = smem_desc_sw128(sQi, kNip * 128, 1024);
      for (int j = 0; j < nsteps && !failed; ++j) {
        const int t = j % ntiles, s = j % STG, rb = j & 1;
        const bool passB = j >= ntiles;
        if (j >= 2) mbar_wait_spin(smem_u32(&bars.rfree[rb]), ((j >> 1) - 1) & 1, a.err, &failed);
        mbar_wait_spin(smem_u32(&bars.full[s]), (j / STG) & 1, a.err, &failed);
        if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
        tc_fence_after();
        const uint64_t dk_k = smem_desc_sw128(sK + s * C::kStage, 16, 1024);
        if (elect_one()) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int u = 0; u < 4; ++u)
              umma_f16<1>(tR + 64 * rb, dk_k + (uint64_t)((c * kIKeys * 128 + u * 32) >> 4),
                          dqi_k + (uint64_t)((c * kNip * 128 + u * 32) >> 4), id_r, (c | u) != 0);
          umma_commit(smem_u32(&bars.rfull[rb]));
          if (!passB) umma_commit(smem_u32(&bars.empty[s]));
        }
        __syncwarp();
        if (!passB) continue;
        // pass B: wait for C of this tile, then dQI^T and dKI
        const int tb = t, cb = tb & 1;
        const int db = tb & 1;
        mbar_wait_spin(smem_u32(&bars.cready[cb]), (tb >> 1) & 1, a.err, &failed);
        if (tb >= 2) mbar_wait_spin(smem_u32(&bars.dfree[db]), ((tb >> 1) - 1) & 1, a.err, &failed);
        if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
        tc_fence_after();
        const uint64_t dc_k = smem_desc_sw128(sC + cb * C::kCBytes, 16, 1024);
        const uint64_t dc_mn = smem_desc_sw128(sC + cb * C::kCBytes, 16, 1024);
        const uint64_t dk_mn = smem_desc_sw128(sK + s * C::kStage, kIKeys * 128, 1024);
        if (elect_one()) {
#pragma unroll
          for (int part = 0; part < 2; ++part) {   // C = hi + lo
            const uint32_t po = part * kIKeys * 128;
#pragma unroll
            for (int k = 0; k < kIKeys / 16; ++k)   // K = keys
              umma_f16<1>(tQ, dk_mn + (uint64_t)((k * 2048) >> 4),
                          dc_mn + (uint64_t)((po + k * 2048) >> 4), id_q, (tb | k | part) != 0);
#pragma unroll
            for (int u = 0; u < kNip / 16; ++u)     // K = index heads
              umma_f16<1>(tD + 128 * db, dc_k + (uint64_t)((po + u * 32) >> 4),
                          dqi_mn + (uint64_t)((u * 2048) >> 4), id_d, (u | part) != 0);
          }
          umma_commit(smem_u32(&bars.empty[s]));
          umma_commit(smem_u32(&bars.cfree[cb]));
          umma_commit(smem_u32(&bars.dfull[db]));
        }
        __syncwarp();
      }
      if (!failed && elect_one()) umma_commit(smem_u32(&bars.qdone));
      __syncwarp();
    }
    __syncwarp();
  } else if (warp >= kIDrain0) {
    // ---- dKI drain: warp = (TMEM lane quadrant, 64-column half); thread = key row ----
    // Eight warps keep enough fp32 vector reductions in flight (one SM needs about 16 for
    // its share of the L2 reduction rate; four left the drain the slowest stage), and the
    // double-buffered TMEM tile lets the next tile's C and MMAs run meanwhile.
    const int qd = warp & 3, half = (warp - kIDrain0) >> 2;
    const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
    float* stage = reinterpret_cast<float*>(smem_raw + C::kOffStage) + (warp - kIDrain0) * 32 * 33;
    float* acc_out = a.dki_acc;
    // accumulator row of this thread's key in tile t (-1: none); the next tile's is loaded
    // while the current tile drains
    auto key_row = [&](int t) {
      const int my_key = kIKeys * t + 32 * qd + lane;
      return my_key < n ? key_row_of(a, b, row, my_key) : -1;
    };
    int next_row = ntiles > 0 ? key_row(0) : -1;
    for (int t = 0; t < ntiles; ++t) {
      const int db = t & 1;
      const int my_row = next_row;
      if (t + 1 < ntiles) next_row = key_row(t + 1);
      mbar_wait(smem_u32(&bars.dfull[db]), (t >> 1) & 1, a.err, &failed);
      const bool dfail = __any_sync(0xffffffffu, failed);
      tc_fence_after();
      if (!dfail) {
        for (int c0 = 64 * half; c0 < 64 * half + 64; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tD + 128 * db + lane_addr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) stage[lane * 33 + i] = __uint_as_float(r[i]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int kr = 4 * it + (lane >> 3), cc = 4 * (lane & 7);
            const int dst = __shfl_sync(0xffffffffu, my_row, kr);
            if (dst >= 0) {
              const float* sp = stage + kr * 33 + cc;
              asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                               acc_out + (size_t)dst * kDi + c0 + cc),
                           "f"(sp[0]), "f"(sp[1]), "f"(sp[2]), "f"(sp[3])
                           : "memory");
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars.dfree[db]));
    }
  } else {
    // ---- epilogue (128 threads, thread = key of the tile / dim of dQI) ----
    // TMEM lane quadrant of this warp; et = TMEM row (key of the tile / dim of dQI^T)
    const int qd = warp & 3, et = 32 * qd + lane;
    const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
    float* red = reinterpret_cast<float*>(smem_raw + C::kOffRed);
    float dw[kNip];
#pragma unroll
    for (int g = 0; g < kNip; ++g) dw[g] = 0.f;
    // ---------------- pass A: I ----------------
    for (int t = 0; t < ntiles; ++t) {
      const int rb = t & 1;
      mbar_wait(smem_u32(&bars.rfull[rb]), (t >> 1) & 1, a.err, &failed);
      const bool wfail = __any_sync(0xffffffffu, failed);
      tc_fence_after();
      float acc = 0.f;
      if (!wfail) {
        for (int g0 = 0; g0 < kNip; g0 += 32) {
          uint32_t r[32];
          tmem_ld32(tR + lane_addr + 64 * rb + g0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc = fmaf(bars.w[g0 + i], fmaxf(__uint_as_float(r[i]), 0.f), acc);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars.rfree[rb]));
      const int e = kIKeys * t + et;
      if (e < n) Ibuf[e] = acc;
    }
    named_bar(1, 128);
    // ---------------- softmax(I), dI, KL loss ----------------
    float mx = -INFINITY;
    for (int e = et; e < n; e += 128) mx = fmaxf(mx, Ibuf[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) bars.red[qd] = mx;
    named_bar(1, 128);
    mx = fmaxf(fmaxf(bars.red[0], bars.red[1]), fmaxf(bars.red[2], bars.red[3]));
    float sm = 0.f;
    for (int e = et; e < n; e += 128) sm += __expf(Ibuf[e] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    named_bar(1, 128);
    if (lane == 0) bars.red[qd] = sm;
    named_bar(1, 128);
    const float inv = 1.f / (bars.red[0] + bars.red[1] + bars.red[2] + bars.red[3] + kEps);
    const float* prow = a.p + (size_t)row * a.topk;
    float kl = 0.f;
    for (int e = et; e < n; e += 128) {
      const float si = __expf(Ibuf[e] - mx) * inv;
      const float pv = prow[e];
      const float pc = fmaxf(pv, kEps), sc = fmaxf(si, kEps);
      kl += pc * (__logf(pc) - __logf(sc));
      Ibuf[e] = si - pv;   // dI overwrites I
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kl += __shfl_xor_sync(0xffffffffu, kl, o);
    named_bar(1, 128);
    if (lane == 0) bars.red[4 + qd] = kl;
    named_bar(1, 128);
    if (et == 0 && n > 0) atomicAdd(a.loss, bars.red[4] + bars.red[5] + bars.red[6] + bars.red[7]);
    // ---------------- pass B: C, dW, dQI, dKI ----------------
    for (int t = 0; t < ntiles; ++t) {
      const int j = ntiles + t, rb = j & 1, cb = t & 1;
      mbar_wait(smem_u32(&bars.rfull[rb]), (j >> 1) & 1, a.err, &failed);
      if (t >= 2) mbar_wait(smem_u32(&bars.cfree[cb]), ((t >> 1) - 1) & 1, a.err, &failed);
      const bool wfail = __any_sync(0xffffffffu, failed);
      tc_fence_after();
      const int e = kIKeys * t + et;
      const float di = e < n ? Ibuf[e] : 0.f;
      uint8_t* crow = smem_raw + C::kOffC + cb * C::kCBytes + et * 128;
      for (int g0 = 0; g0 < kNip; g0 += 32) {
        uint32_t r[32];
        if (!wfail) {
          tmem_ld32(tR + lane_addr + 64 * rb + g0, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        uint32_t pk[16], pl[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float r0 = __uint_as_float(r[i]), r1 = __uint_as_float(r[i + 1]);
          dw[g0 + i] = fmaf(di, fmaxf(r0, 0.f), dw[g0 + i]);
          dw[g0 + i + 1] = fmaf(di, fmaxf(r1, 0.f), dw[g0 + i + 1]);
          const float c0 = r0 > 0.f ? di * bars.w[g0 + i] : 0.f;
          const float c1 = r1 > 0.f ? di * bars.w[g0 + i + 1] : 0.f;
          const uint32_t h = ElemTraits<T>::pack2(c0, c1);
          pk[i / 2] = h;
          const T* hh = reinterpret_cast<const T*>(&h);
          pl[i / 2] = ElemTraits<T>::pack2(c0 - ElemTraits<T>::to_f(hh[0]),
                                           c1 - ElemTraits<T>::to_f(hh[1]));
        }
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int chunk = g0 / 8 + v;
          *reinterpret_cast<uint4*>(crow + ((chunk ^ (et & 7)) << 4)) =
              make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          *reinterpret_cast<uint4*>(crow + kIKeys * 128 + ((chunk ^ (et & 7)) << 4)) =
              make_uint4(pl[4 * v], pl[4 * v + 1], pl[4 * v + 2], pl[4 * v + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar(1, 128);
      if (et == 0) mbar_arrive(smem_u32(&bars.cready[cb]));
      if (lane == 0) mbar_arrive(smem_u32(&bars.rfree[rb]));
    }
    // the last tile's MMAs are done: the key ring is free for the dW sums, dQI is final
    if (ntiles > 0) mbar_wait(smem_u32(&bars.qdone), 0, a.err, &failed);
    // ---------------- dW: column sums of the per-thread partials ----------------
    for (int g = 0; g < kNip; ++g) red[et * 65 + g] = dw[g];
    named_bar(1, 128);
    if (et < a.Ni) {
      float s = 0.f;
      for (int i = 0; i < 128; ++i) s += red[i * 65 + et];
      const size_t wi = (size_t)row * a.Ni + et;
      if (a.w_dtype == DSA_DTYPE_FP32) static_cast<float*>(a.dw)[wi] = s;
      else if (a.w_dtype == DSA_DTYPE_BF16) static_cast<__nv_bfloat16*>(a.dw)[wi] = __float2bfloat16_rn(s);
      else static_cast<__half*>(a.dw)[wi] = __float2half_rn(s);
    }
    // ---------------- dQI: TMEM lanes = dims, columns = index heads ----------------
    const bool qfail = ntiles == 0 || __any_sync(0xffffffffu, failed);
    tc_fence_after();
    T* dq = static_cast<T*>(a.dqi) + (size_t)row * a.Ni * kDi;
    for (int g0 = 0; g0 < kNip; g0 += 32) {
      uint32_t r[32];
      if (!qfail) {
        tmem_ld32(tQ + lane_addr + g0, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (g0 + i < a.Ni) dq[(size_t)(g0 + i) * kDi + et] = ElemTraits<T>::from_f(__uint_as_float(r[i]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc<1>(tmem, 512);
}

template <typename T>
__global__ void sli_cast_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = ElemTraits<T>::from_f(src[i]);
}

template <int D, typename T>
int launch(const DsaSliParams* p, cudaStream_t stream) {
  const bool bf16 = ElemTraits<T>::kIsBf16;
  Args a;
  a.q = p->query;
  a.qr = p->query_rope;
  a.k = p->key;
  a.kr = p->key_rope;
  a.qi = p->query_index;
  a.ki = p->key_index;
  a.w = p->weights;
  a.idx = p->sparse_indices;
  a.smax = p->softmax_max;
  a.ssum = p->softmax_sum;
  a.act_q = p->act_q;
  a.act_k = p->act_k;
  // the teacher distribution: a caller's (e.g. from the attention backward), else this
  // call's own teacher pass writes it into the workspace
  a.p = p->teacher ? const_cast<float*>(p->teacher) : static_cast<float*>(p->workspace);
  a.dqi = p->d_query_index;
  a.dki_acc = p->dki_acc;
  a.dw = p->d_weights;
  a.loss = p->loss;
  a.err = p->error_flag;
  a.rows = (int)(p->batch * p->s1);
  a.S1 = (int)p->s1;
  a.S2 = (int)p->s2;
  a.N1 = (int)p->n1;
  a.Ni = (int)p->n_index;
  a.topk = (int)p->topk;
  a.w_dtype = p->weights_dtype;
  a.scale = p->scale;
  const uint64_t qrows = (uint64_t)a.rows * p->n1;
  const uint64_t krows = (uint64_t)p->batch * p->s2;
  TMaps tm;
  IMaps im;
  if (!make_tmap_2d_16b(&tm.q, p->query, bf16, qrows, D, (uint64_t)D * 2, 64, 64) ||
      !make_tmap_2d_16b(&tm.qr, p->query_rope, bf16, qrows, 64, 128, 64, 64) ||
      !make_tmap_2d_16b(&tm.k, p->key, bf16, krows, D, (uint64_t)D * 2, 64, 1) ||
      !make_tmap_2d_16b(&tm.kr, p->key_rope, bf16, krows, 64, 128, 64, 1) ||
      !make_tmap_2d_16b(&im.ki, p->key_index, bf16, krows, kDi, kDi * 2, 64, 1))
    return DSA_ERR_TMA_DESCRIPTOR;
  // the index kernel keeps a row's topk scores in shared memory: three key stages when
  // they leave room, two otherwise (rows of up to 8192 entries); checked before any launch
  const int ipad = ((a.topk + 3) & ~3) * 4;
  const int ismem3 = ICfg<3>::kOffI + ipad + (int)sizeof(IBars<3>);
  const int ismem2 = ICfg<2>::kOffI + ipad + (int)sizeof(IBars<2>);
  if (ismem2 > 232448) return DSA_ERR_INVALID_ARG;
  if (cudaMemsetAsync(p->dki_acc, 0, sizeof(float) * krows * kDi, stream) != cudaSuccess ||
      cudaMemsetAsync(p->loss, 0, sizeof(float), stream) != cudaSuccess)
    return DSA_ERR_CUDA;
  if (!p->teacher) {
    auto k = sli_teacher_kernel<D, T>;
    const int smem = TCfg<D>::kOffBars + (int)sizeof(TBars);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    k<<<dim3(2 * (unsigned)a.rows), dim3(kTThreads), smem, stream>>>(tm, a);
  }
  {
    const bool three = ismem3 <= 232448;
    auto k = three ? sli_index_kernel<T, 3> : sli_index_kernel<T, 2>;
    const int smem = three ? ismem3 : ismem2;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    k<<<dim3((unsigned)a.rows), dim3(kIThreads), smem, stream>>>(im, a);
  }
  if (p->d_key_index) {
    const int64_t nk = (int64_t)krows * kDi;
    sli_cast_kernel<T><<<dim3((unsigned)((nk + 255) / 256)), dim3(256), 0, stream>>>(
        p->dki_acc, static_cast<T*>(p->d_key_index), nk);
  }
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

}  // namespace sli
}  // namespace dsa

extern "C" int64_t dsa_sli_workspace_size(int64_t batch, int64_t s1, int64_t topk) {
  if (batch < 0 || s1 < 0 || topk < 0) return -1;
  return 4 * batch * s1 * topk;
}

extern "C" int dsa_sli_grad(const DsaSliParams* p, void* stream_) {
  using namespace dsa::sli;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!p || !p->query || !p->key || !p->query_rope || !p->key_rope || !p->query_index ||
      !p->key_index || !p->weights || !p->sparse_indices || !p->softmax_max || !p->softmax_sum ||
      !p->act_q || !p->act_k || !p->d_query_index || !p->d_weights || !p->dki_acc || !p->loss ||
      (!p->workspace && !p->teacher))
    return DSA_ERR_INVALID_ARG;
  if (p->batch < 1 || p->s1 < 1 || p->s2 < 1 || p->n1 < 1 || p->n1 > 128 || p->n_index < 1 ||
      p->n_index > kNip || p->d_index != kDi || p->topk < 1 || p->topk > 8192)
    return DSA_ERR_INVALID_ARG;
  if (!p->teacher && p->workspace_bytes < dsa_sli_workspace_size(p->batch, p->s1, p->topk))
    return DSA_ERR_INVALID_ARG;
  const int D = (int)p->d;
  if (p->dtype == DSA_DTYPE_BF16) {
    if (D == 512) return launch<512, __nv_bfloat16>(p, stream);
    if (D == 256) return launch<256, __nv_bfloat16>(p, stream);
    if (D == 128) return launch<128, __nv_bfloat16>(p, stream);
  } else if (p->dtype == DSA_DTYPE_FP16) {
    if (D == 512) return launch<512, __half>(p, stream);
    if (D == 256) return launch<256, __half>(p, stream);
    if (D == 128) return launch<128, __half>(p, stream);
  }
  return DSA_ERR_INVALID_ARG;
}

// Cast of the fp32 dKeyIndex accumulator into the key_index dtype: the tail of dsa_sli_grad,
// for callers that pass d_key_index = NULL there and reduce dki_acc themselves first (query
// rows sharded across GPUs).
extern "C" int dsa_sli_cast(const DsaSliParams* p, void* stream_) {
  using namespace dsa::sli;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!p || !p->dki_acc || !p->d_key_index || p->batch < 1 || p->s2 < 1) return DSA_ERR_INVALID_ARG;
  const int64_t nk = p->batch * p->s2 * kDi;
  const dim3 grid((unsigned)((nk + 255) / 256));
  if (p->dtype == DSA_DTYPE_BF16)
    sli_cast_kernel<__nv_bfloat16><<<grid, dim3(256), 0, stream>>>(
        p->dki_acc, static_cast<__nv_bfloat16*>(p->d_key_index), nk);
  else if (p->dtype == DSA_DTYPE_FP16)
    sli_cast_kernel<__half><<<grid, dim3(256), 0, stream>>>(p->dki_acc, static_cast<__half*>(p->d_key_index), nk);
  else
    return DSA_ERR_INVALID_ARG;
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}
