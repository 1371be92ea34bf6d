// Sparse flash attention backward for sm_100a (tcgen05).
//
// Replaces the reference launch core `_sfa_grad_core` / `_sfa_grad_kernel`
// (sparse_flash_attention_grad_triton.py:158-308, :334-376).  Same math per query row
// (b, s1) and valid key u:
//   P[h,u]  = exp(scale*(q.k_u + qr.kr_u) - softmax_max[h]) / softmax_sum[h]  (sum<=0 -> 1)
//   dS[h,u] = P[h,u] * (dO[h].v_u - delta[h]) * scale,  delta[h] = dO[h].O[h],  v = k[:D]
//   dQ = dS K,  dQr = dS Kr,  dK += dS^T Q,  dKr += dS^T Qr,  dV += P^T dO
// P and dS are rounded to the input dtype before the three products, exactly where the
// reference kernel rounds them (`.to(k_full.dtype)`, :271-298).
//
// Four stages (the per-query working set -- Q, dO, dQ, 128 heads x 576 dims -- does not
// fit one SM, and the dK/dV products need the heads as their reduction dimension):
//   K1 probs : CTA pair per query row: S^T = K Q^T and dP^T = V dO^T on tcgen05 (2-SM,
//              M = 256 keys, 128 per CTA, N = 128 heads; one gathered key chunk feeds
//              both products), then P and dS -> key-major bf16 scratch [row][key][head].
//   K2 dq    : CTA pair per query row: dQ = dS K (nope dims split across the pair like
//              the forward's P V; rope dims on a padded N=128 MMA).
//   K3 dkv   : persistent; work items (query row, column part) walk the row's 128-key
//              tiles: dK^T = Q^T dS^T, dV^T = dO^T P^T, dKr^T = Qr^T dS^T on tcgen05
//              (M = 128 output columns, N = 128 keys, K = 128 heads), double-buffered in
//              TMEM and drained into fp32 accumulators with whole-row vector reductions
//              (red.global.add.v2.f32), the scatter-add of the reference (:289-300).
//              Adjacent rows share keys, so a pass after the compaction reorders their key
//              lists into runs of shared keys and K3 reduces a shared key once: groups of
//              four rows (two when key == value) on CTA pairs (sfa_bwd_group4_kernel,
//              sfa_bwd_dkv4_kernel) where their slices fit, else row pairs on single CTAs
//              (sfa_bwd_group_kernel, K3's grouped mode).
//   K4 cast  : fp32 accumulators -> key dtype (separate entry point so a multi-GPU
//              caller can all-reduce the fp32 accumulators first).

#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_b200.h"
#include "sfa_common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace dsa {
namespace sfa_bwd {

using namespace dsa::sfa;

constexpr int kTile = 64;       // keys per pair tile (K1, K2)
constexpr int kOwn = 32;        // keys per CTA in a QK^T B operand
constexpr int kHeads = 64;      // heads per CTA of a pair
constexpr int kChunk = kOwn * 128;   // one 64-dim chunk of 32 keys
constexpr int kHeadsPad = 128;  // heads per query row in the dS/P scratch
constexpr int kKeyTile3 = 128;  // keys per K3 CTA

struct Args {
  // index fields (see sfa_common.cuh)
  const int32_t* idx;
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  const int32_t* k_row_base;
  const int32_t* block_table;
  int num_rows, B, N1, topk, block, kv_rows, page, max_blocks, s2_cap, sparse_mode;
  float scale;
  const void* key;
  const void* key_rope;
  const void* dout;
  const void* out;
  const float* smax;
  const float* ssum;
  void* dq;
  void* dqr;
  float* dk_acc;
  float* dkr_acc;
  float* dv_acc;
  float* teacher;           // NULL or [num_rows][topk]: (1/N1) sum_h P of each valid entry (K1)
  const int32_t* ws_rows;
  const int32_t* ws_count;
  const int4* runs;  // NULL, or [num_rows / 2 rounded up][3] key runs of row pairs (K3 grouped)
  const int4* recs;  // NULL, or [groups][kRec4] records of the CTA-pair K3's row groups
  int16_t* orig;     // NULL, or [num_rows][topk]: a reordered slot's position in the compacted
                     // list (teacher with row groups: K1 writes the teacher there)
  void* ds;        // [num_rows][kp][128 heads] scratch (key-major), dtype of the inputs
  void* pp;        // [num_rows][kp][128 heads]
  const float* delta;   // [num_rows][N1] rowsum(dO * O), from sfa_bwd_delta_kernel
  int kp;          // key slots per row in the scratch (multiple of 256)
  int* err;
};

// bar.sync is the aligned form: the whole warp must arrive converged, so converge it first
// (a lane that left a wait early, e.g. after a timeout, rejoins here)
__device__ __forceinline__ void named_bar(int id, int n) {
  __syncwarp();
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// =====================================================================================
// K0: delta = rowsum(dO * O) per (query row, head), coalesced: one warp per head row
// =====================================================================================
template <int D, typename T>
__global__ void __launch_bounds__(256) sfa_bwd_delta_kernel(const T* __restrict__ dout,
                                                            const T* __restrict__ out,
                                                            float* __restrict__ delta, int64_t n) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const uint4* a = reinterpret_cast<const uint4*>(dout + w * D);
  const uint4* b = reinterpret_cast<const uint4*>(out + w * D);
  float acc = 0.f;
#pragma unroll
  for (int i = lane; i < D / 8; i += 32) {
    const uint4 u0 = __ldg(a + i), u1 = __ldg(b + i);
    const T* x0 = reinterpret_cast<const T*>(&u0);
    const T* x1 = reinterpret_cast<const T*>(&u1);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += ElemTraits<T>::to_f(x0[e]) * ElemTraits<T>::to_f(x1[e]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[w] = acc;
}

// =====================================================================================
// K1: probabilities and dS
// =====================================================================================
// One CTA pair per query row with the keys as the MMA's M dimension: a pair tile is 256
// keys (128 gathered by each CTA) and N = the 128 heads, so S^T = K Q^T and dP^T = V dO^T
// run at the full 2-SM rate (M = 256, N = 128) and both read the same gathered key chunk.
// Each CTA keeps its 64 heads of Q and dO resident as the B operands; the keys stream
// through a ring of 64-dim chunks (TMA gather4 in the 2-SM form).  In TMEM every CTA holds
// its 128 keys (lanes) x all 128 heads (columns), so P = exp(s scale - max_h) / sum_h and
// dS = P (dP - delta_h) scale need only per-head constants, no reduction across threads.
// P and dS go to the scratch key-major: [row][key][128 heads].
constexpr int kKeys1 = 128;     // keys per CTA per pair tile
constexpr int kStages1 = 5;     // key chunk ring (16 KB each)

template <int D>
struct Cfg1 {
  static constexpr int kNope = D / 64;
  static constexpr int kChunks = kNope + 1;
  static constexpr int kQBytes = kChunks * kHeads * 128;      // this CTA's 64 heads of Q
  static constexpr int kOBytes = kNope * kHeads * 128;        // and of dO
  static constexpr int kStage = kKeys1 * 128;                 // 128 keys x 64 dims
  static constexpr int kOffQ = 0;
  static constexpr int kOffO = kOffQ + kQBytes;
  static constexpr int kOffX = kOffO + kOBytes;
  static constexpr int kOffBars = kOffX + kStages1 * kStage;
};

struct Maps1 {
  CUtensorMap q, qr, dout, k, kr;
};

struct __align__(16) Bars1 {
  uint64_t q_full, full[kStages1], empty[kStages1], tfull[2], tfree[2];
  uint32_t tmem_slot;
  // per head: softmax_max * log2(e) (+inf for padded heads), 1 / softmax_sum (0 for padded
  // heads), rowsum(dO * O), unused -- one 16-byte broadcast load per head
  float4 hc[128];
};

constexpr int kElemWarps1 = 8;     // two per TMEM lane quadrant, 64 heads each
constexpr int kGatherWarp1 = 2 + kElemWarps1;
constexpr int kGatherWarps1 = 6;   // a thread issues one gather4 every ~100 cycles and the
                                   // lanes of a warp take turns: at most 6 gathers per warp
constexpr int kThreads1 = 32 * (kGatherWarp1 + kGatherWarps1);   // 0: Q/dO TMA, 1: MMA,
                                                                 // 2-9: elementwise, 10-15: keys

template <int D, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads1, 1)
    sfa_bwd_probs_kernel(const __grid_constant__ Maps1 maps, const Args a) {
  using C = Cfg1<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Bars1& bars = *reinterpret_cast<Bars1*>(smem_raw + C::kOffBars);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sQ = sbase + C::kOffQ, sO = sbase + C::kOffO, sX = sbase + C::kOffX;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const uint32_t cta = cluster_ctarank();
  const int row = blockIdx.x >> 1;
  const RowInfo ri = row_info(a, row);
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const int nvalid = (ri.active && !abort) ? __ldg(a.ws_count + row) : 0;
  const int ntiles = (nvalid + 2 * kKeys1 - 1) / (2 * kKeys1);
  const int nsteps = ntiles * C::kChunks;
  const int32_t* rows = a.ws_rows + (size_t)row * a.topk * a.block;

  for (int h = threadIdx.x; h < 128; h += kThreads1) {
    if (h < a.N1 && ntiles > 0) {
      const size_t hidx = (size_t)row * a.N1 + h;
      const float sm = __ldg(a.ssum + hidx);
      bars.hc[h] = make_float4(__ldg(a.smax + hidx) * 1.4426950408889634f, 1.f / (sm > 0.f ? sm : 1.f),
                               __ldg(a.delta + hidx), 0.f);
    } else {   // padded heads: exp2(s - inf) = 0, so P = dS = 0
      bars.hc[h] = make_float4(INFINITY, 0.f, 0.f, 0.f);
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars.q_full), 1);
    for (int s = 0; s < kStages1; ++s) {
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
    tmem_alloc<2>(smem_u32(&bars.tmem_slot), 512);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool failed = false;

  if (warp == 0) {
    // ---- Q and dO of this CTA's 64 heads (once) ----
    if (ntiles > 0) {
      const uint32_t lead = mapa_shared(smem_u32(&bars.q_full), 0);
      if (cta == 0 && lane == 0)
        mbar_arrive_expect_tx(smem_u32(&bars.q_full), 2 * (C::kQBytes + C::kOBytes));
      __syncwarp();
      const int qrow0 = row * a.N1 + kHeads * (int)cta;
      if (lane < C::kChunks) {
        const CUtensorMap* m = lane < C::kNope ? &maps.q : &maps.qr;
        tma_load_2d_pair(sQ + lane * kHeads * 128, m, lead, lane < C::kNope ? 64 * lane : 0, qrow0);
      } else if (lane < C::kChunks + C::kNope) {
        const int c = lane - C::kChunks;
        tma_load_2d_pair(sO + c * kHeads * 128, &maps.dout, lead, 64 * c, qrow0);
      }
    }
  } else if (warp >= kGatherWarp1) {
    // ---- the CTA's 128 keys of each tile, chunk by chunk (TMA gather4, 2-SM form):
    // key group g (keys 4g..4g+3) on gather warp g % W, lane g / W ----
    const int w = warp - kGatherWarp1;
    const int g = w + kGatherWarps1 * lane;
    const bool issuer = g < kKeys1 / 4;
    const int filler = nvalid > 0 ? __ldg(rows) : 0;
    int r4[4] = {0, 0, 0, 0};
    for (int j = 0; j < nsteps && !failed; ++j) {
      const int t = j / C::kChunks, c = j % C::kChunks, s = j % kStages1;
      if (c == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int e = 2 * kKeys1 * t + kKeys1 * (int)cta + 4 * g + q;
          r4[q] = issuer && e < nvalid ? __ldg(rows + e) : filler;
        }
      }
      mbar_wait(smem_u32(&bars.empty[s]), ((j / kStages1) & 1) ^ 1, a.err, &failed);
      if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
      const uint32_t full = smem_u32(&bars.full[s]);
      if (cta == 0 && w == 0 && lane == 0) mbar_arrive_expect_tx(full, 2 * C::kStage);
      if (issuer)
        tma_gather4_pair(sX + s * C::kStage + g * 512,
                         c < C::kNope ? &maps.k : &maps.kr, mapa_shared(full, 0),
                         c < C::kNope ? 64 * c : 0, r4[0], r4[1], r4[2], r4[3]);
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---- UMMA issue (pair leader): S^T and dP^T, M = 256 keys, N = 128 heads ----
    // The whole warp runs the loop (waits included); one elected lane issues each tcgen05
    // instruction (a lone lane issues MMAs much more slowly).
    if (cta == 0 && ntiles > 0) {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id = idesc_f16(256, 128, bf16, false, false);
      const uint64_t dq = smem_desc_sw128(sQ, 16, 1024);
      const uint64_t dd = smem_desc_sw128(sO, 16, 1024);
      const uint64_t dx0 = smem_desc_sw128(sX, 16, 1024);
      mbar_wait_spin(smem_u32(&bars.q_full), 0, a.err, &failed);
      for (int t = 0; t < ntiles && !failed; ++t) {
        const int b = t & 1;
        if (t >= 2)
          mbar_wait_spin(smem_u32(&bars.tfree[b]), (uint32_t)((t >> 1) - 1) & 1u, a.err, &failed, true);
        const uint32_t d_s = tmem + 256 * b, d_p = tmem + 256 * b + 128;
        for (int c = 0; c < C::kChunks; ++c) {
          const int j = t * C::kChunks + c, s = j % kStages1;
          mbar_wait_spin(smem_u32(&bars.full[s]), (uint32_t)(j / kStages1) & 1u, a.err, &failed, true);
          if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
          tc_fence_after();
          const uint64_t bx = dx0 + (uint64_t)((s * C::kStage) >> 4);
          if (elect_one()) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              umma_f16<2>(d_s, bx + (uint64_t)((u * 32) >> 4),
                          dq + (uint64_t)((c * kHeads * 128 + u * 32) >> 4), id, (c | u) != 0);
            if (c < C::kNope) {
#pragma unroll
              for (int u = 0; u < 4; ++u)
                umma_f16<2>(d_p, bx + (uint64_t)((u * 32) >> 4),
                            dd + (uint64_t)((c * kHeads * 128 + u * 32) >> 4), id, (c | u) != 0);
            }
            umma_commit_pair(smem_u32(&bars.empty[s]), 3);
          }
          __syncwarp();
        }
        if (failed) break;
        if (elect_one()) umma_commit_pair(smem_u32(&bars.tfull[b]), 3);
        __syncwarp();
      }
    }
    __syncwarp();
  } else {
    // ---- elementwise: thread = key (TMEM lane); warps 2-5 heads 0-63, warps 6-9 64-127 ----
    const int qd = warp & 3;
    const int hbase = 64 * ((warp - 2) >> 2);
    const int kk = 32 * qd + lane;
    const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
    const float c2 = a.scale * 1.4426950408889634f;
    const uint32_t lead_f0 = mapa_shared(smem_u32(&bars.tfree[0]), 0);
    const uint32_t lead_f1 = mapa_shared(smem_u32(&bars.tfree[1]), 0);
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1;
      mbar_wait(smem_u32(&bars.tfull[b]), (uint32_t)(t >> 1) & 1u, a.err, &failed);
      const bool wfail = __any_sync(0xffffffffu, failed);
      tc_fence_after();
      const int e = 2 * kKeys1 * t + kKeys1 * (int)cta + kk;   // key slot of the row
      const bool valid = e < nvalid;
      uint4* ds_row = reinterpret_cast<uint4*>(static_cast<T*>(a.ds) + ((size_t)row * a.kp + e) * kHeadsPad);
      uint4* p_row = reinterpret_cast<uint4*>(static_cast<T*>(a.pp) + ((size_t)row * a.kp + e) * kHeadsPad);
      float psum = 0.f;   // sum over this thread's 64 heads of P (fp32, before rounding)
#pragma unroll 1
      for (int h0 = hbase; h0 < hbase + 64; h0 += 16) {
        uint32_t sr[16], pr[16];
        if (!wfail) {
          tmem_ld16(tmem + lane_addr + 256 * b + h0, sr);
          tmem_ld16(tmem + lane_addr + 256 * b + 128 + h0, pr);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) sr[i] = pr[i] = 0u;
        }
        uint32_t pk_p[8], pk_s[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float p[2], g[2];
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const float4 hc = bars.hc[h0 + 2 * i + x];
            const float pe = valid ? ex2(fmaf(__uint_as_float(sr[2 * i + x]), c2, -hc.x)) * hc.y : 0.f;
            p[x] = pe;
            g[x] = valid ? pe * (__uint_as_float(pr[2 * i + x]) - hc.z) * a.scale : 0.f;
          }
          psum += p[0] + p[1];
          pk_p[i] = ElemTraits<T>::pack2(p[0], p[1]);
          pk_s[i] = ElemTraits<T>::pack2(g[0], g[1]);
        }
        // 16 heads of one key = one 32-byte sector (rows are 256 B, the scratch 256 B aligned)
        st_global_v8(ds_row + h0 / 8, pk_s);
        st_global_v8(p_row + h0 / 8, pk_p);
      }
      // the indexer loss's teacher: (1/N1) sum_h P; the two head halves of a key add theirs;
      // at the key's position in the compacted list (row groups reorder the list)
      if (a.teacher != nullptr && valid && !wfail) {
        const int eo = a.orig != nullptr ? (int)a.orig[(size_t)row * a.topk + e] : e;
        atomicAdd(a.teacher + (size_t)row * a.topk + eo, psum * (1.f / (float)a.N1));
      }
      tc_fence_before();
      named_bar(1, 32 * kElemWarps1);
      if (warp == 2 && lane == 0) mbar_arrive_cluster(b ? lead_f1 : lead_f0);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, 512);
}

// =====================================================================================
// K2: dQ = dS K, dQr = dS Kr
// =====================================================================================
template <int D>
struct Cfg2 {
  static constexpr int kNope = D / 64;
  static constexpr int kNPV = D < 256 ? D : 256;
  static constexpr int kNumPV = D / kNPV;
  static constexpr int kCpj = kNPV / 128;
  static constexpr int kSlots = kNope / 2;
  static constexpr int kABytes = kHeads * 128;               // dS tile: 64 heads x 64 keys
  static constexpr int kHHalf = kSlots * kChunk;
  static constexpr int kHNope = 2 * kHHalf;
  static constexpr int kRope = kTile * 128;                   // rope of all 64 keys
  static constexpr int kHBytes = kHNope + kRope;
  static constexpr int kOffA = 0;
  static constexpr int kOffH = kOffA + 2 * kABytes;
  static constexpr int kOffBars = kOffH + 2 * kHBytes;
  static constexpr int kTmemRope = D / 2;
};

struct Maps2 {
  CUtensorMap ds, k, kr;
};

struct __align__(16) Bars2 {
  uint64_t a_full[2], a_empty[2], h_full[2], h_empty[2], done;
  uint32_t tmem_slot;
};

constexpr int kGatherWarp0 = 6;
constexpr int kGatherWarps = 10;
constexpr int kThreads2 = 32 * (kGatherWarp0 + kGatherWarps);   // 0: dS tiles, 1: MMA,
                                                                 // 2-5: epilogue, 6-15: gathers

template <int D, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads2, 1)
    sfa_bwd_dq_kernel(const __grid_constant__ Maps2 maps, const Args a) {
  using C = Cfg2<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Bars2& bars = *reinterpret_cast<Bars2*>(smem_raw + C::kOffBars);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sA = sbase + C::kOffA, sH = sbase + C::kOffH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const uint32_t cta = cluster_ctarank();
  const int row = blockIdx.x >> 1;
  const RowInfo ri = row_info(a, row);
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const int nvalid = (ri.active && !abort) ? __ldg(a.ws_count + row) : 0;
  const int ntiles = (nvalid + kTile - 1) / kTile;
  const int32_t* rows = a.ws_rows + (size_t)row * a.topk * a.block;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars.a_full[s]), 1);
      mbar_init(smem_u32(&bars.a_empty[s]), 1);
      mbar_init(smem_u32(&bars.h_full[s]), 1);
      mbar_init(smem_u32(&bars.h_empty[s]), 1);
    }
    mbar_init(smem_u32(&bars.done), 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(smem_u32(&bars.tmem_slot), 512);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool failed = false;

  if (warp == 0) {
    // ---- dS tiles of this CTA's 64 heads ----
    if (lane == 0) {
      for (int t = 0; t < ntiles && !failed; ++t) {
        const int s = t & 1;
        if (!mbar_wait(smem_u32(&bars.a_empty[s]), ((t >> 1) & 1) ^ 1, a.err, &failed)) break;
        const uint32_t lead = mapa_shared(smem_u32(&bars.a_full[s]), 0);
        if (cta == 0) mbar_arrive_expect_tx(smem_u32(&bars.a_full[s]), 2 * C::kABytes);
        // key-major scratch: box of 64 heads (this CTA's) x 64 keys -> A is MN-major
        tma_load_2d_pair(sA + s * C::kABytes, &maps.ds, lead, kHeads * (int)cta,
                         row * a.kp + kTile * t);
      }
    }
    __syncwarp();
  } else if (warp >= kGatherWarp0) {
    // ---- V slices of all 64 keys (+ rope of all keys in the leader), TMA gather4 ----
    // Items: 16 key groups x kSlots chunks, then (leader) 16 rope groups; item i goes to
    // gather warp i % kGatherWarps, lane i / kGatherWarps (at most 8 per warp: a thread
    // issues one gather4 every ~100 cycles and the lanes of a warp take turns).
    const int lw = warp - kGatherWarp0;
    const int nitems = 16 * C::kSlots + (cta == 0 ? 16 : 0);
    const int item = lw + kGatherWarps * lane;
    const bool rope_item = item >= 16 * C::kSlots;
    const int g = rope_item ? item - 16 * C::kSlots : item & 15;   // key group: keys 4g..4g+3
    const int filler = nvalid > 0 ? __ldg(rows) : 0;
    uint32_t dst_off = C::kHNope + g * 512;
    int x = 0;
    if (!rope_item) {
      const int sl = item >> 4;
      const int j = sl / C::kCpj;
      const int chunk = j * 2 * C::kCpj + (int)cta * C::kCpj + sl % C::kCpj;
      dst_off = (g >> 3) * C::kHHalf + sl * kChunk + (g & 7) * 512;
      x = 64 * chunk;
    }
    for (int t = 0; t < ntiles && !failed; ++t) {
      const int s = t & 1;
      int r[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int jj = kTile * t + 4 * g + e;
        r[e] = item < nitems && jj < nvalid ? __ldg(rows + jj) : filler;
      }
      mbar_wait(smem_u32(&bars.h_empty[s]), ((t >> 1) & 1) ^ 1, a.err, &failed);
      failed = __any_sync(0xffffffffu, failed);
      if (failed) break;
      const uint32_t lead = mapa_shared(smem_u32(&bars.h_full[s]), 0);
      if (lw == 0 && cta == 0 && lane == 0)
        mbar_arrive_expect_tx(smem_u32(&bars.h_full[s]), 2 * C::kHNope + C::kRope);
      if (item < nitems)
        tma_gather4_pair(sH + s * C::kHBytes + dst_off, rope_item ? &maps.kr : &maps.k, lead, x,
                         r[0], r[1], r[2], r[3]);
      __syncwarp();
    }
  } else if (warp == 1) {
    // (whole warp runs the loop, one elected lane issues; see K1)
    if (cta == 0 && ntiles > 0) {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id_n = idesc_f16(128, C::kNPV, bf16, true, true);
      const uint32_t id_r = idesc_f16(128, 128, bf16, true, true);
      const uint64_t da0 = smem_desc_sw128(sA, kHeads * 128, 1024);
      const uint64_t da1 = smem_desc_sw128(sA + C::kABytes, kHeads * 128, 1024);
      const uint64_t dh0 = smem_desc_sw128(sH, kChunk, 1024);
      const uint64_t dh1 = smem_desc_sw128(sH + C::kHBytes, kChunk, 1024);
      for (int t = 0; t < ntiles && !failed; ++t) {
        const int s = t & 1;
        mbar_wait_spin(smem_u32(&bars.a_full[s]), (t >> 1) & 1, a.err, &failed);
        mbar_wait_spin(smem_u32(&bars.h_full[s]), (t >> 1) & 1, a.err, &failed);
        if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
        tc_fence_after();
        const uint64_t ba = s ? da1 : da0, bh = s ? dh1 : dh0;
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < C::kNumPV; ++j)
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k)
              umma_f16<2>(tmem + j * (C::kNPV / 2), ba + (uint64_t)((k * 2048) >> 4),
                          bh + (uint64_t)(((k >> 1) * C::kHHalf + j * C::kCpj * kChunk + (k & 1) * 2048) >> 4),
                          id_n, (t | k) != 0);
          // rope: N=128 with the leader's B half holding the 64 rope dims; the other half
          // is never read back (it lands in TMEM lanes 64-127)
#pragma unroll
          for (int k = 0; k < kTile / 16; ++k)
            umma_f16<2>(tmem + C::kTmemRope, ba + (uint64_t)((k * 2048) >> 4),
                        bh + (uint64_t)((C::kHNope + k * 2048) >> 4), id_r, (t | k) != 0);
          umma_commit_pair(smem_u32(&bars.a_empty[s]), 3);
          umma_commit_pair(smem_u32(&bars.h_empty[s]), 3);
        }
        __syncwarp();
      }
      if (!failed && elect_one()) umma_commit_pair(smem_u32(&bars.done), 3);
      __syncwarp();
    }
    __syncwarp();
  } else {
    // ---- epilogue: dQ, dQr (both CTAs) ----
    const int q = warp & 3;
    const int hrow = 32 * (q & 1) + lane;
    const int half = q >> 1;
    const int head = kHeads * (int)cta + hrow;
    const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
    if (ntiles > 0) mbar_wait(smem_u32(&bars.done), 0, a.err, &failed);
    const bool read = ntiles > 0 && !__any_sync(0xffffffffu, failed);
    tc_fence_after();
    T* qrow = reinterpret_cast<T*>(a.dq) + ((size_t)row * a.N1 + min(head, a.N1 - 1)) * D;
    for (int j = 0; j < C::kNumPV; ++j) {
      const int dbase = j * C::kNPV + half * (C::kNPV / 2);
      for (int cc = 0; cc < C::kNPV / 2; cc += 32) {
        uint32_t o[32];
        if (read) {
          tmem_ld32(tmem + lane_addr + j * (C::kNPV / 2) + cc, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (head < a.N1) {
          uint4* dst = reinterpret_cast<uint4*>(qrow + dbase + cc);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 0]), __uint_as_float(o[8 * v + 1]));
            w.y = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 2]), __uint_as_float(o[8 * v + 3]));
            w.z = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 4]), __uint_as_float(o[8 * v + 5]));
            w.w = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 6]), __uint_as_float(o[8 * v + 7]));
            dst[v] = w;
          }
        }
      }
    }
    if (half == 0) {   // lanes 0-63 of the rope accumulator hold dQr of the CTA's heads
      T* rrow = reinterpret_cast<T*>(a.dqr) + ((size_t)row * a.N1 + min(head, a.N1 - 1)) * 64;
      for (int cc = 0; cc < 64; cc += 32) {
        uint32_t o[32];
        if (read) {
          tmem_ld32(tmem + lane_addr + C::kTmemRope + cc, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (head < a.N1) {
          uint4* dst = reinterpret_cast<uint4*>(rrow + cc);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 0]), __uint_as_float(o[8 * v + 1]));
            w.y = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 2]), __uint_as_float(o[8 * v + 3]));
            w.z = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 4]), __uint_as_float(o[8 * v + 5]));
            w.w = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 6]), __uint_as_float(o[8 * v + 7]));
            dst[v] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, 512);
}

// =====================================================================================
// Row pairs for K3.  Adjacent query rows share many keys (a causal top-k picks from nearly
// the same window), and K3 reduces every (row, key) product into the key's fp32 accumulator
// row.  Grouped, the two rows' products for a shared key are summed in TMEM first (one GEMM
// with K = 2 x 128 heads) and reach L2 once.  This pass reorders each row's compacted key
// list into runs -- keys of row 0 only, keys of both rows, keys of row 1 only -- with the
// shared run listed in the same order in both rows, so that the run's dS / P slots are
// consecutive in either row's scratch and a K3 tile of it is one TMA box per row.  K1 and
// K2 take the list in any order.
// One CTA per pair: a shared-memory hash set of the pair's keys (open addressing) marks each
// key with the rows that hold it; block scans over the two lists then rank the keys of each
// run in list order: row 0's keys keep row 0's order (own run, then shared run), row 1 lists
// the shared run in row 0's order and then its own keys in its own order.  The result
// depends only on the two lists (not on which thread won a hash slot), so a call is
// reproducible and a call over a row range that starts on an even row orders every pair as
// the whole call does.  A pair with an empty row, or whose lists hold a key twice, keeps its
// order and is described as two unshared runs.
// runs[pair][r] = (mask of member rows, length, first slot in row 0, first slot in row 1),
// in the order K3 walks them: row 0 only, shared, row 1 only.
// =====================================================================================
constexpr int kGroupThreads = 512;

__device__ __forceinline__ uint32_t group_hash(int k, int lg) {
  return ((uint32_t)k * 2654435761u) >> (32 - lg);
}

// shared memory of one pair: keys [H], words [H] (member mask | shared rank << 2), and the
// table slot of every list entry [H / 2]
inline int group_smem_bytes(int lg) { return 10 << lg; }

__global__ void __launch_bounds__(kGroupThreads) sfa_bwd_group_kernel(const Args a,
                                                                      int32_t* ws_rows,
                                                                      int4* runs, int lg) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t warp_sum[kGroupThreads / 32];
  __shared__ int dup;
  const int H = 1 << lg;   // >= 2 x the pair's keys: the probe loops end
  int* keys = reinterpret_cast<int*>(smem_raw);
  uint32_t* word = reinterpret_cast<uint32_t*>(keys + H);
  int* slot_of = reinterpret_cast<int*>(word + H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = 2 * blockIdx.x, r1 = r0 + 1;
  const size_t nent = (size_t)a.topk * a.block;
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  auto count = [&](int r) {
    if (r >= a.num_rows || abort) return 0;
    const RowInfo ri = row_info(a, r);
    return ri.active ? __ldg(a.ws_count + r) : 0;
  };
  const int n0 = count(r0), n1 = count(r1);
  int4* out = runs + 3 * blockIdx.x;
  auto unshared = [&]() {
    if (threadIdx.x == 0) {
      out[0] = make_int4(1, n0, 0, 0);
      out[1] = make_int4(3, 0, 0, 0);
      out[2] = make_int4(2, n1, 0, 0);
    }
  };
  if (n0 == 0 || n1 == 0 || 2 * (n0 + n1) > H) {   // uniform over the block
    unshared();
    return;
  }
  for (int i = threadIdx.x; i < H; i += kGroupThreads) {
    keys[i] = -1;
    word[i] = 0u;
  }
  if (threadIdx.x == 0) dup = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n0 + n1; i += kGroupThreads) {
    const int g = i >= n0;
    const int k = ws_rows[(size_t)(g ? r1 : r0) * nent + (g ? i - n0 : i)];
    uint32_t h = group_hash(k, lg);
    for (int probe = 0; probe < H; ++probe) {
      const int prev = atomicCAS(&keys[h], -1, k);
      if (prev == -1 || prev == k) {
        if (atomicOr(&word[h], 1u << g) & (1u << g)) dup = 1;   // listed twice in row g
        slot_of[i] = (int)h;
        break;
      }
      h = (h + 1) & (uint32_t)(H - 1);
    }
  }
  __syncthreads();
  if (dup) {   // uniform: read after the barrier
    unshared();
    return;
  }
  // each thread ranks a contiguous chunk of either list; counts in 16-bit fields: row 0's
  // own keys (0), row 0's shared keys (1), row 1's own keys (2), each at most 4096
  const int p0 = (n0 + kGroupThreads - 1) / kGroupThreads;
  const int p1 = (n1 + kGroupThreads - 1) / kGroupThreads;
  const int i0 = min(n0, (int)threadIdx.x * p0), i1 = min(n0, i0 + p0);
  const int j0 = min(n1, (int)threadIdx.x * p1), j1 = min(n1, j0 + p1);
  uint64_t c = 0;
  for (int i = i0; i < i1; ++i) c += (word[slot_of[i]] & 3u) == 1u ? 1ull : 1ull << 16;
  for (int j = j0; j < j1; ++j)
    if ((word[slot_of[n0 + j]] & 3u) == 2u) c += 1ull << 32;
  uint64_t v = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) warp_sum[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint64_t w = lane < kGroupThreads / 32 ? warp_sum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kGroupThreads / 32) warp_sum[lane] = w;
  }
  __syncthreads();
  uint64_t e = v - c + (warp > 0 ? warp_sum[warp - 1] : 0);
  const uint64_t tot = warp_sum[kGroupThreads / 32 - 1];
  const int c1 = (int)(tot & 0xffff), c3 = (int)((tot >> 16) & 0xffff), c2 = (int)(tot >> 32);
  // every list entry was read into the table above, so the lists are rewritten in place
  for (int i = i0; i < i1; ++i) {
    const int h = slot_of[i];
    const uint32_t w = word[h];
    int pos;
    if ((w & 3u) == 1u) {
      pos = (int)(e & 0xffff);
      e += 1;
    } else {
      const int r = (int)((e >> 16) & 0xffff);
      pos = c1 + r;
      e += 1ull << 16;
      word[h] = w | ((uint32_t)r << 2);   // row 1 places the key at the same rank
    }
    ws_rows[(size_t)r0 * nent + pos] = keys[h];
  }
  __syncthreads();
  for (int j = j0; j < j1; ++j) {
    const int h = slot_of[n0 + j];
    const uint32_t w = word[h];
    int pos;
    if ((w & 3u) == 2u) {
      pos = c3 + (int)((e >> 32) & 0xffff);
      e += 1ull << 32;
    } else {
      pos = (int)(w >> 2);
    }
    ws_rows[(size_t)r1 * nent + pos] = keys[h];
  }
  if (threadIdx.x == 0) {
    out[0] = make_int4(1, c1, 0, 0);
    out[1] = make_int4(3, c3, c1, 0);
    out[2] = make_int4(2, c2, 0, c3);
  }
}

// =====================================================================================
// K3: dK = dS^T Q, dV = P^T dO, dKr = dS^T Qr  (scatter-add into fp32)
// =====================================================================================
// Work items are (query row, part) pairs.  Parts split the output columns so that a part's
// slice of the row's Q / dO / Qr (K = 128 heads) is loaded once per item: for D = 512,
// parts 0-1 are dK columns [0,256) and [256,512) (Q slice, dS tiles), parts 2-3 the same
// columns of dV (dO slice, P tiles) and part 4 is dKr (Qr, dS tiles).  The kernel is
// persistent (one CTA per SM, items strided by the grid; the parts of one row are
// adjacent items, so they run together and their dS / P tiles are read from L2).
//
// Per 128-key tile it computes the transposed products, dK^T = Q^T dS^T and so on:
// M = 128 output columns (TMEM lanes), N = 128 keys (TMEM columns), K = 128 heads.  With
// one output column per lane, a warp holds 32 consecutive columns of every key; one
// shuffle per key pair turns that into two whole 128-byte rows per
// red.global.add.v2.f32 (even lanes carry key 2j, odd lanes key 2j+1).  That reduction
// form runs at the L2 reduction ceiling, and no shared-memory transpose is needed.
// The reductions are the bound (4352 bytes per valid pair at D = 512).
//
// Merged key gradient (dv_acc == NULL): key and value are one tensor (MLA), so the caller
// wants dK + dV only.  A merged part takes both slots, the Q slice and the dO slice of its
// columns, and each tile runs dS^T Q and then P^T dO into the same TMEM accumulator (two
// B-ring entries: the dS tile, then the P tile).  Parts per row: D / 256 merged + the
// rope part; the reductions drop to 4 (D + 64) bytes per valid pair.
//
// Grouped mode (runs != NULL, 5-output calls): an item is a pair of adjacent rows and a part,
// and its tiles walk the pair's three key runs (sfa_bwd_group_kernel).  Slot g holds row g's
// slice; a tile of the shared run takes two B entries, row 0's dS (or P) tile and then row
// 1's, into one TMEM accumulator, so a shared key is reduced once for both rows.  A slot is
// released after the last tile that reads it, so the next item's row-0 slice loads while
// the row-1-only run still runs.
//
// Roles: warp 0 (one lane) loads the item slices into two slots and the dS / P tiles
// through a 3-stage ring, so the next item's slice arrives while the current item's last
// tiles run; warp 1 (one lane) issues the MMAs into two TMEM buffers; warps 2-17 drain
// a finished buffer (4 warps per TMEM lane quadrant, each owning a quarter of its columns)
// while the MMAs of the next tile run.
constexpr int kStages3 = 3;

template <int D>
struct Cfg3 {
  static constexpr int kW = D < 256 ? D : 256;              // output columns per part
  static constexpr int kDParts = D / kW;
  static constexpr int kParts = 2 * kDParts + 1;
  static constexpr int kBox = 128 * 128;                    // 64 columns x 128 heads, MN-major
  static constexpr int kSlice = (kW / 64) * kBox;           // one slot: a part's slice
  static constexpr int kTileB = kHeadsPad * kKeyTile3 * 2;  // 128 keys x 128 heads, K-major
  static constexpr int kOffA = 0;
  static constexpr int kOffB = 2 * kSlice;
  static constexpr int kOffBars = kOffB + kStages3 * kTileB;
};

struct Maps3 {
  CUtensorMap ds, pp, q, qr, dout;
};

struct __align__(16) Bars3 {
  uint64_t a_full[2], a_empty[2];
  uint64_t b_full[kStages3], b_empty[kStages3];
  uint64_t t_full[2], t_empty[2];
  uint32_t tmem_slot;
};

constexpr int kThreads3 = 18 * 32;   // warp 0: TMA, 1: MMA, 2-17: drain

// One K3 work item: a query row (or, grouped, a row pair) and a column part.  Its keys come
// as up to three runs (mask of member rows, length, first slot in row 0, in row 1); a
// single row is one run of all its keys.  Every role walks the same sequence.
struct Item3 {
  int row0, part, ntiles;
  int4 r0, r1, r2;   // the runs in walking order
};

__device__ __forceinline__ int tiles3(int len) { return (len + kKeyTile3 - 1) / kKeyTile3; }

// work items of a call: (rows, or row pairs) x parts
__device__ __forceinline__ int groups3(const Args& a) {
  return a.runs != nullptr ? (a.num_rows + 1) / 2 : a.num_rows;
}

template <int D>
__device__ __forceinline__ Item3 item3(const Args& a, int it, int nparts) {
  Item3 x;
  const int g = it / nparts;
  x.part = it % nparts;
  if (a.runs != nullptr) {
    x.row0 = 2 * g;
    x.r0 = __ldg(a.runs + 3 * g);
    x.r1 = __ldg(a.runs + 3 * g + 1);
    x.r2 = __ldg(a.runs + 3 * g + 2);
  } else {
    x.row0 = g;
    const RowInfo ri = row_info(a, g);
    x.r0 = make_int4(1, ri.active ? __ldg(a.ws_count + g) : 0, 0, 0);
    x.r1 = x.r2 = make_int4(0, 0, 0, 0);
  }
  x.ntiles = tiles3(x.r0.y) + tiles3(x.r1.y) + tiles3(x.r2.y);
  return x;
}

// Tile t of an item: member rows, keys (<= 128) and first slot in row 0 / row 1
struct Tile3 {
  int mask, len, off0, off1;
};

__device__ __forceinline__ Tile3 tile3(const Item3& x, int t) {
  const int n0 = tiles3(x.r0.y), n1 = tiles3(x.r1.y);
  const bool in2 = t >= n0 + n1, in1 = !in2 && t >= n0;
  t -= in2 ? n0 + n1 : in1 ? n0 : 0;
  Tile3 y;
  y.mask = in2 ? x.r2.x : in1 ? x.r1.x : x.r0.x;
  y.len = min(kKeyTile3, (in2 ? x.r2.y : in1 ? x.r1.y : x.r0.y) - kKeyTile3 * t);
  y.off0 = (in2 ? x.r2.z : in1 ? x.r1.z : x.r0.z) + kKeyTile3 * t;
  y.off1 = (in2 ? x.r2.w : in1 ? x.r1.w : x.r0.w) + kKeyTile3 * t;
  return y;
}

// Grouped mode: the last tile of the item that reads row g (-1: the row has no keys)
__device__ __forceinline__ int last_tile3(const Item3& x, int g) {
  int end = tiles3(x.r0.y), last = ((x.r0.x >> g) & 1) && x.r0.y > 0 ? end - 1 : -1;
  end += tiles3(x.r1.y);
  if (((x.r1.x >> g) & 1) && x.r1.y > 0) last = end - 1;
  end += tiles3(x.r2.y);
  if (((x.r2.x >> g) & 1) && x.r2.y > 0) last = end - 1;
  return last;
}

// The B entries of a tile: A slot, first scratch row (key slot) of the 128-key box, P or dS.
struct Entry3 {
  int slot, srow;
  bool p;
};

__device__ __forceinline__ int entries3(const Args& a, const Item3& x, const Tile3& y, bool mixed,
                                        bool is_dv, int ab1, Entry3 (&en)[2]) {
  if (mixed) {   // merged part: the dS tile (slot 0, Q), then the P tile (slot 1, dO)
    en[0] = {0, x.row0 * a.kp + y.off0, false};
    en[1] = {1, x.row0 * a.kp + y.off0, true};
    return 2;
  }
  if (a.runs == nullptr) {
    en[0] = {ab1, x.row0 * a.kp + y.off0, is_dv};
    return 1;
  }
  const Entry3 e1 = {1, (x.row0 + 1) * a.kp + y.off1, is_dv};
  en[0] = (y.mask & 1) ? Entry3{0, x.row0 * a.kp + y.off0, is_dv} : e1;
  en[1] = e1;
  return (y.mask & 1) + ((y.mask >> 1) & 1);
}

// The A slots an item loads (bit s: slot s) and, per slot, its last reading tile.
__device__ __forceinline__ int slots3(const Args& a, const Item3& x, bool mixed, int ab1,
                                      int (&last)[2]) {
  last[0] = last[1] = x.ntiles - 1;
  if (mixed) return 3;
  if (a.runs == nullptr) return 1 << ab1;
  last[0] = last_tile3(x, 0);
  last[1] = last_tile3(x, 1);
  return (last[0] >= 0 ? 1 : 0) | (last[1] >= 0 ? 2 : 0);
}

// What a part computes: rope (dKr: Qr and dS), dK (Q, dS), dV (dO, P) or, merged, dK + dV
// of its columns (Q and dS, then dO and P).
struct Part3 {
  bool rope, is_dv, mixed;
  int col0, nbox;
};

template <int D>
__device__ __forceinline__ Part3 part3(int part, bool merged) {
  using C = Cfg3<D>;
  Part3 k;
  k.rope = part == (merged ? C::kDParts : 2 * C::kDParts);
  k.mixed = merged && !k.rope;
  k.is_dv = !merged && !k.rope && part >= C::kDParts;
  k.col0 = k.rope ? 0 : (part % C::kDParts) * C::kW;
  k.nbox = k.rope ? 1 : C::kW / 64;
  return k;
}

// One drain warp's share of a finished tile: NK keys (TMEM columns) x 32 output columns
// (its TMEM lanes), read 16 keys at a time; the buffer is released after the last read
// (the MMAs of the next tile go to the other buffer, and the drain is the slower side).
// Lane l holds column c0 + l of every key; for keys (2j, 2j+1) the lanes swap one value
// with their neighbour so that even lanes hold columns (l, l+1) of key 2j and odd lanes
// columns (l-1, l) of key 2j+1: each red.v2 then covers two whole 128-byte rows.
// rows[i]: accumulator row of key 32i + l of the share (-1 = no key).  kCluster: `t_empty`
// is a cluster-window address (the pair leader's barrier); the arrive is relaxed, because it
// only has to follow the warp's completed TMEM reads (a cluster-scope release would wait for
// the warp's reductions in flight to reach L2).
template <int NK, bool kCluster = false>
__device__ __forceinline__ void dkv_drain(uint32_t taddr, uint32_t t_empty, bool lanes_ok,
                                          float* gcol, int ld, const int (&rows)[NK / 32],
                                          int lane) {
  const int odd = lane & 1;
#pragma unroll
  for (int h = 0; h < NK / 16; ++h) {
    uint32_t r[16];
    if (lanes_ok) {
      tmem_ld16(taddr + 16 * h, r);
      tmem_ld_wait();
    }
    if (h == NK / 16 - 1) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kCluster)
          mbar_arrive_cluster_relaxed(t_empty);
        else
          mbar_arrive(t_empty);
      }
    }
    if (!lanes_ok) continue;
    // all exchanges first (independent shuffles in flight), then the reductions back to back
    int dst_row[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x0 = __uint_as_float(r[2 * j]), x1 = __uint_as_float(r[2 * j + 1]);
      const float recv = __shfl_xor_sync(0xffffffffu, odd ? x0 : x1, 1);
      r[2 * j] = __float_as_uint(odd ? recv : x0);
      r[2 * j + 1] = __float_as_uint(odd ? x1 : recv);
      dst_row[j] = __shfl_sync(0xffffffffu, rows[h >> 1], 16 * (h & 1) + 2 * j + odd);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (dst_row[j] >= 0) {
        float* gp = gcol + (size_t)dst_row[j] * ld;
        asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(gp),
                     "f"(__uint_as_float(r[2 * j])), "f"(__uint_as_float(r[2 * j + 1]))
                     : "memory");
      }
    }
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads3, 1)
    sfa_bwd_dkv_kernel(const __grid_constant__ Maps3 maps, const Args a) {
  using C = Cfg3<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Bars3& bars = *reinterpret_cast<Bars3*>(smem_raw + C::kOffBars);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sA = sbase + C::kOffA, sB = sbase + C::kOffB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  // uniform across the CTA: an error flagged by an earlier kernel skips the work
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const bool merged = a.dv_acc == nullptr;
  const int nparts = merged ? C::kDParts + 1 : C::kParts;
  const int nitems = abort ? 0 : groups3(a) * nparts;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars.a_full[s]), 1);
      mbar_init(smem_u32(&bars.a_empty[s]), 1);
      mbar_init(smem_u32(&bars.t_full[s]), 1);
      mbar_init(smem_u32(&bars.t_empty[s]), 16);
    }
    for (int s = 0; s < kStages3; ++s) {
      mbar_init(smem_u32(&bars.b_full[s]), 1);
      mbar_init(smem_u32(&bars.b_empty[s]), 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(&bars.tmem_slot), 512);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool failed = false;

  if (warp == 0) {
    // ---- TMA: item slices (2 slots), dS / P tiles (ring) ----
    if (lane == 0) {
      int ua0 = 0, ua1 = 0, nb = 0, ni = 0;   // loads per A slot, B entries, non-empty items
      for (int it = blockIdx.x; it < nitems && !failed; it += gridDim.x) {
        const Item3 x = item3<D>(a, it, nparts);
        if (x.ntiles == 0) continue;
        const Part3 pk = part3<D>(x.part, merged);
        // slots: a merged part fills both (Q, dO); a grouped item one per member row with
        // keys; otherwise one, alternating per item
        const int ab1 = merged ? 0 : (ni & 1);
        int last[2];
        const int used = slots3(a, x, pk.mixed, ab1, last);
        for (int ab = 0; ab < 2; ++ab) {
          if (!((used >> ab) & 1)) continue;
          const CUtensorMap* am = pk.rope ? &maps.qr
                                  : (pk.is_dv || (pk.mixed && ab == 1)) ? &maps.dout : &maps.q;
          const int qrow = x.row0 + (a.runs != nullptr ? ab : 0);
          if (!mbar_wait_sleep(smem_u32(&bars.a_empty[ab]), ((ab ? ua1 : ua0) & 1) ^ 1, a.err, &failed))
            break;
          const uint32_t fb = smem_u32(&bars.a_full[ab]);
          mbar_arrive_expect_tx(fb, pk.nbox * C::kBox);
          for (int c = 0; c < pk.nbox; ++c)
            tma_load_2d(sA + ab * C::kSlice + c * C::kBox, am, fb, pk.col0 + 64 * c, qrow * a.N1);
          if (ab) ++ua1; else ++ua0;
        }
        if (failed) break;
        for (int t = 0; t < x.ntiles && !failed; ++t) {
          Entry3 en[2];
          const int ne = entries3(a, x, tile3(x, t), pk.mixed, pk.is_dv, ab1, en);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (e >= ne) break;
            const CUtensorMap* bm = en[e].p ? &maps.pp : &maps.ds;
            const int s = nb % kStages3;
            if (!mbar_wait_sleep(smem_u32(&bars.b_empty[s]), ((nb / kStages3) & 1) ^ 1, a.err, &failed))
              break;
            const uint32_t fb = smem_u32(&bars.b_full[s]);
            mbar_arrive_expect_tx(fb, C::kTileB);
            for (int c = 0; c < 2; ++c)   // heads [64c, 64c+64) of the tile's 128 key slots
              tma_load_2d(sB + s * C::kTileB + c * kKeyTile3 * 128, bm, fb, 64 * c, en[e].srow);
            ++nb;
          }
        }
        ++ni;
      }
      // on a failure, let the copies already issued land before the exit
      if (failed) {
        bool f2 = false;
        if (ua0 > 0) mbar_wait(smem_u32(&bars.a_full[0]), (ua0 - 1) & 1, a.err, &f2);
        if (ua1 > 0) mbar_wait(smem_u32(&bars.a_full[1]), (ua1 - 1) & 1, a.err, &f2);
        for (int i = nb > kStages3 ? nb - kStages3 : 0; i < nb; ++i)
          mbar_wait(smem_u32(&bars.b_full[i % kStages3]), (i / kStages3) & 1, a.err, &f2);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA: per tile and 128-column block, 8 K-steps of 16 heads ----
    // The whole warp runs the loop (waits included); one elected lane issues each tcgen05
    // instruction (a lone lane issues MMAs much more slowly).
    {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id = idesc_f16(128, kKeyTile3, bf16, true, false);
      int ua0 = 0, ua1 = 0, nb = 0, nt = 0, ni = 0;   // uses per A slot, B entries, tiles, items
      for (int it = blockIdx.x; it < nitems && !failed; it += gridDim.x) {
        const Item3 x = item3<D>(a, it, nparts);
        if (x.ntiles == 0) continue;
        const Part3 pk = part3<D>(x.part, merged);
        const int nblk = pk.rope ? 1 : C::kW / 128;
        const int ab1 = merged ? 0 : (ni & 1);   // the slot of a single-slot part
        int last[2];
        const int used = slots3(a, x, pk.mixed, ab1, last);
        int waited = 0;   // slots whose slice this item has seen land
        for (int t = 0; t < x.ntiles; ++t) {
          const int tb = nt & 1;
          Entry3 en[2];
          const int ne = entries3(a, x, tile3(x, t), pk.mixed, pk.is_dv, ab1, en);
          mbar_wait_spin(smem_u32(&bars.t_empty[tb]), ((nt >> 1) & 1) ^ 1, a.err, &failed);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (e >= ne) break;
            const int s = nb % kStages3;
            const int ab = en[e].slot;
            if (!((waited >> ab) & 1)) {
              mbar_wait_spin(smem_u32(&bars.a_full[ab]), (ab ? ua1 : ua0) & 1, a.err, &failed);
              waited |= 1 << ab;
            }
            mbar_wait_spin(smem_u32(&bars.b_full[s]), (nb / kStages3) & 1, a.err, &failed);
            if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
            tc_fence_after();
            const uint64_t db = smem_desc_sw128(sB + s * C::kTileB, 16, 1024);
            if (elect_one()) {
              for (int m = 0; m < nblk; ++m) {
                // A: columns [128m, 128m+128) = two 64-column boxes (lbo = box stride); the
                // rope part has one box, and lanes 64-127 of its result are never read
                const uint64_t da = smem_desc_sw128(sA + ab * C::kSlice + 2 * m * C::kBox, C::kBox, 1024);
#pragma unroll
                for (int k = 0; k < kHeadsPad / 16; ++k)
                  umma_f16<1>(tmem + tb * 256 + m * 128, da + (uint64_t)((k * 2048) >> 4),
                              db + (uint64_t)(((k >> 2) * kKeyTile3 * 128 + (k & 3) * 32) >> 4), id,
                              (e | k) != 0);
              }
              umma_commit(smem_u32(&bars.b_empty[s]));
              if (e == ne - 1) umma_commit(smem_u32(&bars.t_full[tb]));
              // the slot's last reads of this item: free it for the next item's slice
              if (t == (ab ? last[1] : last[0])) umma_commit(smem_u32(&bars.a_empty[ab]));
            }
            __syncwarp();
            ++nb;
          }
          if (failed) break;
          ++nt;
        }
        if (failed) break;
        if (used & 1) ++ua0;
        if (used & 2) ++ua1;
        ++ni;
      }
      // the MMAs issued last complete before the exit (their TMEM is freed afterwards)
      if (nt > 0) {
        bool f2 = false;
        mbar_wait(smem_u32(&bars.t_full[(nt - 1) & 1]), ((nt - 1) >> 1) & 1, a.err, &f2);
      }
    }
    __syncwarp();
  } else {
    // ---- drain: TMEM lane = output column, column = key; red.v2 into fp32 ----
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int cg = (warp - 2) >> 2;    // column group 0..3
    int nt = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
      const Item3 x = item3<D>(a, it, nparts);
      if (x.ntiles == 0) continue;
      const Part3 pk = part3<D>(x.part, merged);
      const bool rope = pk.rope;
      float* acc = rope ? a.dkr_acc : pk.is_dv ? a.dv_acc : a.dk_acc;   // merged: dK + dV
      const int ld = rope ? 64 : D;
      const int col0 = pk.col0;
      const int nk = rope ? 32 : C::kW / 4;   // keys of a tile per column group: 64 or 32
      const int c_off = cg * nk;              // TMEM column of the share within a buffer
      const int mblk = c_off >> 7, key0 = c_off & 127;
      const bool lanes_ok = !rope || q < 2;   // rope: 64 output columns
      float* gcol = acc + col0 + mblk * 128 + 32 * q + lane - (lane & 1);
      const size_t nent = (size_t)a.topk * a.block;
      // accumulator rows of the share's keys of tile t (-1: no key); the keys of a tile are
      // listed in the key list of any of its member rows (the first)
      auto load_rows = [&](int t, int (&r)[2]) {
        const Tile3 y = tile3(x, t);
        const int g0 = (y.mask & 1) ? 0 : 1;
        const int32_t* rows = a.ws_rows + (size_t)(x.row0 + g0) * nent + (g0 ? y.off1 : y.off0);
        r[0] = key0 + lane < y.len ? __ldg(rows + key0 + lane) : -1;
        r[1] = nk == 64 && key0 + 32 + lane < y.len ? __ldg(rows + key0 + 32 + lane) : -1;
      };
      int kr[2];
      load_rows(0, kr);
      for (int t = 0; t < x.ntiles; ++t) {
        const int tb = nt & 1;
        int kn[2] = {-1, -1};
        if (t + 1 < x.ntiles) load_rows(t + 1, kn);   // in flight while this tile drains
        mbar_wait(smem_u32(&bars.t_full[tb]), (nt >> 1) & 1, a.err, &failed);
        if (__any_sync(0xffffffffu, failed)) break;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + tb * 256 + c_off;
        const uint32_t t_empty = smem_u32(&bars.t_empty[tb]);
        if (nk == 64)
          dkv_drain<64>(taddr, t_empty, lanes_ok, gcol, ld, kr, lane);
        else
          dkv_drain<32>(taddr, t_empty, lanes_ok, gcol, ld,
                        *reinterpret_cast<const int(*)[1]>(&kr[0]), lane);
        kr[0] = kn[0];
        kr[1] = kn[1];
        ++nt;
      }
      if (failed) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc<1>(tmem, 512);
}

// =====================================================================================
// K3 over groups of four rows (5-output calls, D = 256 or 512, at most 2048 keys a row)
// =====================================================================================
// Four adjacent query rows share more keys than two (config 4: the union of four rows'
// lists is 0.48 of their valid pairs, of two rows' 0.73).  sfa_bwd_group4_kernel reorders
// the four lists in place into runs, one per member mask (the rows that select the key).
// A key's rank in its run is its rank in the list of the run's lowest member row, so every
// member row lists the run's keys in the same order and a 128-key tile of the run is one TMA
// box per member row.  The runs are walked with the masks that hold row 0 first (odd masks),
// then those with row 1 (2, 6, 10, 14), row 2 (4, 12) and row 3 (8), so that each row's
// slice is released for the next item as early as the walk allows.  A group whose lists
// hold a key twice keeps its lists, one run per row.
// The merged mode (key == value) groups two rows (`gs` = 2): its slices are twice as many
// (Q and dO), so two rows fill the four slots; its records have rows 2 and 3 empty.
// Record of a group (kRec4 int4): [0] = (tiles, last tile of row 0, of row 1, of row 2),
// [1] = (last tile of row 3, runs, 0, 0), then per non-empty run in walking order
// (mask, length, first slot in row 0, in row 1) and (first slot in row 2, in row 3, 0, 0).
// Last tile -1: the row has no keys.
constexpr int kRec4 = 32;
constexpr int kGroup4Threads = 1024;

__device__ __forceinline__ int walk4(int p) {
  return p < 8 ? 2 * p + 1 : p < 12 ? 2 + 4 * (p - 8) : p < 14 ? 4 + 8 * (p - 12) : 8;
}

__device__ __forceinline__ uint32_t field12(const uint64_t (&c)[3], int f) {
  return (uint32_t)(c[f / 5] >> (12 * (f % 5))) & 0xfffu;
}

__global__ void __launch_bounds__(kGroup4Threads) sfa_bwd_group4_kernel(const Args a,
                                                                       int32_t* ws_rows,
                                                                       int4* recs, int lg,
                                                                       int gs) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t warp_sum[3][kGroup4Threads / 32];
  __shared__ int offs[4][16];   // first slot of the run of mask m in row g
  __shared__ int cnt[16];       // keys of each mask
  __shared__ int dup;
  const int H = 1 << lg;   // >= 2 x the group's keys: the probe loops end
  int* keys = reinterpret_cast<int*>(smem_raw);
  uint32_t* word = reinterpret_cast<uint32_t*>(keys + H);   // mask | rank << 4
  int* slot_of = reinterpret_cast<int*>(word + H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = gs * blockIdx.x;
  const size_t nent = (size_t)a.topk * a.block;
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  int n[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int r = r0 + g;
    n[g] = 0;
    if (g < gs && r < a.num_rows && !abort) {
      const RowInfo ri = row_info(a, r);
      n[g] = ri.active ? __ldg(a.ws_count + r) : 0;
    }
  }
  const int b1 = n[0], b2 = b1 + n[1], b3 = b2 + n[2], N = b3 + n[3];
  int4* rec = recs + (size_t)kRec4 * blockIdx.x;
  auto unshared = [&]() {   // lists unchanged: one run per row with keys
    if (a.orig != nullptr)
      for (int g = 0; g < 4; ++g)
        for (int j = threadIdx.x; j < n[g]; j += kGroup4Threads)
          a.orig[(size_t)(r0 + g) * nent + j] = (int16_t)j;
    if (threadIdx.x == 0) {
      int t = 0, nr = 0, last[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        last[g] = -1;
        if (n[g] == 0) continue;
        rec[2 + 2 * nr] = make_int4(1 << g, n[g], 0, 0);
        rec[3 + 2 * nr] = make_int4(0, 0, 0, 0);
        ++nr;
        t += tiles3(n[g]);
        last[g] = t - 1;
      }
      rec[0] = make_int4(t, last[0], last[1], last[2]);
      rec[1] = make_int4(last[3], nr, 0, 0);
    }
  };
  if (N == 0 || 2 * N > H) {   // uniform over the block
    unshared();
    return;
  }
  for (int i = threadIdx.x; i < H; i += kGroup4Threads) {
    keys[i] = -1;
    word[i] = 0u;
  }
  if (threadIdx.x == 0) dup = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += kGroup4Threads) {
    const int g = (i >= b1) + (i >= b2) + (i >= b3);
    const int j = i - (g == 0 ? 0 : g == 1 ? b1 : g == 2 ? b2 : b3);
    const int k = ws_rows[(size_t)(r0 + g) * nent + j];
    uint32_t h = group_hash(k, lg);
    for (int probe = 0; probe < H; ++probe) {
      const int prev = atomicCAS(&keys[h], -1, k);
      if (prev == -1 || prev == k) {
        if (atomicOr(&word[h], 1u << g) & (1u << g)) dup = 1;   // listed twice in row g
        slot_of[i] = (int)h;
        break;
      }
      h = (h + 1) & (uint32_t)(H - 1);
    }
  }
  __syncthreads();
  if (dup) {   // uniform: read after the barrier
    unshared();
    return;
  }
  // Each thread takes a contiguous chunk of every list; per mask it counts the entries of the
  // mask's lowest member row (12-bit fields: masks 1-5 in c[0], 6-10 in c[1], 11-15 in c[2];
  // a count is at most 2048).
  int j0[4], j1[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int pg = (n[g] + kGroup4Threads - 1) / kGroup4Threads;
    j0[g] = min(n[g], (int)threadIdx.x * pg);
    j1[g] = min(n[g], j0[g] + pg);
  }
  const int bs[4] = {0, b1, b2, b3};
  uint64_t c[3] = {0, 0, 0};
#pragma unroll
  for (int g = 0; g < 4; ++g)
    for (int j = j0[g]; j < j1[g]; ++j) {
      const int m = (int)(word[slot_of[bs[g] + j]] & 15u);
      if (__ffs(m) - 1 == g) {
        const int f = m - 1;
        c[f / 5] += 1ull << (12 * (f % 5));
      }
    }
  uint64_t v[3];
#pragma unroll
  for (int x = 0; x < 3; ++x) {
    v[x] = c[x];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, v[x], o);
      if (lane >= o) v[x] += y;
    }
    if (lane == 31) warp_sum[x][warp] = v[x];
  }
  __syncthreads();
  if (warp < 3) {
    uint64_t w = lane < kGroup4Threads / 32 ? warp_sum[warp][lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kGroup4Threads / 32) warp_sum[warp][lane] = w;
  }
  __syncthreads();
  uint64_t e[3], tot[3];
#pragma unroll
  for (int x = 0; x < 3; ++x) {
    e[x] = v[x] - c[x] + (warp > 0 ? warp_sum[x][warp - 1] : 0);
    tot[x] = warp_sum[x][kGroup4Threads / 32 - 1];
  }
  if (threadIdx.x < 15) cnt[threadIdx.x + 1] = (int)field12(tot, threadIdx.x);
  __syncthreads();
  if (threadIdx.x < 64) {   // offs[g][m]: keys of the earlier runs (walking order) that row g holds
    const int g = threadIdx.x >> 4, m = threadIdx.x & 15;
    int off = 0;
    for (int p = 0; p < 15; ++p) {
      const int mp = walk4(p);
      if (mp == m) break;
      if ((mp >> g) & 1) off += cnt[mp];
    }
    offs[g][m] = off;
  }
  __syncthreads();
  // every list entry was read into the table above, so the lists are rewritten in place:
  // first the lowest member row of each key (which leaves the rank for the others), ...
#pragma unroll
  for (int g = 0; g < 4; ++g)
    for (int j = j0[g]; j < j1[g]; ++j) {
      const int h = slot_of[bs[g] + j];
      const uint32_t w = word[h];
      const int m = (int)(w & 15u);
      if (__ffs(m) - 1 != g) continue;
      const int f = m - 1;
      const int rank = (int)((e[f / 5] >> (12 * (f % 5))) & 0xfffu);
      e[f / 5] += 1ull << (12 * (f % 5));
      ws_rows[(size_t)(r0 + g) * nent + offs[g][m] + rank] = keys[h];
      if (a.orig != nullptr) a.orig[(size_t)(r0 + g) * nent + offs[g][m] + rank] = (int16_t)j;
      if (m != (1 << g)) word[h] = w | ((uint32_t)rank << 4);
    }
  __syncthreads();
  // ... then the other member rows at the same rank
#pragma unroll
  for (int g = 0; g < 4; ++g)
    for (int j = j0[g]; j < j1[g]; ++j) {
      const int h = slot_of[bs[g] + j];
      const uint32_t w = word[h];
      const int m = (int)(w & 15u);
      if (__ffs(m) - 1 == g) continue;
      ws_rows[(size_t)(r0 + g) * nent + offs[g][m] + (int)(w >> 4)] = keys[h];
      if (a.orig != nullptr) a.orig[(size_t)(r0 + g) * nent + offs[g][m] + (int)(w >> 4)] = (int16_t)j;
    }
  if (threadIdx.x == 0) {
    int t = 0, nr = 0, last[4] = {-1, -1, -1, -1};
    for (int p = 0; p < 15; ++p) {
      const int m = walk4(p);
      if (cnt[m] == 0) continue;
      rec[2 + 2 * nr] = make_int4(m, cnt[m], offs[0][m], offs[1][m]);
      rec[3 + 2 * nr] = make_int4(offs[2][m], offs[3][m], 0, 0);
      ++nr;
      t += tiles3(cnt[m]);
#pragma unroll
      for (int g = 0; g < 4; ++g)
        if ((m >> g) & 1) last[g] = t - 1;
    }
    rec[0] = make_int4(t, last[0], last[1], last[2]);
    rec[1] = make_int4(last[3], nr, 0, 0);
  }
}

// K3 of a four-row group runs on a CTA pair (tcgen05 cta_group::2): M = 256 output columns
// of the part (128 per CTA), N = 128 keys of the tile (each CTA loads 64 of them), K = 128
// heads per member row.  Each CTA keeps its 128 columns of the four rows' slices (4 x 32 KB)
// and a 6-stage ring of 64-key dS / P halves (16 KB); a tile of a run with r member rows
// takes r ring entries into one of four TMEM accumulators (128 columns each; the drains of
// both CTAs free it), so a key the r rows share is reduced once.
// Each CTA drains its own 128 columns of the 128 keys (16 warps: 4 TMEM lane quadrants x 32
// keys) with the same whole-row red.v2 form as K3.  Roles: warp 0 (one lane) loads the
// slices and the ring entries in both CTAs, warp 1 of the leader issues the MMAs, warps 2-17
// drain.  Parts: dK columns [0,256) and [256,512) (D = 512), the same of dV, and dKr (64
// columns on the leader; the peer's half of that product is never read).  Merged mode
// (dv_acc == NULL): groups of two rows, row g's Q and dO slices in slots 2g and 2g+1, parts
// dK + dV of [0,256) and [256,512) and dKr; a merged part's tile takes two entries per member
// row, dS with Q and then P with dO, into the same accumulator.
constexpr int kStages4 = 6;

template <int D>
struct Cfg4 {
  static constexpr int kW = 256;                           // output columns per part
  static constexpr int kDParts = D / kW;
  static constexpr int kParts = 2 * kDParts + 1;
  static constexpr int kBox = 128 * 128;                   // 64 columns x 128 heads, MN-major
  static constexpr int kSlot = 2 * kBox;                   // this CTA's 128 columns of a row
  static constexpr int kHalf = 64 * 128;                   // 64 key slots x 64 heads
  static constexpr int kTileB = 2 * kHalf;                 // 64 key slots x 128 heads
  static constexpr int kOffA = 0;
  static constexpr int kOffB = 4 * kSlot;
  static constexpr int kOffBars = kOffB + kStages4 * kTileB;
};

struct Maps4 {
  CUtensorMap ds, pp, q, qr, dout;   // scratch boxes 64 heads x 64 slots; slices 64 x 128
};

struct __align__(16) Bars4 {
  uint64_t a_full[4], a_empty[4];
  uint64_t b_full[kStages4], b_empty[kStages4];
  uint64_t t_full[4], t_empty[4];
  uint32_t tmem_slot;
};

constexpr int kThreads4 = 18 * 32;   // warp 0: TMA, 1: MMA (leader), 2-17: drain

// Tile cursor over a group record's runs (every role walks the same sequence).
struct Cur4 {
  int r, i, nt;
  int4 ra, rb;
};

__device__ __forceinline__ void cur4_init(Cur4& c, const int4* rec) {
  c.r = 0;
  c.i = 0;
  c.ra = __ldg(rec + 2);
  c.rb = __ldg(rec + 3);
  c.nt = tiles3(c.ra.y);
}

__device__ __forceinline__ void cur4_next(Cur4& c, const int4* rec, int nruns) {
  if (++c.i < c.nt) return;
  c.i = 0;
  if (++c.r < nruns) {
    c.ra = __ldg(rec + 2 + 2 * c.r);
    c.rb = __ldg(rec + 3 + 2 * c.r);
    c.nt = tiles3(c.ra.y);
  }
}

// first slot of the current tile in row g
__device__ __forceinline__ int cur4_off(const Cur4& c, int g) {
  return (g == 0 ? c.ra.z : g == 1 ? c.ra.w : g == 2 ? c.rb.x : c.rb.y) + kKeyTile3 * c.i;
}

template <int D, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads4, 1)
    sfa_bwd_dkv4_kernel(const __grid_constant__ Maps4 maps, const Args a) {
  using C = Cfg4<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Bars4& bars = *reinterpret_cast<Bars4*>(smem_raw + C::kOffBars);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sA = sbase + C::kOffA, sB = sbase + C::kOffB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {   // identical in both CTAs of the pair, so both leave together
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const uint32_t cta = cluster_ctarank();
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const bool merged = a.dv_acc == nullptr;
  const int gs = merged ? 2 : 4;                       // rows per group
  const int nparts = merged ? C::kDParts + 1 : C::kParts;
  const int ngroups = (a.num_rows + gs - 1) / gs;
  const int nitems = abort ? 0 : ngroups * nparts;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const size_t nent = (size_t)a.topk * a.block;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; ++s) {
      mbar_init(smem_u32(&bars.a_full[s]), 1);    // leader: bytes of both CTAs
      mbar_init(smem_u32(&bars.a_empty[s]), 1);
    }
    for (int s = 0; s < kStages4; ++s) {
      mbar_init(smem_u32(&bars.b_full[s]), 1);    // leader: bytes of both CTAs
      mbar_init(smem_u32(&bars.b_empty[s]), 1);
    }
    for (int s = 0; s < 4; ++s) {
      mbar_init(smem_u32(&bars.t_full[s]), 1);
      mbar_init(smem_u32(&bars.t_empty[s]), 32);  // leader: 16 drain warps of each CTA
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(smem_u32(&bars.tmem_slot), 512);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool failed = false;

  if (warp == 0) {
    // ---- TMA (both CTAs): this CTA's columns of the member rows' slices, its 64 key slots
    // of every ring entry; completion counted on the leader's barriers ----
    if (lane == 0) {
      int ua[4] = {0, 0, 0, 0}, nb = 0;
      for (int it = pair; it < nitems && !failed; it += npairs) {
        const int grp = it / nparts, part = it % nparts;
        const int4* rec = a.recs + (size_t)kRec4 * grp;
        const int4 h0 = __ldg(rec), h1 = __ldg(rec + 1);
        if (h0.x == 0) continue;
        const bool rope = part == (merged ? C::kDParts : 2 * C::kDParts);
        const bool mixed = merged && !rope;
        const bool is_dv = !merged && !rope && part >= C::kDParts;
        const int col0 = rope ? 0 : (part % C::kDParts) * C::kW;
        const int row0 = gs * grp;
        // a slice is loaded just before the first ring entry that needs it, so the item's
        // first tiles do not wait for the slots the previous item releases last
        int loaded = 0;
        Cur4 cu;
        cur4_init(cu, rec);
        for (int t = 0; t < h0.x && !failed; ++t) {
          const int mask = cu.ra.x;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            if (!((mask >> g) & 1)) continue;
#pragma unroll
            for (int hm = 0; hm < 2; ++hm) {
              if ((hm == 1 && !mixed) || failed) continue;
              // slot and operands of this entry: the member row's slice (merged: Q then dO)
              const int slot = merged ? 2 * g + hm : g;
              const bool second = is_dv || hm == 1;   // dO / P
              if (!((loaded >> slot) & 1)) {
                if (!mbar_wait_sleep(smem_u32(&bars.a_empty[slot]), (ua[slot] & 1) ^ 1, a.err, &failed))
                  continue;
                const CUtensorMap* am = rope ? &maps.qr : second ? &maps.dout : &maps.q;
                const uint32_t fa = smem_u32(&bars.a_full[slot]);
                if (cta == 0) mbar_arrive_expect_tx(fa, 2 * C::kSlot);
                for (int c = 0; c < 2; ++c)
                  tma_load_2d_pair(sA + slot * C::kSlot + c * C::kBox, am, mapa_shared(fa, 0),
                                   col0 + 128 * (int)cta + 64 * c, (row0 + g) * a.N1);
                ++ua[slot];
                loaded |= 1 << slot;
              }
              const int s = nb % kStages4;
              if (!mbar_wait_sleep(smem_u32(&bars.b_empty[s]), ((nb / kStages4) & 1) ^ 1, a.err, &failed))
                continue;
              const uint32_t fb = smem_u32(&bars.b_full[s]);
              if (cta == 0) mbar_arrive_expect_tx(fb, 2 * C::kTileB);
              const int srow = (row0 + g) * a.kp + cur4_off(cu, g) + 64 * (int)cta;
              const CUtensorMap* bm = second ? &maps.pp : &maps.ds;
              for (int c = 0; c < 2; ++c)   // heads [64c, 64c+64) of this CTA's 64 key slots
                tma_load_2d_pair(sB + s * C::kTileB + c * C::kHalf, bm, mapa_shared(fb, 0), 64 * c, srow);
              ++nb;
            }
          }
          cur4_next(cu, rec, h1.y);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA (leader; the whole warp runs the loop, one elected lane issues) ----
    if (cta == 0) {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id = idesc_f16(256, kKeyTile3, bf16, true, false);
      int ua[4] = {0, 0, 0, 0}, nb = 0, nt = 0;
      for (int it = pair; it < nitems && !failed; it += npairs) {
        const int grp = it / nparts, part = it % nparts;
        const int4* rec = a.recs + (size_t)kRec4 * grp;
        const int4 h0 = __ldg(rec), h1 = __ldg(rec + 1);
        if (h0.x == 0) continue;
        const bool mixed = merged && part != C::kDParts;
        const int last[4] = {h0.y, h0.z, h0.w, h1.x};
        int waited = 0, used = 0;
        Cur4 cu;
        cur4_init(cu, rec);
        for (int t = 0; t < h0.x; ++t) {
          const int tb = nt & 3;
          const int mask = cu.ra.x;
          const int ne = __popc(mask) * (mixed ? 2 : 1);
          mbar_wait_spin(smem_u32(&bars.t_empty[tb]), ((nt >> 2) & 1) ^ 1, a.err, &failed, true);
          int e = 0;
#pragma unroll 1
          for (int x = 0; x < 8; ++x) {   // entry x: member row x >> 1, Q / dO part x & 1
            const int g = x >> 1, hm = x & 1;
            if (!((mask >> g) & 1) || (hm == 1 && !mixed)) continue;
            const int slot = merged ? 2 * g + hm : g;
            const int s = nb % kStages4;
            if (!((waited >> slot) & 1)) {
              const int u = slot == 0 ? ua[0] : slot == 1 ? ua[1] : slot == 2 ? ua[2] : ua[3];
              mbar_wait_spin(smem_u32(&bars.a_full[slot]), u & 1, a.err, &failed, true);
              waited |= 1 << slot;
              used |= 1 << slot;
            }
            mbar_wait_spin(smem_u32(&bars.b_full[s]), (nb / kStages4) & 1, a.err, &failed, true);
            if (__any_sync(0xffffffffu, failed)) {
              failed = true;
              break;
            }
            tc_fence_after();
            const uint64_t da = smem_desc_sw128(sA + slot * C::kSlot, C::kBox, 1024);
            const uint64_t db = smem_desc_sw128(sB + s * C::kTileB, 16, 1024);
            if (elect_one()) {
#pragma unroll
              for (int k = 0; k < kHeadsPad / 16; ++k)
                umma_f16<2>(tmem + tb * kKeyTile3, da + (uint64_t)((k * 2048) >> 4),
                            db + (uint64_t)(((k >> 2) * C::kHalf + (k & 3) * 32) >> 4), id,
                            (e | k) != 0);
              umma_commit_pair(smem_u32(&bars.b_empty[s]), 3);
              if (e == ne - 1) umma_commit_pair(smem_u32(&bars.t_full[tb]), 3);
              // the member row's last tile of this item: its slot is free for the next item
              if (t == (g == 0 ? last[0] : g == 1 ? last[1] : g == 2 ? last[2] : last[3]))
                umma_commit_pair(smem_u32(&bars.a_empty[slot]), 3);
            }
            __syncwarp();
            ++nb;
            ++e;
          }
          if (failed) break;
          ++nt;
          cur4_next(cu, rec, h1.y);
        }
        if (failed) break;
#pragma unroll
        for (int sl = 0; sl < 4; ++sl)
          if ((used >> sl) & 1) ++ua[sl];
      }
      // the MMAs issued last complete before the exit (their TMEM is freed afterwards)
      if (nt > 0) {
        bool f2 = false;
        mbar_wait(smem_u32(&bars.t_full[(nt - 1) & 3]), ((nt - 1) >> 2) & 1, a.err, &f2);
      }
    }
    __syncwarp();
  } else {
    // ---- drain (both CTAs): TMEM lane = output column, column = key ----
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int cg = (warp - 2) >> 2;    // keys [32 cg, 32 cg + 32) of a tile
    const uint32_t lead_te = mapa_shared(smem_u32(&bars.t_empty[0]), 0);
    int nt = 0;
    for (int it = pair; it < nitems; it += npairs) {
      const int grp = it / nparts, part = it % nparts;
      const int4* rec = a.recs + (size_t)kRec4 * grp;
      const int4 h0 = __ldg(rec), h1 = __ldg(rec + 1);
      if (h0.x == 0) continue;
      const bool rope = part == (merged ? C::kDParts : 2 * C::kDParts);
      const bool is_dv = !merged && !rope && part >= C::kDParts;
      const int col0 = rope ? 0 : (part % C::kDParts) * C::kW;
      float* acc = rope ? a.dkr_acc : is_dv ? a.dv_acc : a.dk_acc;   // merged: dK + dV
      const int ld = rope ? 64 : D;
      const bool lanes_ok = !rope || (cta == 0 && q < 2);   // rope: 64 output columns
      float* gcol = acc + col0 + 128 * (int)cta + 32 * q + lane - (lane & 1);
      const int row0 = gs * grp;
      // accumulator row of this lane's key of the cursor's tile (-1: none); a tile's keys
      // are listed in the key list of any of its member rows (the lowest)
      auto key_row = [&](const Cur4& c) {
        const int g0 = __ffs(c.ra.x) - 1;
        const int k = 32 * cg + lane;
        const int len = min(kKeyTile3, c.ra.y - kKeyTile3 * c.i);
        return k < len ? __ldg(a.ws_rows + (size_t)(row0 + g0) * nent + cur4_off(c, g0) + k) : -1;
      };
      Cur4 cu;   // one tile ahead of the tile being drained
      cur4_init(cu, rec);
      int kr = key_row(cu);
      cur4_next(cu, rec, h1.y);
      for (int t = 0; t < h0.x; ++t) {
        const int tb = nt & 3;
        const int kn = t + 1 < h0.x ? key_row(cu) : -1;   // in flight while this tile drains
        if (t + 1 < h0.x) cur4_next(cu, rec, h1.y);
        mbar_wait(smem_u32(&bars.t_full[tb]), (nt >> 2) & 1, a.err, &failed);
        if (__any_sync(0xffffffffu, failed)) break;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + tb * kKeyTile3 + 32 * cg;
        const int rows[1] = {kr};
        dkv_drain<32, true>(taddr, lead_te + 8 * tb, lanes_ok, gcol, ld, rows, lane);
        kr = kn;
        ++nt;
      }
      if (failed) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, 512);
}

// =====================================================================================
// K4: fp32 accumulators -> key dtype
// =====================================================================================
template <typename T>
__global__ void cast_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    uint2 w;
    w.x = ElemTraits<T>::pack2(v.x, v.y);
    w.y = ElemTraits<T>::pack2(v.z, v.w);
    *reinterpret_cast<uint2*>(dst + i) = w;
  } else {
    for (int64_t j = i; j < n; ++j) dst[j] = ElemTraits<T>::from_f(src[j]);
  }
}

template <typename T>
int cast_all(const DsaSfaBwdParams* p, cudaStream_t stream) {
  const int64_t D = p->d;
  const int64_t n[3] = {p->kv_rows * D, p->kv_rows * 64, p->kv_rows * D};
  const float* src[3] = {p->dk_acc, p->dkr_acc, p->dv_acc};
  void* dst[3] = {p->dk, p->dkr, p->dv};
  for (int i = 0; i < 3; ++i) {
    if (!dst[i] || !src[i]) continue;
    const int64_t threads = (n[i] + 3) / 4;
    cast_kernel<T><<<dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, stream>>>(
        src[i], static_cast<T*>(dst[i]), n[i]);
  }
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

// SMs of the current device (persistent K3 grid), cached per device
inline int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// key slots per row in the P / dS scratch: whole K1 pair tiles (256 keys)
inline int64_t padded_keys(int64_t nent) { return (nent + 255) / 256 * 256; }
inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }
// run table of the row pairs, or records of the groups of the CTA-pair K3 (four rows, or
// two in the merged mode)
inline int64_t runs_bytes(int64_t num_rows) {
  const int64_t pairs = (num_rows + 1) / 2 * 3 * 16, recs = (num_rows + 1) / 2 * kRec4 * 16;
  return align256(pairs > recs ? pairs : recs);
}
// hash table of one group (log2 of its entries): at least twice the group's keys; groups of
// longer key lists than kGroup4MaxKeys (four rows) or kGroupMaxKeys (pairs) per row are
// formed smaller or not at all
constexpr int64_t kGroupMaxKeys = 4096;
constexpr int64_t kGroup4MaxKeys = 2048;
inline int group_lg(int64_t keys_per_group) {
  int lg = 10;
  while ((int64_t(1) << lg) < 2 * keys_per_group) ++lg;
  return lg;
}

template <int D, typename T>
int launch(const DsaSfaBwdParams* p, cudaStream_t stream) {
  const bool bf16 = ElemTraits<T>::kIsBf16;
  const int64_t nent = p->topk * p->sparse_block_size;
  const int64_t kp = padded_keys(nent);
  const uint64_t qrows = (uint64_t)p->num_rows * p->n1;
  Args a = {};
  a.idx = p->sparse_indices;
  a.act_q = p->act_q;
  a.act_k = p->act_k;
  a.q_row_base = p->q_row_base;
  a.k_row_base = p->k_row_base;
  a.block_table = p->block_table;
  a.num_rows = (int)p->num_rows;
  a.B = (int)p->batch;
  a.N1 = (int)p->n1;
  a.topk = (int)p->topk;
  a.block = (int)p->sparse_block_size;
  a.kv_rows = (int)p->kv_rows;
  a.page = (int)p->page_size;
  a.max_blocks = (int)p->max_blocks;
  a.s2_cap = (int)p->s2_cap;
  a.sparse_mode = p->sparse_mode;
  a.scale = p->scale;
  a.key = p->key;
  a.key_rope = p->key_rope;
  a.dout = p->d_out;
  a.out = p->out;
  a.smax = p->softmax_max;
  a.ssum = p->softmax_sum;
  a.dq = p->dq;
  a.dqr = p->dqr;
  a.dk_acc = p->dk_acc;
  a.dkr_acc = p->dkr_acc;
  a.dv_acc = p->dv_acc;
  a.teacher = p->teacher;
  a.err = p->error_flag;
  char* ws = static_cast<char*>(p->workspace);
  a.ws_rows = reinterpret_cast<const int32_t*>(ws);
  ws += align256(4 * p->num_rows * nent);
  a.ws_count = reinterpret_cast<const int32_t*>(ws);
  ws += align256(4 * p->num_rows);
  a.ds = ws;
  ws += align256(p->num_rows * kHeadsPad * kp * 2);
  a.pp = ws;
  ws += align256(p->num_rows * kHeadsPad * kp * 2);
  a.delta = reinterpret_cast<const float*>(ws);
  ws += align256(4 * p->num_rows * kHeadsPad);
  // adjacent rows share their keys' reductions in K3: on CTA pairs where the slices fit
  // (256-column parts; groups of four rows, of two in the merged mode; with the teacher, K1
  // writes it through the map of original positions), else in pairs on single CTAs
  // (5-output calls without the teacher)
  const bool grouped4 = p->num_rows >= 2 && nent <= kGroup4MaxKeys && (D == 256 || D == 512);
  const bool grouped = !grouped4 && p->teacher == nullptr && p->num_rows >= 2 &&
                       p->dv_acc != nullptr && nent <= kGroupMaxKeys;
  const int gs4 = p->dv_acc != nullptr ? 4 : 2;   // rows per group of the CTA-pair K3
  a.runs = grouped ? reinterpret_cast<const int4*>(ws) : nullptr;
  a.recs = grouped4 ? reinterpret_cast<const int4*>(ws) : nullptr;
  ws += runs_bytes(p->num_rows);
  a.orig = grouped4 && p->teacher != nullptr ? reinterpret_cast<int16_t*>(ws) : nullptr;
  a.kp = (int)kp;

  Maps1 m1;
  Maps2 m2;
  Maps3 m3;
  Maps4 m4;
  const uint64_t krows_s = (uint64_t)p->num_rows * kp;   // scratch rows: one per key slot
  if (!make_tmap_2d_16b(&m1.q, p->q, bf16, qrows, D, (uint64_t)D * 2, 64, 64) ||
      !make_tmap_2d_16b(&m1.qr, p->q_rope, bf16, qrows, 64, 128, 64, 64) ||
      !make_tmap_2d_16b(&m1.dout, p->d_out, bf16, qrows, D, (uint64_t)D * 2, 64, 64) ||
      !make_tmap_2d_16b(&m1.k, p->key, bf16, p->kv_rows, D, (uint64_t)D * 2, 64, 1) ||
      !make_tmap_2d_16b(&m1.kr, p->key_rope, bf16, p->kv_rows, 64, 128, 64, 1) ||
      !make_tmap_2d_16b(&m2.ds, a.ds, bf16, krows_s, kHeadsPad, kHeadsPad * 2, 64, 64) ||
      !make_tmap_2d_16b(&m2.k, p->key, bf16, p->kv_rows, D, (uint64_t)D * 2, 64, 1) ||
      !make_tmap_2d_16b(&m2.kr, p->key_rope, bf16, p->kv_rows, 64, 128, 64, 1) ||
      !make_tmap_2d_16b(&m3.ds, a.ds, bf16, krows_s, kHeadsPad, kHeadsPad * 2, 64, 128) ||
      !make_tmap_2d_16b(&m3.pp, a.pp, bf16, krows_s, kHeadsPad, kHeadsPad * 2, 64, 128) ||
      !make_tmap_2d_16b(&m3.q, p->q, bf16, qrows, D, (uint64_t)D * 2, 64, 128) ||
      !make_tmap_2d_16b(&m3.qr, p->q_rope, bf16, qrows, 64, 128, 64, 128) ||
      !make_tmap_2d_16b(&m3.dout, p->d_out, bf16, qrows, D, (uint64_t)D * 2, 64, 128))
    return DSA_ERR_TMA_DESCRIPTOR;
  if (grouped4) {
    m4.q = m3.q;
    m4.qr = m3.qr;
    m4.dout = m3.dout;
    if (!make_tmap_2d_16b(&m4.ds, a.ds, bf16, krows_s, kHeadsPad, kHeadsPad * 2, 64, 64) ||
        !make_tmap_2d_16b(&m4.pp, a.pp, bf16, krows_s, kHeadsPad, kHeadsPad * 2, 64, 64))
      return DSA_ERR_TMA_DESCRIPTOR;
  }

  // fp32 accumulators start at zero unless the caller adds several calls into them; the
  // prep pass compacts the valid keys of each row
  if (!p->accumulate &&
      (cudaMemsetAsync(p->dk_acc, 0, sizeof(float) * p->kv_rows * D, stream) != cudaSuccess ||
       cudaMemsetAsync(p->dkr_acc, 0, sizeof(float) * p->kv_rows * 64, stream) != cudaSuccess ||
       (p->dv_acc &&
        cudaMemsetAsync(p->dv_acc, 0, sizeof(float) * p->kv_rows * D, stream) != cudaSuccess)))
    return DSA_ERR_CUDA;
  launch_prep(a, const_cast<int32_t*>(a.ws_rows), const_cast<int32_t*>(a.ws_count), p->num_rows,
              stream);
  if (grouped4) {
    const int lg = group_lg(gs4 * nent);
    const int smem = group_smem_bytes(lg);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(sfa_bwd_group4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    sfa_bwd_group4_kernel<<<dim3((unsigned)((p->num_rows + gs4 - 1) / gs4)), dim3(kGroup4Threads),
                            smem, stream>>>(a, const_cast<int32_t*>(a.ws_rows),
                                            const_cast<int4*>(a.recs), lg, gs4);
  }
  if (grouped) {
    const int lg = group_lg(2 * nent);
    const int smem = group_smem_bytes(lg);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(sfa_bwd_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    sfa_bwd_group_kernel<<<dim3((unsigned)((p->num_rows + 1) / 2)), dim3(kGroupThreads), smem,
                           stream>>>(a, const_cast<int32_t*>(a.ws_rows), const_cast<int4*>(a.runs),
                                     lg);
  }
  {
    const int64_t n = p->num_rows * p->n1;
    sfa_bwd_delta_kernel<D, T><<<dim3((unsigned)((n + 7) / 8)), dim3(256), 0, stream>>>(
        static_cast<const T*>(p->d_out), static_cast<const T*>(p->out),
        const_cast<float*>(a.delta), n);
  }

  {
    auto k = sfa_bwd_probs_kernel<D, T>;
    const int smem = Cfg1<D>::kOffBars + (int)sizeof(Bars1);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    k<<<dim3(2 * (unsigned)p->num_rows), dim3(kThreads1), smem, stream>>>(m1, a);
  }
  {
    auto k = sfa_bwd_dq_kernel<D, T>;
    const int smem = Cfg2<D>::kOffBars + (int)sizeof(Bars2);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    k<<<dim3(2 * (unsigned)p->num_rows), dim3(kThreads2), smem, stream>>>(m2, a);
  }
  if (grouped4) {
    if constexpr (D >= 256) {
      auto k = sfa_bwd_dkv4_kernel<D, T>;
      const int smem = Cfg4<D>::kOffBars + (int)sizeof(Bars4);
      static_assert(Cfg4<D>::kOffBars + (int)sizeof(Bars4) <= 232448, "K3 pair smem");
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return DSA_ERR_CUDA;
      const int64_t items = (p->num_rows + gs4 - 1) / gs4 *
                            (p->dv_acc ? Cfg4<D>::kParts : Cfg4<D>::kDParts + 1);
      const int64_t pairs_max = sm_count() / 2;
      const int npairs = (int)(items < pairs_max ? items : pairs_max);
      k<<<dim3(2 * (unsigned)npairs), dim3(kThreads4), smem, stream>>>(m4, a);
    }
  } else {
    auto k = sfa_bwd_dkv_kernel<D, T>;
    const int smem = Cfg3<D>::kOffBars + (int)sizeof(Bars3);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return DSA_ERR_CUDA;
    // the kernel walks the same count (groups3)
    const int64_t groups = grouped ? (p->num_rows + 1) / 2 : p->num_rows;
    const int64_t items = groups * (p->dv_acc ? Cfg3<D>::kParts : Cfg3<D>::kDParts + 1);
    const int grid = (int)(items < sm_count() ? items : sm_count());
    k<<<dim3((unsigned)grid), dim3(kThreads3), smem, stream>>>(m3, a);
  }
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  if (p->defer_cast) return DSA_OK;
  return cast_all<T>(p, stream);
}

}  // namespace sfa_bwd
}  // namespace dsa

extern "C" int64_t dsa_sfa_bwd_workspace_size(int64_t num_rows, int64_t topk, int64_t sparse_block_size) {
  using namespace dsa::sfa_bwd;
  if (num_rows < 0 || topk < 0 || sparse_block_size < 1) return -1;
  const int64_t nent = topk * sparse_block_size;
  return align256(4 * num_rows * nent) + align256(4 * num_rows) +
         2 * align256(num_rows * kHeadsPad * padded_keys(nent) * 2) + align256(4 * num_rows * kHeadsPad) +
         runs_bytes(num_rows) + align256(2 * num_rows * nent);
}

extern "C" int dsa_sfa_bwd(const DsaSfaBwdParams* p, void* stream_) {
  using namespace dsa::sfa_bwd;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!p) return DSA_ERR_INVALID_ARG;
  if (p->num_rows < 0 || p->n1 < 1 || p->n1 > 128 || p->batch < 1 || p->topk < 1 ||
      p->sparse_block_size < 1 || p->kv_rows < 1 || !p->q || !p->q_rope || !p->key ||
      !p->key_rope || !p->d_out || !p->out || !p->softmax_max || !p->softmax_sum ||
      !p->sparse_indices || !p->act_q || !p->act_k || !p->q_row_base || !p->dq || !p->dqr ||
      !p->dk_acc || !p->dkr_acc || (!p->dv_acc && p->dv))
    return DSA_ERR_INVALID_ARG;
  if (!p->block_table && !p->k_row_base) return DSA_ERR_INVALID_ARG;
  if (p->teacher && p->sparse_block_size != 1) return DSA_ERR_INVALID_ARG;
  if (!p->workspace || (reinterpret_cast<uintptr_t>(p->workspace) & 255u) != 0 ||
      p->workspace_bytes < dsa_sfa_bwd_workspace_size(p->num_rows, p->topk, p->sparse_block_size))
    return DSA_ERR_INVALID_ARG;
  if (p->num_rows == 0) return DSA_OK;
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

extern "C" int dsa_sfa_bwd_cast(const DsaSfaBwdParams* p, void* stream_) {
  using namespace dsa::sfa_bwd;
  if (!p || !p->dk_acc || !p->dkr_acc || (!p->dv_acc && p->dv) || p->kv_rows < 1)
    return DSA_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (p->dtype == DSA_DTYPE_BF16) return cast_all<__nv_bfloat16>(p, stream);
  if (p->dtype == DSA_DTYPE_FP16) return cast_all<__half>(p, stream);
  return DSA_ERR_INVALID_ARG;
}
