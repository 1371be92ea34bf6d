// Lightning indexer for sm_100a: score (tcgen05) + top-k (radix select).
//
// Replaces the reference's `_lightning_indexer_score_core` / `_lightning_indexer_score_kernel`
// (lightning_indexer_triton.py:147-280, :382-413) and its top-k `_stable_topk` (:339-357).
//
// score[row, n2, s2] = sum_{g in group n2} ReLU(q[row, g] . k[s2, n2]) * w[row, g]   (fp32)
//
// Score kernel: persistent, one CTA per SM working through items (batch, block of Tq
// query tokens, key head n2), heaviest first.  The UMMA computes S^T with the keys as M
// (128 per tile) and the block's (token, head) pairs as N (Tq * G <= 256 columns), so the
// head reduction of one key is a row of TMEM owned by one thread: ReLU, weight and sum
// happen in registers and each thread writes Tq scores.  Q blocks arrive by TMA into a
// double buffer, keys stream through a TMA ring (contiguous rows, no gather); TMEM is
// double buffered so the epilogue of tile t overlaps the MMAs of tile t+1, also across
// items.  Invisible positions get -inf
// (lightning_indexer_triton.py:271-276); tiles past the block's last visible key are
// never computed (the top-k pass never reads them).
//
// Top-k kernel: one CTA per (row, n2), output ordered by (score desc, index asc) over the
// visible prefix.  Bucket path: one histogram of the scores over 4096 equal value buckets
// between the row's minimum and maximum finds the bucket of the k-th score; the buckets
// above it are scattered in descending order and every score finds its place inside its
// bucket by counting (a few entries each for spread-out scores).  Radix path, for rows with
// non-finite or clustered scores: 4-pass 8-bit radix select of the k-th largest, ordered
// compaction (ties at the threshold taken in ascending index order), then a stable LSD
// radix sort by score.  Slots past the visible keys get index -1 (:353-355).  Values are
// returned in the query dtype (:541-542).
//
// FP8 indexer (no counterpart in the reference): e4m3 query and key with a positive fp32
// scale per key row, score = key_scale * sum_g ReLU(q_g . k) * w_g (a query scale is folded
// into the weights by the caller).  The same kernel with tcgen05.mma kind::f8f6f4 (fp32
// accumulation): a 128-byte smem row holds 128 fp8 elements and one MMA takes 32 of them,
// so the shared-memory layout and descriptors are those of the 16-bit path; values come
// back in fp32.

#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "dsa_b200.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace dsa {

// fp8 (e4m3) query / key elements for the FP8 indexer, and fp32 output values
template <>
struct ElemTraits<__nv_fp8_e4m3> {
  static constexpr bool kIsBf16 = false;
  __device__ static __forceinline__ float to_f(__nv_fp8_e4m3 x) { return float(x); }
  __device__ static __forceinline__ __nv_fp8_e4m3 from_f(float x) { return __nv_fp8_e4m3(x); }
};
template <>
struct ElemTraits<float> {
  static constexpr bool kIsBf16 = false;
  __device__ static __forceinline__ float to_f(float x) { return x; }
  __device__ static __forceinline__ float from_f(float x) { return x; }
};

namespace li {

template <typename T>
constexpr bool kIsFp8 = std::is_same<T, __nv_fp8_e4m3>::value;

// tcgen05 MMA of e4m3 operands with fp32 accumulation (kind::f8f6f4; the instruction
// descriptor's A / B format code 0 is E4M3, so idesc_f16(.., false, ..) encodes it)
__device__ __forceinline__ void umma_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

constexpr int kKeys = 128;          // keys per tile (UMMA M)
constexpr int kEpiWarps = 8;        // two per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;   // 0: TMA, 1: MMA + TMEM, 2-9: epilogue

struct Args {
  const void* q;            // [q_rows][N1][D]
  const void* w;            // [q_rows][N1], fp32 / fp16 / bf16
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  const int32_t* k_row_base;
  float* scores;            // [q_rows][N2][s2_row]
  int* err;
  int B, N1, N2, G, D, Tq, N, nblk, q_rows_max, s2_row, s2_cap, sparse_mode, w_dtype;
  int q_len_dense;          // >0: BSND query, every batch has this many rows
  int items;                // B * nblk * N2 work items (one block of Tq query tokens, one key head)
  // paged keys (block_table != NULL): position s2 of batch b is pool row
  // block_table[b][s2 / page] * page + s2 % page; a tile of 128 keys is fetched as boxes of
  // box_rows rows (box_rows = min(page, 128), so a box never crosses a block)
  const int32_t* block_table;
  int page, max_blocks, box_rows;
  const float* kscale;      // fp8 keys: per (key row, n2) scale, laid out like the key rows
};

__device__ __forceinline__ float load_w(const void* w, int dtype, size_t i) {
  if (dtype == 2) return __ldg(static_cast<const float*>(w) + i);
  if (dtype == DSA_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]);
  return __half2float(static_cast<const __half*>(w)[i]);
}

// Visible keys of query position s1 (lightning_indexer_triton.py:219-227); non-decreasing
// in s1 below aq.
__device__ __forceinline__ int visible_limit(int s1, int aq, int ak, int s2, int mode) {
  if (s1 >= aq) return 0;
  if (mode == 3) {
    int causal = min(max(ak - aq + s1 + 1, 0), s2);
    return max(0, min(ak, causal));
  }
  return max(0, min(ak, s2));
}

template <int DP>
struct Cfg {
  static constexpr int kChunks = DP / 64;                   // 128-byte chunks of a row
  static constexpr int kStageBytes = kChunks * kKeys * 128;
  static constexpr int kStages = DP <= 128 ? 3 : 1;
  static constexpr int kQBytes = kChunks * 256 * 128;       // up to 256 (token, head) rows
  static constexpr int kQBufs = DP <= 128 ? 2 : 1;          // the next item's Q lands early
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kQBufs * kQBytes;
  static constexpr int kOffW = kOffK + kStages * kStageBytes;   // 2 x 256 fp32 weights
  static constexpr int kOffBars = kOffW + 2 * 256 * 4;
};

struct __align__(8) Bars {
  uint64_t full[3], empty[3], tfull[2], tfree[2], qfull[2], qfree[2];
  uint32_t tmem_slot;
};

// One work item: Tq query tokens of batch b against key head n2, keys [0, kmax) in
// ntiles tiles of 128.
struct Item {
  int b, n2, s1_0, aq, ak, nrows, qbase, kbase, kmax, ntiles;
};

// Items run heaviest first (the causal block of the last tokens has the most tiles).
__device__ __forceinline__ bool decode_item(const Args& a, int i, Item& it) {
  const int per = a.B * a.N2;
  const int blk = a.nblk - 1 - i / per;
  const int rem = i % per;
  it.b = rem / a.N2;
  it.n2 = rem % a.N2;
  it.s1_0 = blk * a.Tq;
  it.aq = __ldg(a.act_q + it.b);
  it.ak = __ldg(a.act_k + it.b);
  it.nrows = a.q_len_dense > 0 ? a.q_len_dense : it.aq;
  it.qbase = __ldg(a.q_row_base + it.b);
  it.kbase = a.block_table == nullptr ? __ldg(a.k_row_base + it.b) : 0;
  // the visible limit grows with the token, so the block's last live token has the most
  const int hi = min(min(it.s1_0 + a.Tq, it.nrows), it.aq) - 1;
  it.kmax = hi >= it.s1_0 ? visible_limit(hi, it.aq, it.ak, a.s2_cap, a.sparse_mode) : 0;
  it.ntiles = (it.kmax + kKeys - 1) / kKeys;
  return it.ntiles > 0;
}

// Persistent score kernel, one CTA per SM.  CTA c takes items c, 2G-1-c, 2G+c, ... (G CTAs;
// the heaviest-first order then spreads the work evenly).  Warp 0 streams each item's Q
// block (TMA, double buffered so that it lands during the previous item) and its key
// tiles (3-stage ring); warp 1 issues the UMMAs S^T[key, (token, head)] into one of two
// 256-column TMEM accumulators; warps 2-9 reduce them: ReLU, weight and sum over each
// token's heads, one key per thread, two warps per TMEM lane quarter splitting the columns.
// GF > 0: the head-group size G is the compile-time GF (32, 64 or 128) and N = 256, so
// every 32-column TMEM load belongs to one token; GF == 0 handles any G (one warp per
// quarter does all N columns).
template <int DP, typename T, int GF>
__global__ void __launch_bounds__(kThreads, 1)
    li_score_kernel(const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap qmap, const Args a) {
  using C = Cfg<DP>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Bars& bars = *reinterpret_cast<Bars*>(smem_raw + C::kOffBars);
  float* w_s = reinterpret_cast<float*>(smem_raw + C::kOffW);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sQ = sbase + C::kOffQ, sK = sbase + C::kOffK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const int N = a.N, G = a.G, Tq = a.Tq;
  constexpr int kEpc = 128 / (int)sizeof(T);   // elements per 128-byte chunk
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars.tfull[s]), 1);
      mbar_init(smem_u32(&bars.tfree[s]), kEpiWarps);
      mbar_init(smem_u32(&bars.qfull[s]), 1);
      mbar_init(smem_u32(&bars.qfree[s]), 1);
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
  const int ncta = gridDim.x, cta = blockIdx.x;
  auto item_at = [&](int r) { return r * ncta + ((r & 1) ? ncta - 1 - cta : cta); };

  if (warp == 0) {
    // ---- producer: Q block per item, then its key tiles ----
    if (lane == 0) {
      const uint32_t qtx = (uint32_t)(Tq * G * 128 * C::kChunks);
      int gt = 0, jq = 0;
      for (int r = 0; !failed; ++r) {
        const int i = item_at(r);
        if (i >= a.items) break;
        Item it;
        if (!decode_item(a, i, it)) continue;
        const int qb = jq % C::kQBufs;
        if (jq >= C::kQBufs &&
            !mbar_wait(smem_u32(&bars.qfree[qb]), ((jq / C::kQBufs) - 1) & 1, a.err, &failed))
          break;
        const uint32_t qf = smem_u32(&bars.qfull[qb]);
        mbar_arrive_expect_tx(qf, qtx);
        for (int c = 0; c < C::kChunks; ++c)
          tma_load_3d(sQ + qb * C::kQBytes + c * N * 128, &qmap, qf, kEpc * c, it.n2 * G,
                      it.qbase + it.s1_0);
        for (int t = 0; t < it.ntiles; ++t, ++gt) {
          const int s = gt % C::kStages;
          if (!mbar_wait_spin(smem_u32(&bars.empty[s]), ((gt / C::kStages) & 1) ^ 1, a.err, &failed))
            break;
          const uint32_t fb = smem_u32(&bars.full[s]);
          mbar_arrive_expect_tx(fb, C::kStageBytes);
          if (a.block_table == nullptr) {
            for (int c = 0; c < C::kChunks; ++c)
              tma_load_3d(sK + s * C::kStageBytes + c * kKeys * 128, &kmap, fb, kEpc * c, it.n2,
                          it.kbase + kKeys * t);
          } else {
            for (int r0 = 0; r0 < kKeys; r0 += a.box_rows) {
              const int tok = kKeys * t + r0;
              const int pidx = tok / a.page;
              // no block: a box that lies wholly before the pool, which the TMA unit fills
              // with zeros (those positions are past the row's visible keys anyway)
              int prow = -a.box_rows;
              if (pidx < a.max_blocks) {
                const int blk = __ldg(a.block_table + (size_t)it.b * a.max_blocks + pidx);
                if (blk >= 0) prow = blk * a.page + tok % a.page;
              }
              for (int c = 0; c < C::kChunks; ++c)
                tma_load_3d(sK + s * C::kStageBytes + c * kKeys * 128 + r0 * 128, &kmap, fb,
                            kEpc * c, it.n2, prow);
            }
          }
        }
        ++jq;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: the whole warp runs the loop (waits included); one elected lane
    // issues each tcgen05 instruction (a lone lane issues MMAs much more slowly) ----
    const bool bf16 = ElemTraits<T>::kIsBf16;
    const uint32_t id = idesc_f16(128, N, bf16, false, false);
    int gt = 0, jq = 0;
    for (int r = 0; !failed; ++r) {
      const int i = item_at(r);
      if (i >= a.items) break;
      Item it;
      if (!decode_item(a, i, it)) continue;
      const int qb = jq % C::kQBufs;
      mbar_wait_spin(smem_u32(&bars.qfull[qb]), (jq / C::kQBufs) & 1, a.err, &failed);
      if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
      const uint64_t dq = smem_desc_sw128(sQ + qb * C::kQBytes, 16, 1024);
      for (int t = 0; t < it.ntiles; ++t, ++gt) {
        const int s = gt % C::kStages, buf = gt & 1;
        if (gt >= 2) mbar_wait_spin(smem_u32(&bars.tfree[buf]), ((gt >> 1) - 1) & 1, a.err, &failed);
        mbar_wait_spin(smem_u32(&bars.full[s]), (gt / C::kStages) & 1, a.err, &failed);
        if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
        tc_fence_after();
        const uint64_t dk = smem_desc_sw128(sK + s * C::kStageBytes, 16, 1024);
        if (elect_one()) {
#pragma unroll
          for (int c = 0; c < C::kChunks; ++c)
#pragma unroll
            for (int u = 0; u < 4; ++u) {   // 32 bytes of K per MMA (16 bf16 / fp16, 32 fp8)
              const uint64_t ka = dk + (uint64_t)((c * kKeys * 128 + u * 32) >> 4);
              const uint64_t qd = dq + (uint64_t)((c * N * 128 + u * 32) >> 4);
              if constexpr (kIsFp8<T>) umma_e4m3(tmem + 256 * buf, ka, qd, id, (c | u) != 0);
              else umma_f16<1>(tmem + 256 * buf, ka, qd, id, (c | u) != 0);
            }
          umma_commit(smem_u32(&bars.empty[s]));
          umma_commit(smem_u32(&bars.tfull[buf]));
          if (t == it.ntiles - 1) umma_commit(smem_u32(&bars.qfree[qb]));
        }
        __syncwarp();
      }
      ++jq;
    }
    __syncwarp();
  } else {
    // ---- epilogue: one key per thread, ReLU * w summed over each token's G heads ----
    const int e = warp - 2;                 // 0..7
    const int et = threadIdx.x - 64;        // 0..255: this thread's weight slot
    const int qd = warp & 3;                // TMEM lane quarter
    const int half = e >> 2;                // GF > 0: columns [128 half, 128 half + 128)
    const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
    int gt = 0, jq = 0;
    for (int r = 0;; ++r) {
      const int i = item_at(r);
      if (i >= a.items) break;
      Item it;
      if (!decode_item(a, i, it)) continue;
      float* wb = w_s + (jq & 1) * 256;
      // this item's weights (slot = token * G + head); the buffer was last read for the item
      // before the previous one, which every epilogue warp finished before the last barrier
      if (et < N) {
        const int tq = et / G, g = et % G, s1 = it.s1_0 + tq;
        wb[et] = (tq < Tq && s1 < it.nrows)
                     ? load_w(a.w, a.w_dtype, (size_t)(it.qbase + s1) * a.N1 + it.n2 * G + g)
                     : 0.f;
      }
      if (named_bar_or(1, 32 * kEpiWarps, failed)) {
        failed = true;
        break;
      }
      for (int t = 0; t < it.ntiles; ++t, ++gt) {
        const int buf = gt & 1;
        mbar_wait_spin(smem_u32(&bars.tfull[buf]), (gt >> 1) & 1, a.err, &failed);
        const bool wfail = __any_sync(0xffffffffu, failed);
        tc_fence_after();
        const int key = kKeys * t + 32 * qd + lane;
        // fp8 keys carry a positive per-key scale: key_scale * sum_g w_g ReLU(q_g . k)
        float ks = 1.f;
        if (a.kscale != nullptr && key < it.kmax) {
          int krow = -1;
          if (a.block_table == nullptr) {
            krow = it.kbase + key;
          } else if (key / a.page < a.max_blocks) {
            const int blk = __ldg(a.block_table + (size_t)it.b * a.max_blocks + key / a.page);
            if (blk >= 0) krow = blk * a.page + key % a.page;
          }
          ks = krow >= 0 ? __ldg(a.kscale + (size_t)krow * a.N2 + it.n2) : 0.f;
        }
        auto emit = [&](int tq, float v) {
          const int s1 = it.s1_0 + tq;
          if (s1 < it.nrows && key < a.s2_row) {
            const int lim = visible_limit(s1, it.aq, it.ak, a.s2_cap, a.sparse_mode);
            float* dst = a.scores + ((size_t)(it.qbase + s1) * a.N2 + it.n2) * a.s2_row + key;
            *dst = key < lim ? v * ks : -INFINITY;
          }
        };
        if constexpr (GF > 0) {
          // 128 columns per warp in four 32-column loads, the next load in flight while
          // this one is reduced; four independent partial sums per load
          const uint32_t tb = tmem + lane_addr + 256 * buf + 128 * half;
          uint32_t ra[32], rb[32];
#pragma unroll
          for (int i2 = 0; i2 < 32; ++i2) ra[i2] = rb[i2] = 0u;
          if (!wfail) {
            tmem_ld32(tb, ra);
            tmem_ld_wait_regs(ra);
          }
          float acc = 0.f;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t(&cur)[32] = (cc & 1) ? rb : ra;
            uint32_t(&nxt)[32] = (cc & 1) ? ra : rb;
            if (cc + 1 < 4 && !wfail) tmem_ld32(tb + 32 * (cc + 1), nxt);
            const int c0 = 128 * half + 32 * cc;
            const float4* w4 = reinterpret_cast<const float4*>(wb + c0);
            float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
            for (int i2 = 0; i2 < 32; i2 += 4) {
              const float4 w = w4[i2 / 4];
              p0 = fmaf(fmaxf(__uint_as_float(cur[i2]), 0.f), w.x, p0);
              p1 = fmaf(fmaxf(__uint_as_float(cur[i2 + 1]), 0.f), w.y, p1);
              p2 = fmaf(fmaxf(__uint_as_float(cur[i2 + 2]), 0.f), w.z, p2);
              p3 = fmaf(fmaxf(__uint_as_float(cur[i2 + 3]), 0.f), w.w, p3);
            }
            acc += (p0 + p1) + (p2 + p3);
            if ((c0 + 32) % GF == 0) {
              emit(c0 / GF, acc);
              acc = 0.f;
            }
            if (cc + 1 < 4 && !wfail) tmem_ld_wait_regs(nxt);
          }
        } else if (half == 0) {
          int tok = 0, gcount = 0;
          float acc = 0.f;
          for (int c0 = 0; c0 < N; c0 += 32) {
            uint32_t rr[32];
            if (!wfail) {
              tmem_ld32(tmem + lane_addr + 256 * buf + c0, rr);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int i2 = 0; i2 < 32; ++i2) rr[i2] = 0u;
            }
#pragma unroll
            for (int i2 = 0; i2 < 32; ++i2) {
              if (tok < Tq) {
                acc = fmaf(fmaxf(__uint_as_float(rr[i2]), 0.f), wb[c0 + i2], acc);
                if (++gcount == G) {
                  emit(tok, acc);
                  ++tok;
                  gcount = 0;
                  acc = 0.f;
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars.tfree[buf]));
      }
      ++jq;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc<1>(tmem, 512);
}

// =====================================================================================
// top-k
// =====================================================================================
constexpr int kTopkThreads = 512;

// Unsigned key with the order of the float (-0 counts as +0, as in a float comparison).
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct TopkArgs {
  const float* scores;      // [q_rows][N2][s2_row]
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  int32_t* out_idx;         // [q_rows][N2][K]
  void* out_val;            // [q_rows][N2][K] query dtype, or NULL
  int* err;
  int B, N2, K, KP, s2_row, s2_cap, sparse_mode, q_rows, q_len_dense, val_dtype;
  int keys_in_gmem;         // 1: rows too long for shared memory are read from `scores` per pass
};

// Block-wide exclusive scan of one int per thread (kTopkThreads threads); returns the
// exclusive prefix and writes the block total into *total.
__device__ __forceinline__ int block_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < kTopkThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kTopkThreads / 32) warp_sums[lane] = s;
  }
  __syncthreads();
  const int base = warp > 0 ? warp_sums[warp - 1] : 0;
  const int tot = warp_sums[kTopkThreads / 32 - 1];
  __syncthreads();
  *total = tot;
  return base + x - v;
}

// Lanes of this warp whose 8-bit `digit` equals this lane's, among the lanes in `m`
// (8 ballots: one per digit bit).
__device__ __forceinline__ unsigned digit_peers(unsigned m, uint32_t digit) {
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const bool bit = (digit >> b) & 1u;
    const unsigned v = __ballot_sync(0xffffffffu, bit);
    m &= bit ? v : ~v;
  }
  return m;
}

constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kHistInts = 256 * kTopkWarps;   // one 256-digit histogram per warp
constexpr int kBuckets = 4096;                // value buckets of the bucket path
constexpr int kMaxBucket = 64;                // a larger selected bucket sends the row to the radix path
static_assert(2 * kHistInts >= 2 * kBuckets, "bucket counts and cursors share the histogram space");

// Bucket of score x: the range [xmin, xmax] cut into kBuckets equal parts.  Subtraction,
// multiplication by a positive scale and truncation are all monotone, so a larger score
// never lands in a lower bucket.
__device__ __forceinline__ int value_bucket(float x, float xmin, float scale) {
  const int b = __float2int_rz((x - xmin) * scale);
  return min(max(b, 0), kBuckets - 1);
}

// Stable sort of the n packed (key << 32 | index) pairs in sel by key, descending, in
// place: least-significant-digit radix sort, 8-bit digits.  Warp w holds positions
// [32 E w, 32 E (w + 1)) in registers (E per lane, in rounds of 32).  Each pass counts the
// digits of every round in the warp's own histogram (ballots give the lanes with the same
// digit, so the rank among them is a popcount and one lane adds their count), scans the
// histograms in (digit, warp) order, which is position order within each digit, and
// scatters.  Equal keys therefore keep their input order.  The histograms are laid out
// [warp][digit] so that different digits fall in different shared-memory banks; the scan
// runs down the columns (thread d owns digit d).  Two histogram buffers alternate: the
// threads that own no digit clear the next pass's buffer during the scan.  Passes over a
// byte in which all keys agree are skipped.  hist holds 2 * kHistInts ints.
template <int E>
__device__ __forceinline__ void radix_sort_desc(unsigned long long* sel, int n, int* hist,
                                                int* warp_sums, uint32_t* s_and_or) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned lt_mask = (1u << lane) - 1u;
  unsigned long long v[E];
  int off[E];
  uint32_t all_and = 0xffffffffu, all_or = 0u;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int p = 32 * E * warp + 32 * r + lane;
    v[r] = p < n ? sel[p] : 0ull;
    if (p < n) {
      all_and &= (uint32_t)(v[r] >> 32);
      all_or |= (uint32_t)(v[r] >> 32);
    }
  }
  if (threadIdx.x == 0) {
    s_and_or[0] = 0xffffffffu;
    s_and_or[1] = 0u;
  }
  for (int i = threadIdx.x; i < kHistInts / 4; i += kTopkThreads)
    reinterpret_cast<int4*>(hist)[i] = make_int4(0, 0, 0, 0);
  __syncthreads();
  all_and = __reduce_and_sync(0xffffffffu, all_and);
  all_or = __reduce_or_sync(0xffffffffu, all_or);
  if (lane == 0) {
    atomicAnd(&s_and_or[0], all_and);
    atomicOr(&s_and_or[1], all_or);
  }
  __syncthreads();
  const uint32_t diff = s_and_or[0] ^ s_and_or[1];
  int buf = 0;
  for (int shift = 0; shift < 32; shift += 8) {
    if (((diff >> shift) & 255u) == 0u) continue;   // uniform
    int* h = hist + buf * kHistInts;
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const bool valid = 32 * E * warp + 32 * r + lane < n;
      // descending order of the key = ascending order of its complement
      const uint32_t d = ((~(uint32_t)(v[r] >> 32)) >> shift) & 255u;
      const unsigned peers = digit_peers(__ballot_sync(0xffffffffu, valid), d);
      const int rank = __popc(peers & lt_mask);
      int old = 0;
      if (valid && rank == 0) old = atomicAdd(&h[warp * 256 + d], __popc(peers));
      old = __shfl_sync(0xffffffffu, old, (__ffs(peers) - 1) & 31);
      off[r] = old + rank;
    }
    __syncthreads();
    {
      int tot = 0;
      if (threadIdx.x < 256) {
#pragma unroll
        for (int w = 0; w < kTopkWarps; ++w) tot += h[w * 256 + threadIdx.x];
      } else {
        int4* z = reinterpret_cast<int4*>(hist + (buf ^ 1) * kHistInts);
        for (int i = threadIdx.x - 256; i < kHistInts / 4; i += kTopkThreads - 256)
          z[i] = make_int4(0, 0, 0, 0);
      }
      int all;
      int run = block_scan(threadIdx.x < 256 ? tot : 0, warp_sums, &all);
      if (threadIdx.x < 256) {
#pragma unroll
        for (int w = 0; w < kTopkWarps; ++w) {
          const int c = h[w * 256 + threadIdx.x];
          h[w * 256 + threadIdx.x] = run;
          run += c;
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < E; ++r) {
      if (32 * E * warp + 32 * r + lane < n) {
        const uint32_t d = ((~(uint32_t)(v[r] >> 32)) >> shift) & 255u;
        sel[h[warp * 256 + d] + off[r]] = v[r];
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int p = 32 * E * warp + 32 * r + lane;
      if (p < n) v[r] = sel[p];
    }
    buf ^= 1;
  }
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads, 2) li_topk_kernel(const TopkArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const bool gmem = a.keys_in_gmem != 0;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);                       // s2_row
  // selected pairs: KP + kMaxBucket packed entries (key << 32 | index in the radix path,
  // key << 32 | ~index in the bucket path)
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(
      smem_raw + (gmem ? 0 : ((a.s2_row * 4 + 15) / 16) * 16));
  __shared__ __align__(16) int hist[2 * kHistInts];
  __shared__ int warp_sums[32];
  __shared__ int s_digit, s_above, s_t;
  __shared__ uint32_t s_and_or[2];
  __shared__ uint32_t s_min[kTopkWarps], s_max[kTopkWarps];
  const int row = blockIdx.x, n2 = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // batch of this query row
  int lo = 0, hi = a.B - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(a.q_row_base + mid) <= row) lo = mid; else hi = mid - 1;
  }
  const int b = lo, s1 = row - __ldg(a.q_row_base + b);
  const int aq = __ldg(a.act_q + b), ak = __ldg(a.act_k + b);
  int lim = visible_limit(s1, aq, ak, a.s2_cap, a.sparse_mode);
  if (a.q_len_dense <= 0 && s1 >= aq) lim = 0;
  lim = min(lim, a.s2_row);
  const float* src = a.scores + ((size_t)row * a.N2 + n2) * a.s2_row;
  int32_t* oi = a.out_idx + ((size_t)row * a.N2 + n2) * a.K;
  T* ov = a.out_val ? static_cast<T*>(a.out_val) + ((size_t)row * a.N2 + n2) * a.K : nullptr;
  // keys into shared memory (when the row fits) and their range
  uint32_t kmn = 0xffffffffu, kmx = 0u;
  for (int i = threadIdx.x; i < lim; i += kTopkThreads) {
    const uint32_t k = order_key(src[i]);
    if (!gmem) keys[i] = k;
    kmn = min(kmn, k);
    kmx = max(kmx, k);
  }
  kmn = __reduce_min_sync(0xffffffffu, kmn);
  kmx = __reduce_max_sync(0xffffffffu, kmx);
  if (lane == 0) {
    s_min[warp] = kmn;
    s_max[warp] = kmx;
  }
  if (threadIdx.x == 0) s_t = 0;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kTopkWarps; ++w) {
    kmn = min(kmn, s_min[w]);
    kmx = max(kmx, s_max[w]);
  }
  // order-preserving key of score i: from shared memory, or from the score row (L2) when
  // the row does not fit
  auto key_at = [&](int i) -> uint32_t { return gmem ? order_key(__ldg(src + i)) : keys[i]; };

  // ---- bucket path: finite scores that are not all equal (uniform decision) ----
  // One histogram of the scores over kBuckets value buckets gives, by a descending scan,
  // the number of scores above each bucket and the bucket t holding the K-th score.  The
  // scores of buckets >= t are scattered bucket by bucket (descending), and each finds its
  // place in its bucket by counting the bucket's entries that order before it by
  // (score desc, index asc); the first K places are the output.  Exact for any input; a
  // selected bucket above kMaxBucket entries (clustered scores) takes the radix path.
  const float xmin = key_float(kmn), xmax = key_float(kmx);
  bool fast = lim > 0 && kmn > 0x007fffffu && kmx < 0xff800000u && kmx > kmn;
  const float scale = fast ? (float)kBuckets / (xmax - xmin) : 0.f;
  fast = fast && scale > 0.f && scale < 3.0e38f;
  if (fast) {
    int* cnt = hist;                 // [kBuckets]
    int* cur = hist + kBuckets;      // [kBuckets]: first place of each bucket, then its end
    for (int i = threadIdx.x; i < kBuckets / 4; i += kTopkThreads)
      reinterpret_cast<int4*>(cnt)[i] = make_int4(0, 0, 0, 0);
    __syncthreads();
    for (int i = threadIdx.x; i < lim; i += kTopkThreads)
      atomicAdd(&cnt[value_bucket(key_float(key_at(i)), xmin, scale)], 1);
    __syncthreads();
    // descending scan: thread t owns buckets [kBuckets - 8 t - 8, kBuckets - 8 t)
    constexpr int kPer = kBuckets / kTopkThreads;
    static_assert(kPer == 8, "two int4 per thread");
    const int b0 = kBuckets - kPer * (int)threadIdx.x - kPer;
    const int4 lo4 = reinterpret_cast<const int4*>(cnt + b0)[0];
    const int4 hi4 = reinterpret_cast<const int4*>(cnt + b0)[1];
    const int c[kPer] = {hi4.w, hi4.z, hi4.y, hi4.x, lo4.w, lo4.z, lo4.y, lo4.x};   // highest first
    int sum = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) sum += c[j];
    int all;
    int run = block_scan(sum, warp_sums, &all);
    const int K = a.K;
    int st[kPer];
    bool big = false;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      st[j] = run;
      if (run < K && run + c[j] >= K) s_t = b0 + kPer - 1 - j;   // the bucket of the K-th score
      big |= run < K && c[j] > kMaxBucket;
      run += c[j];
    }
    reinterpret_cast<int4*>(cur + b0)[0] = make_int4(st[7], st[6], st[5], st[4]);
    reinterpret_cast<int4*>(cur + b0)[1] = make_int4(st[3], st[2], st[1], st[0]);
    fast = !__syncthreads_or(big);
  }
  if (fast) {
    int* cnt = hist;
    int* cur = hist + kBuckets;
    const int K = a.K;
    const int t = s_t;
    for (int i = threadIdx.x; i < lim; i += kTopkThreads) {
      const uint32_t k = key_at(i);
      const int bk = value_bucket(key_float(k), xmin, scale);
      if (bk >= t) sel[atomicAdd(&cur[bk], 1)] = ((unsigned long long)k << 32) | (uint32_t)(~(uint32_t)i);
    }
    __syncthreads();
    const int ntot = cur[t];   // end of bucket t: every scattered entry lies below it
    for (int q = threadIdx.x; q < ntot; q += kTopkThreads) {
      const unsigned long long e = sel[q];
      const int bk = value_bucket(key_float((uint32_t)(e >> 32)), xmin, scale);
      const int end = cur[bk], start = end - cnt[bk];
      int place = start;
      for (int j = start; j < end; ++j) place += sel[j] > e;
      if (place < K) {
        oi[place] = (int32_t)(~(uint32_t)(e & 0xffffffffull));
        if (ov) ov[place] = ElemTraits<T>::from_f(key_float((uint32_t)(e >> 32)));
      }
    }
    for (int j = min(lim, K) + threadIdx.x; j < K; j += kTopkThreads) {
      oi[j] = -1;
      if (ov) ov[j] = ElemTraits<T>::from_f(-INFINITY);
    }
    return;
  }

  // ---- radix path: 4-pass radix select, ordered compaction, stable radix sort ----
  const int K = a.K;
  int nsel;
  if (lim <= K) {
    for (int i = threadIdx.x; i < lim; i += kTopkThreads)
      sel[i] = ((unsigned long long)key_at(i) << 32) | (uint32_t)i;
    nsel = lim;
  } else {
    // radix select: after the 4 passes `prefix` is the key of the K-th largest element
    uint32_t prefix = 0, mask = 0;
    int remaining = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += kTopkThreads) hist[i] = 0;
      __syncthreads();
      // the lanes of a warp with the same digit add their count once (one atomic per
      // distinct digit instead of one per key)
      for (int base = 32 * warp; base < lim; base += kTopkThreads) {
        const int i = base + lane;
        const uint32_t k = i < lim ? key_at(i) : 0u;
        const bool in = i < lim && (k & mask) == prefix;
        const uint32_t d = (k >> shift) & 255u;
        const unsigned m = __ballot_sync(0xffffffffu, in);
        if (m == 0u) continue;   // uniform: no key of this round is still a candidate
        const unsigned peers = digit_peers(m, d);
        if (in && (peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&hist[d], __popc(peers));
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        // digit of the `remaining`-th largest key: lane l sums digits 255-8l .. 248-8l, a
        // warp prefix sum over the lanes (highest digits first) finds the lane, then the digit
        int c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = hist[255 - 8 * lane - j];
          sum += c[j];
        }
        int incl = sum;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += v;
        }
        const bool mine = incl - sum < remaining && remaining <= incl;
        const unsigned found = __ballot_sync(0xffffffffu, mine);   // every lane, before branching
        if (mine) {
          int above = incl - sum, d = 255 - 8 * lane - 7;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (above + c[j] >= remaining) { d = 255 - 8 * lane - j; break; }
            above += c[j];
          }
          s_digit = d;
          s_above = above;
        } else if (found == 0u && lane == 31) {
          s_digit = 0;                 // not reached: `remaining` never exceeds the count
          s_above = incl - c[7];
        }
      }
      __syncthreads();
      // s_digit / s_above are rewritten only after the next pass's two barriers, and every
      // thread has read them by then
      prefix |= (uint32_t)s_digit << shift;
      mask |= 255u << shift;
      remaining -= s_above;
    }
    const uint32_t thr = prefix;
    // ordered compaction: all keys > thr, and the first `remaining` keys == thr by index.
    // Each thread takes a contiguous range, so one block scan orders both classes; the
    // counts are packed as gt | eq << 13 (gt < K <= 4096, eq <= lim <= 2^17, so the block total stays below 2^31).
    const int per = (lim + kTopkThreads - 1) / kTopkThreads;
    const int i0 = min((int)threadIdx.x * per, lim), i1 = min(i0 + per, lim);
    int ngt = 0, neq = 0;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = key_at(i);
      ngt += k > thr;
      neq += k == thr;
    }
    int tot;
    const int pge = block_scan(ngt | (neq << 13), warp_sums, &tot);
    int gpos = pge & 0x1fff, epos = pge >> 13;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = key_at(i);
      const unsigned long long comp = ((unsigned long long)k << 32) | (uint32_t)i;
      if (k > thr) {
        sel[gpos++] = comp;
      } else if (k == thr) {
        if (epos < remaining) sel[(K - remaining) + epos] = comp;
        ++epos;
      }
    }
    nsel = K;
  }
  __syncthreads();
  // The pairs are in ascending index order within each key (keys above the threshold
  // first, then the ties at the threshold), so a stable sort by key, descending, orders
  // them by (score desc, index asc).
  switch ((a.KP + kTopkThreads - 1) / kTopkThreads) {
    case 1: radix_sort_desc<1>(sel, nsel, hist, warp_sums, s_and_or); break;
    case 2: radix_sort_desc<2>(sel, nsel, hist, warp_sums, s_and_or); break;
    case 4: radix_sort_desc<4>(sel, nsel, hist, warp_sums, s_and_or); break;
    default: radix_sort_desc<8>(sel, nsel, hist, warp_sums, s_and_or); break;
  }
  for (int j = threadIdx.x; j < K; j += kTopkThreads) {
    if (j < nsel) {
      const unsigned long long c = sel[j];
      oi[j] = (int32_t)(uint32_t)(c & 0xffffffffull);
      if (ov) ov[j] = ElemTraits<T>::from_f(key_float((uint32_t)(c >> 32)));
    } else {
      oi[j] = -1;
      if (ov) ov[j] = ElemTraits<T>::from_f(-INFINITY);
    }
  }
}

// SMs of the current device (persistent grid), cached per device
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

template <int DP, typename T, int GF>
int launch_score(const CUtensorMap& kmap, const CUtensorMap& qmap, const Args& a,
                 cudaStream_t stream) {
  using C = Cfg<DP>;
  auto k = li_score_kernel<DP, T, GF>;
  const int smem = C::kOffBars + (int)sizeof(Bars);
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return DSA_ERR_CUDA;
  if (a.items > 0) {
    const int grid = a.items < sm_count() ? a.items : sm_count();
    k<<<dim3((unsigned)grid), dim3(kThreads), smem, stream>>>(kmap, qmap, a);
  }
  return DSA_OK;
}

template <int DP, typename T>
int launch(const DsaLiParams* p, cudaStream_t stream) {
  using C = Cfg<DP>;
  const bool bf16 = ElemTraits<T>::kIsBf16;
  const int G = (int)(p->n1 / p->n2);
  const int Tq = 256 / G > 0 ? 256 / G : 0;
  if (Tq < 1) return DSA_ERR_INVALID_ARG;
  const int N = ((Tq * G + 15) / 16) * 16;
  CUtensorMap kmap;
  const int box_rows = p->block_table ? (int)(p->page_size < kKeys ? p->page_size : kKeys) : kKeys;
  // key viewed as {D, N2, kv_rows}; box {one 128-byte chunk, 1, box_rows}
  const uint64_t esz = sizeof(T);
  const bool mapped =
      kIsFp8<T> ? make_tmap_3d_8b(&kmap, p->key, p->d, p->n2, p->kv_rows, (uint64_t)p->d,
                                  (uint64_t)p->n2 * p->d, 128, 1, box_rows)
                : make_tmap_3d_16b(&kmap, p->key, bf16, p->d, p->n2, p->kv_rows, p->d * esz,
                                   (uint64_t)p->n2 * p->d * esz, 64, 1, box_rows);
  if (!mapped) return DSA_ERR_TMA_DESCRIPTOR;
  // query viewed as {D, N1, q_rows}; box {one 128-byte chunk, G heads, Tq tokens}: the
  // (token, head) rows of one item in one load per chunk
  CUtensorMap qmap;
  const bool qmapped =
      kIsFp8<T> ? make_tmap_3d_8b(&qmap, p->query, p->d, p->n1, p->q_rows, (uint64_t)p->d,
                                  (uint64_t)p->n1 * p->d, 128, (uint32_t)G, (uint32_t)Tq)
                : make_tmap_3d_16b(&qmap, p->query, bf16, p->d, p->n1, p->q_rows, p->d * esz,
                                   (uint64_t)p->n1 * p->d * esz, 64, (uint32_t)G, (uint32_t)Tq);
  if (!qmapped) return DSA_ERR_TMA_DESCRIPTOR;
  Args a;
  a.q = p->query;
  a.w = p->weights;
  a.act_q = p->act_q;
  a.act_k = p->act_k;
  a.q_row_base = p->q_row_base;
  a.k_row_base = p->k_row_base;
  a.scores = static_cast<float*>(p->workspace);
  a.err = p->error_flag;
  a.B = (int)p->batch;
  a.N1 = (int)p->n1;
  a.N2 = (int)p->n2;
  a.G = G;
  a.D = (int)p->d;
  a.Tq = Tq;
  a.N = N;
  a.q_rows_max = (int)p->q_len_max;
  a.nblk = (int)((p->q_len_max + Tq - 1) / Tq);
  const int64_t items = (int64_t)p->batch * a.nblk * p->n2;
  if (items > INT32_MAX) return DSA_ERR_INVALID_ARG;
  a.items = (int)items;
  a.s2_row = (int)p->s2_row;
  a.s2_cap = (int)p->s2_cap;
  a.sparse_mode = p->sparse_mode;
  a.w_dtype = p->weights_dtype;
  a.q_len_dense = (int)p->q_len_dense;
  a.block_table = p->block_table;
  a.page = (int)p->page_size;
  a.max_blocks = (int)p->max_blocks;
  a.box_rows = box_rows;
  a.kscale = kIsFp8<T> ? p->key_scale : nullptr;
  int rc;
  if (N == 256 && G == 64) rc = launch_score<DP, T, 64>(kmap, qmap, a, stream);
  else if (N == 256 && G == 32) rc = launch_score<DP, T, 32>(kmap, qmap, a, stream);
  else if (N == 256 && G == 128) rc = launch_score<DP, T, 128>(kmap, qmap, a, stream);
  else rc = launch_score<DP, T, 0>(kmap, qmap, a, stream);
  if (rc != DSA_OK) return rc;

  TopkArgs t;
  t.scores = a.scores;
  t.act_q = p->act_q;
  t.act_k = p->act_k;
  t.q_row_base = p->q_row_base;
  t.out_idx = p->out_indices;
  t.out_val = p->out_values;
  t.err = p->error_flag;
  t.B = (int)p->batch;
  t.N2 = (int)p->n2;
  t.K = (int)p->sparse_count;
  int kp = 1;
  while (kp < t.K) kp <<= 1;
  t.KP = kp;
  t.s2_row = (int)p->s2_row;
  t.s2_cap = (int)p->s2_cap;
  t.sparse_mode = p->sparse_mode;
  t.q_rows = (int)p->q_rows;
  t.q_len_dense = (int)p->q_len_dense;
  // the row's keys stay in shared memory when they fit; longer rows (decode-length key
  // caches) are read from the score matrix in each pass
  const int64_t sel_bytes = (int64_t)(kp + kMaxBucket) * 8;
  const int64_t tsmem_row = ((int64_t)t.s2_row * 4 + 15) / 16 * 16 + sel_bytes;
  t.keys_in_gmem = tsmem_row > 190 * 1024 ? 1 : 0;   // plus 34 KB of static shared memory
  const int tsmem = t.keys_in_gmem ? (int)sel_bytes : (int)tsmem_row;
  // values in the query dtype; fp32 for fp8 queries
  using VT = std::conditional_t<kIsFp8<T>, float, T>;
  if (cudaFuncSetAttribute(li_topk_kernel<VT>, cudaFuncAttributeMaxDynamicSharedMemorySize, tsmem) !=
      cudaSuccess)
    return DSA_ERR_CUDA;
  li_topk_kernel<VT><<<dim3((unsigned)p->q_rows, (unsigned)p->n2), dim3(kTopkThreads), tsmem, stream>>>(t);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

}  // namespace li
}  // namespace dsa

extern "C" int64_t dsa_li_workspace_size(int64_t q_rows, int64_t n2, int64_t s2_row) {
  if (q_rows < 0 || n2 < 1 || s2_row < 0) return -1;
  return 4 * q_rows * n2 * s2_row;
}

extern "C" int dsa_li_score_topk(const DsaLiParams* p, void* stream_) {
  using namespace dsa::li;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!p || !p->query || !p->key || !p->weights || !p->act_q || !p->act_k || !p->q_row_base ||
      (!p->k_row_base && !p->block_table) || !p->out_indices || !p->workspace)
    return DSA_ERR_INVALID_ARG;
  if (p->block_table &&
      (p->max_blocks < 1 || p->page_size < 8 ||
       (p->page_size % kKeys != 0 && kKeys % p->page_size != 0) ||
       p->max_blocks * p->page_size > (int64_t)1 << 30 || p->kv_rows > (int64_t)1 << 30))
    return DSA_ERR_INVALID_ARG;
  if (p->n1 < 1 || p->n2 < 1 || p->n1 % p->n2 != 0 || p->n1 / p->n2 > 256 || p->d < 16 ||
      p->d > 256 || p->d % (p->dtype == DSA_DTYPE_FP8_E4M3 ? 128 : 8) != 0 ||
      (p->dtype == DSA_DTYPE_FP8_E4M3 && !p->key_scale) || p->sparse_count < 1 || p->sparse_count > 4096 ||
      p->sparse_count > p->s2_row || p->s2_row > (1 << 17) || p->batch < 1 || p->kv_rows < 1)
    return DSA_ERR_INVALID_ARG;
  if (p->workspace_bytes < dsa_li_workspace_size(p->q_rows, p->n2, p->s2_row))
    return DSA_ERR_INVALID_ARG;
  if (p->q_rows == 0) return DSA_OK;
  const int dp = p->d <= 64 ? 64 : p->d <= 128 ? 128 : 256;
  if (p->dtype == DSA_DTYPE_BF16) {
    if (dp == 64) return launch<64, __nv_bfloat16>(p, stream);
    if (dp == 128) return launch<128, __nv_bfloat16>(p, stream);
    return launch<256, __nv_bfloat16>(p, stream);
  }
  if (p->dtype == DSA_DTYPE_FP16) {
    if (dp == 64) return launch<64, __half>(p, stream);
    if (dp == 128) return launch<128, __half>(p, stream);
    return launch<256, __half>(p, stream);
  }
  if (p->dtype == DSA_DTYPE_FP8_E4M3) {   // 128 fp8 elements per 128-byte chunk
    if (p->d <= 128) return launch<64, __nv_fp8_e4m3>(p, stream);
    return launch<128, __nv_fp8_e4m3>(p, stream);
  }
  return DSA_ERR_INVALID_ARG;
}
