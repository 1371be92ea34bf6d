// Sparse flash attention forward for sm_100a (tcgen05, CTA pairs).
//
// Replaces the reference launch core `_sfa_core` / `_sfa_kernel`
// (sparse_flash_attention_triton.py:189-332, :445-477).
//
// Work decomposition: one CTA pair (cluster of 2) per query token.  The 2-SM UMMA
// with M=128 gives each CTA 64 of the 128 query heads (rows) while both CTAs feed
// half of the B operand:
//   * QK^T : B = gathered keys, split by token (CTA r owns tokens [32r, 32r+32) of
//            each 64-token tile, all 576 latent+rope dims)      -> "X" ring (2 tiles)
//   * P V  : B = V (= key[:, :D]) split by head dim (CTA r provides D/2 dims for
//            all 64 tokens of the tile)                          -> "H" ring (2 tiles)
// Every key row crosses L2 -> SM once: each CTA gathers only its own 32 tokens into X
// (TMA gather4 in the 2-SM form, so the bytes of both CTAs are counted on the leader's
// barrier), and once QK^T of the tile is done, two copy warps move the V slices out of X
// -- its own tokens' slices into its own H, the partner's slices straight into the
// partner's H (distributed shared memory stores) -- instead of gathering the partner's
// tokens again.  Copies are done by threads, not by the TMA unit, because there they
// would queue behind the gathers.  P and H are double-buffered so that the slow
// cross-CTA signals (a cluster-scope arrive waits for the CTA's in-flight TMA traffic)
// overlap the next tile instead of stalling it.
// S (64 heads x 64 tokens) and O (64 heads x D) live in TMEM in the 2x2 layout of
// the M=128 pair MMA: lanes 0-63 hold the first half of the columns, lanes 64-127
// the second half.  Valid indices are compacted by sfa_prep_kernel, so causal rows
// with fewer than topK visible keys only pay for their valid keys.
//
// Warp roles (512 threads): warps 0 and 6 copy X -> H (warp 0 first loads Q; at D = 512
// they take alternate tiles, otherwise both copy every tile); warp 1
// issues UMMA (pair leader) and owns TMEM; warps 2-5 run the online softmax, the lazy O
// rescale and the epilogue; warps 7-15 gather the QK^T keys with TMA gather4, one 64-dim
// chunk each.  Rows with few keys per SM (decode) are split into key ranges whose fp32
// partials sfa_fwd_combine_kernel merges.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "dsa_b200.h"
#include "sm100.cuh"
#include "sfa_common.cuh"
#include "tma_host.h"

namespace dsa {
namespace sfa_fwd {

using namespace dsa::sfa;

constexpr int kTile = 64;          // keys per pair tile
constexpr int kOwn = 32;           // keys per CTA in the QK B operand
constexpr int kHeads = 64;         // heads per CTA
constexpr int kChunkBytesX = kOwn * 128;     // one 64-dim chunk of 32 own keys
constexpr int kChunkBytesH = kOwn * 128;     // one 64-dim chunk of 32 keys (a token half)
constexpr int kLoadWarp0 = 7;
// TMA gather4 issuers, one per 64-dim chunk: a thread issues one gather4 every ~100
// cycles and the lanes of a warp take turns, so a stage is issued about as fast as one
// warp issues its 8 gathers only when every chunk has its own warp
constexpr int kLoadWarps = 9;
constexpr int kCopyThreads = 64;             // warps 0 and 6
constexpr int kThreads = 32 * (kLoadWarp0 + kLoadWarps);
constexpr float kRescaleLog2 = 8.0f;         // lazy rescale threshold (log2 units)

template <int D>
struct Cfg {
  static constexpr int kNopeChunks = D / 64;
  static constexpr int kChunks = kNopeChunks + 1;          // + rope
  static constexpr int kNPV = D < 256 ? D : 256;           // N of one PV MMA (both CTAs)
  static constexpr int kNumPV = D / kNPV;                  // PV MMAs per k-step
  static constexpr int kCpj = kNPV / 128;                  // chunks per CTA per PV MMA
  static constexpr int kSlots = kNopeChunks / 2;           // V chunks per CTA
  static constexpr int kQBytes = kChunks * kHeads * 128;
  static constexpr int kXBytes = kChunks * kChunkBytesX;
  static constexpr int kHHalf = kSlots * kChunkBytesH;
  static constexpr int kHBytes = 2 * kHHalf;
  static constexpr int kPBytes = kHeads * 128;
  // smem carve-up (from a 1 KiB aligned base)
  static constexpr int kOffQ = 0;
  static constexpr int kOffX = kOffQ + kQBytes;
  static constexpr int kOffH = kOffX + 2 * kXBytes;
  static constexpr int kOffP = kOffH + 2 * kHBytes;
  static constexpr int kOffBars = kOffP + 2 * kPBytes;
  // the Bars struct follows at kOffBars; total = kOffBars + sizeof(Bars)
  static constexpr int kTmemO = 256;                        // O columns start
  static constexpr int kTmemCols = 512;
  // the own-token X chunk that fills V slot `sl` of CTA `c`
  static __device__ __forceinline__ int slot_chunk(int sl, int c) {
    return (sl / kCpj) * 2 * kCpj + c * kCpj + sl % kCpj;
  }
};

struct __align__(64) Maps {
  CUtensorMap q;    // [rows*N1, D], box 64 x 64
  CUtensorMap qr;   // [rows*N1, 64], box 64 x 64
  CUtensorMap k;    // [kv_rows, D], box 64 x 1 (gather4)
  CUtensorMap kr;   // [kv_rows, 64], box 64 x 1
};

struct Args {
  const int32_t* idx;
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  const int32_t* k_row_base;
  const int32_t* block_table;
  void* out;
  float* smax;
  float* ssum;
  int* err;
  const void* key;          // [kv_rows][D]
  const void* key_rope;     // [kv_rows][64]
  const int32_t* ws_rows;   // [num_rows][nent] compacted key-matrix rows (prep kernel)
  const int32_t* ws_count;  // [num_rows] number of valid keys per query row
  int num_rows, B, N1, topk, block, kv_rows, page, max_blocks, s2_cap, sparse_mode;
  float scale;
  // key splits per query row (1: the kernel writes out / softmax_max / softmax_sum itself;
  // > 1: CTA pair p = row * splits + split handles tiles [split * T / splits, ...) of its
  // row and writes a normalised fp32 partial O and {m_ref, m_run, l} for the combine kernel)
  int splits;
  float* part_o;    // [num_rows * splits][N1][D]
  float4* part_s;   // [num_rows * splits][N1]
};

// Barrier protocol (t = tile, b = t & 1 selects the X stage, H slot, S and P buffer):
//   x_full[b]   (leader) bytes of both CTAs' gathers of tile t: X ready for QK^T
//   x_empty[b]  (each CTA) QK^T(t) done and this CTA's copy warps have read X(t)
//   s_full[b]   QK^T(t) commit, both CTAs: S ready (and X(t) read by the tensor core)
//   h_full[b]   (leader) both CTAs' copy warps finished the H slot of tile t
//   p_full[b]   (leader) both CTAs wrote P(t)
//   pv_done[b]  PV(t) commit, both CTAs: O updated, P buffer and H slot b free again
struct __align__(16) Bars {
  uint64_t q_full;
  uint64_t x_full[2], x_empty[2], s_full[2], h_full[2], p_full[2], pv_done[2];
  uint32_t tmem_slot;
  float red_max[2][4][32];
  float red_sum[4][32];
};


template <int D, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    sfa_fwd_kernel(const __grid_constant__ Maps maps, const Args a) {
  using C = Cfg<D>;
  // All shared state is dynamic (no static smem), so the window starts 1 KiB aligned
  // as the 128-byte swizzle atoms require; checked below.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Bars& bars = *reinterpret_cast<Bars*>(smem_raw + C::kOffBars);
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t sQ = sbase + C::kOffQ, sX = sbase + C::kOffX, sH = sbase + C::kOffH,
                 sP = sbase + C::kOffP;
  uint8_t* gP = smem_raw + C::kOffP;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sbase & 1023u) {  // identical in both CTAs of the pair, so both leave together
    if (threadIdx.x == 0) report_error(a.err, kErrMisaligned);
    return;
  }
  const uint32_t cta = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int row = pair / a.splits;
  const int split = pair - row * a.splits;
  const RowInfo ri = row_info(a, row);

  // Set-up first: this kernel is launched as a programmatic dependent of the compaction
  // pass, so barriers and TMEM are ready while that pass finishes.
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars.q_full), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bars.x_full[b]), 1);
      mbar_init(smem_u32(&bars.x_empty[b]), 1);
      mbar_init(smem_u32(&bars.s_full[b]), 1);
      mbar_init(smem_u32(&bars.h_full[b]), 2);
      mbar_init(smem_u32(&bars.p_full[b]), 2);
      mbar_init(smem_u32(&bars.pv_done[b]), 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(smem_u32(&bars.tmem_slot), C::kTmemCols);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_slot;
  bool failed = false;

  // the compaction pass's results (and any error it recorded) are visible from here on
  griddep_wait();
  griddep_launch_dependents();   // the split-combine kernel may start staging
  // Valid keys of this row, compacted by sfa_prep_kernel (identical in both CTAs).
  // A CTA that finds an earlier error recorded skips its row, so one protocol failure
  // does not turn into a slow cascade of timeouts over the whole grid.
  const bool abort = a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0;
  const int nvalid_row = (ri.active && !abort) ? __ldg(a.ws_count + row) : 0;
  const int ntiles_row = (nvalid_row + kTile - 1) / kTile;
  // this pair's tiles [t0, t1) of the row (all of them unless the row is split)
  const int t0 = (int)((int64_t)split * ntiles_row / a.splits);
  const int t1 = (int)((int64_t)(split + 1) * ntiles_row / a.splits);
  const int ntiles = t1 - t0;
  const int nvalid = ntiles > 0 ? min(nvalid_row - kTile * t0, kTile * ntiles) : 0;
  const int32_t* rows = a.ws_rows + (size_t)row * a.topk * a.block + (size_t)kTile * t0;

  if (warp == 0 || warp == 6) {
    // ====== warp 0: Q of this CTA's 64 heads (once); warps 0 and 6: X -> H copies ======
    if (warp == 0 && ntiles > 0) {
      const uint32_t lead_q = mapa_shared(smem_u32(&bars.q_full), 0);
      if (cta == 0 && lane == 0) mbar_arrive_expect_tx(smem_u32(&bars.q_full), 2 * C::kQBytes);
      __syncwarp();
      const int qrow0 = row * a.N1 + kHeads * (int)cta;
      if (lane < C::kChunks) {
        const CUtensorMap* m = lane < C::kNopeChunks ? &maps.q : &maps.qr;
        int x = lane < C::kNopeChunks ? 64 * lane : 0;
        tma_load_2d_pair(sQ + lane * kHeads * 128, m, lead_q, x, qrow0);
      }
    }
    // D = 512: warp 0 copies the even tiles and warp 6 the odd ones, so a tile's copy and
    // its release arrive overlap the next tile's (2.7 % faster at config 4; at D = 128 the
    // shorter copies gain nothing and both warps share every tile)
    constexpr bool kAlt = D == 512;
    constexpr int kCT = kAlt ? 32 : kCopyThreads;        // copy threads of one tile
    const int ci = kAlt ? lane : (warp == 0 ? 0 : 32) + lane;
    const uint32_t peer = cta ^ 1u;
    const uint32_t lead_h0 = mapa_shared(smem_u32(&bars.h_full[0]), 0);
    const uint32_t lead_h1 = mapa_shared(smem_u32(&bars.h_full[1]), 0);
    for (int t = kAlt && warp == 6 ? 1 : 0; t < ntiles; t += kAlt ? 2 : 1) {
      const int b = t & 1;
      const uint32_t ph = (uint32_t)(t >> 1) & 1u;
      // QK^T(t) done (so X(t) landed in both CTAs) and PV(t-2) done (H slot b free in
      // both CTAs: one pair MMA)
      mbar_wait_spin(smem_u32(&bars.s_full[b]), ph, a.err, &failed);
      mbar_wait_spin(smem_u32(&bars.pv_done[b]), ph ^ 1u, a.err, &failed);
      if (!failed) {
        const uint32_t xs = C::kOffX + b * C::kXBytes;
        const uint32_t hs = C::kOffH + b * C::kHBytes + cta * C::kHHalf;   // my tokens' half
#pragma unroll
        for (int sl = 0; sl < C::kSlots; ++sl) {
          const uint32_t src_own = xs + C::slot_chunk(sl, cta) * kChunkBytesX;
          const uint32_t src_peer = xs + C::slot_chunk(sl, peer) * kChunkBytesX;
          const uint32_t dst = hs + sl * kChunkBytesH;
#pragma unroll
          for (int hh = 0; hh < kChunkBytesH / 16 / kCT / 4; ++hh) {   // 4 own + 4 peer in flight
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int o = 16 * (ci + kCT * (4 * hh + j));
              v[j] = *reinterpret_cast<const uint4*>(smem_raw + src_own + o);
              v[4 + j] = *reinterpret_cast<const uint4*>(smem_raw + src_peer + o);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int o = 16 * (ci + kCT * (4 * hh + j));
              *reinterpret_cast<uint4*>(smem_raw + dst + o) = v[j];
              st_cluster_v4(mapa_shared(sbase + dst + o, peer), v[4 + j]);
            }
          }
        }
      }
      fence_proxy_async_smem();
      asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
      if constexpr (kAlt)
        __syncwarp();
      else
        named_bar_sync(2, kCopyThreads);
      if (ci == 0) {
        mbar_arrive(smem_u32(&bars.x_empty[b]));             // X(t) read: refill it
        mbar_arrive_cluster(b ? lead_h1 : lead_h0);           // H slot b of tile t written
      }
    }
  } else if (warp >= kLoadWarp0) {
    // ====== X loaders: own 32 keys x all dims for QK^T, TMA gather4 (4 keys x 128 B) ======
    // warp w issues chunk w (D < 512: some warps idle), lanes 0-7 the chunk's 8 gathers; the bytes
    // of both CTAs are counted on the leader's x_full, so no thread waits for the data.
    const int wq = warp - kLoadWarp0;
    const int filler = nvalid > 0 ? __ldg(rows) : 0;
    for (int t = 0; t < ntiles && !failed; ++t) {
      const int b = t & 1;
      const int j = kTile * t + kOwn * (int)cta + lane;
      const int my_row = j < nvalid ? __ldg(rows + j) : filler;
      int r4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) r4[e] = __shfl_sync(0xffffffffu, my_row, 4 * (lane & 7) + e);
      mbar_wait_spin(smem_u32(&bars.x_empty[b]), ((uint32_t)(t >> 1) & 1u) ^ 1u, a.err, &failed);
      if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
      const uint32_t full = smem_u32(&bars.x_full[b]);
      if (cta == 0 && wq == 0 && lane == 0) mbar_arrive_expect_tx(full, 2 * C::kXBytes);
      if (lane < 8) {
        const uint32_t lead = mapa_shared(full, 0);
        for (int c = wq; c < C::kChunks; c += kLoadWarps) {
          const CUtensorMap* m = c < C::kNopeChunks ? &maps.k : &maps.kr;
          tma_gather4_pair(sX + b * C::kXBytes + c * kChunkBytesX + lane * 512, m, lead,
                           c < C::kNopeChunks ? 64 * c : 0, r4[0], r4[1], r4[2], r4[3]);
        }
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ================ MMA issuer (pair leader): the whole warp runs the loop =================
    // (waits included) and one elected lane issues each tcgen05 instruction; a single lane
    // running the loop alone issues the MMAs much more slowly (5.9 against 7.8 ms at config 4)
    if (cta == 0 && ntiles > 0) {
      const bool bf16 = ElemTraits<T>::kIsBf16;
      const uint32_t id_qk = idesc_f16(128, kTile, bf16, false, false);
      const uint32_t id_pv = idesc_f16(128, C::kNPV, bf16, false, true);
      mbar_wait_spin(smem_u32(&bars.q_full), 0, a.err, &failed);
      const uint64_t dq = smem_desc_sw128(sQ, 16, 1024);
      const uint64_t dx0 = smem_desc_sw128(sX, 16, 1024);
      const uint64_t dp0 = smem_desc_sw128(sP, 16, 1024);
      const uint64_t dh0 = smem_desc_sw128(sH, kChunkBytesH, 1024);
      auto issue_qk = [&](int t) {
        const int b = t & 1;
        mbar_wait_spin(smem_u32(&bars.x_full[b]), (uint32_t)(t >> 1) & 1u, a.err, &failed, true);
        if (__any_sync(0xffffffffu, failed)) { failed = true; return; }
        tc_fence_after();
        const uint32_t d = tmem + 32 * b;
        const uint64_t bx = dx0 + (uint64_t)((b * C::kXBytes) >> 4);
        if (elect_one()) {
#pragma unroll
          for (int c = 0; c < C::kChunks; ++c)
#pragma unroll
            for (int u = 0; u < 4; ++u)
              umma_f16<2>(d, dq + (uint64_t)((c * kHeads * 128 + u * 32) >> 4),
                          bx + (uint64_t)((c * kChunkBytesX + u * 32) >> 4), id_qk, (c | u) != 0);
          umma_commit_pair(smem_u32(&bars.s_full[b]), 3);
        }
        __syncwarp();
      };
      if (!failed) issue_qk(0);
      for (int t = 0; t < ntiles && !failed; ++t) {
        if (t + 1 < ntiles) issue_qk(t + 1);
        const int b = t & 1;
        const uint32_t par = (uint32_t)(t >> 1) & 1u;
        mbar_wait_spin(smem_u32(&bars.p_full[b]), par, a.err, &failed, true);
        mbar_wait_spin(smem_u32(&bars.h_full[b]), par, a.err, &failed, true);
        if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
        tc_fence_after();
        const uint64_t dp = dp0 + (uint64_t)((b * C::kPBytes) >> 4);
        const uint64_t dh = dh0 + (uint64_t)((b * C::kHBytes) >> 4);
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < C::kNumPV; ++j)
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k)
              umma_f16<2>(tmem + C::kTmemO + j * (C::kNPV / 2), dp + (uint64_t)((k * 32) >> 4),
                          dh + (uint64_t)(((k >> 1) * C::kHHalf + j * C::kCpj * kChunkBytesH +
                                           (k & 1) * 2048) >> 4),
                          id_pv, (t | k) != 0);
          umma_commit_pair(smem_u32(&bars.pv_done[b]), 3);
        }
        __syncwarp();
      }
    }
    __syncwarp();
  } else {
    // ================= softmax / correction / epilogue (both CTAs) =================
    const int q = warp & 3;                  // TMEM lane quadrant of this warp
    const int hrow = 32 * (q & 1) + lane;    // head within the CTA (P row)
    const int half = q >> 1;                 // key half of the tile / O column half
    const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
    const float c2 = a.scale * 1.4426950408889634f;
    const uint32_t lead_p0 = mapa_shared(smem_u32(&bars.p_full[0]), 0);
    const uint32_t lead_p1 = mapa_shared(smem_u32(&bars.p_full[1]), 0);
    float m_run = -INFINITY, m_ref = -INFINITY, l_part = 0.f;

    for (int t = 0; t < ntiles; ++t) {
      const int s = t & 1;
      const uint32_t par = (t >> 1) & 1;
      const int nv = min(kTile, nvalid - kTile * t) - kOwn * half;   // valid keys in my half
      mbar_wait_spin(smem_u32(&bars.s_full[s]), par, a.err, &failed);
      bool wfail = __any_sync(0xffffffffu, failed);                  // warp-uniform
      tc_fence_after();
      uint32_t r[32];
      float mloc = -INFINITY;
      if (!wfail) {
        tmem_ld32(tmem + lane_addr + 32 * s, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nv) mloc = fmaxf(mloc, __uint_as_float(r[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      bars.red_max[s][q][lane] = mloc;
      named_bar_sync(1, 128);
      const float mpart = bars.red_max[s][q ^ 2][lane];
      const float mnew = fmaxf(m_run, fmaxf(mloc, mpart));
      m_run = mnew;
      // Lazy rescale: the exponent reference m_ref only moves when the running max
      // exceeds it by more than 2^8; partner threads (same head) decide identically.
      bool rescale = false;
      float factor = 1.f;
      if (t == 0) {
        m_ref = mnew;
      } else if ((mnew - m_ref) * c2 > kRescaleLog2) {
        rescale = true;
        factor = ex2((m_ref - mnew) * c2);
        m_ref = mnew;
      }
      const float off = m_ref * c2;
      l_part *= factor;   // earlier tiles' sum onto the new reference (factor 1 unless rescaling)
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float p0 = (2 * i < nv) ? ex2(fmaf(__uint_as_float(r[2 * i]), c2, -off)) : 0.f;
        float p1 = (2 * i + 1 < nv) ? ex2(fmaf(__uint_as_float(r[2 * i + 1]), c2, -off)) : 0.f;
        l_part += p0 + p1;
        pk[i] = ElemTraits<T>::pack2(p0, p1);
      }
      // P buffer s was last read by PV(t-2); O may be touched only once PV(t-1) is done.
      if (t >= 2) mbar_wait_spin(smem_u32(&bars.pv_done[s]), par ^ 1u, a.err, &failed);
      if (__any_sync(0xffffffffu, rescale)) {
        if (t >= 1)
          mbar_wait_spin(smem_u32(&bars.pv_done[s ^ 1]), (uint32_t)((t - 1) >> 1) & 1u, a.err, &failed);
        if (!__any_sync(0xffffffffu, failed)) {
          tc_fence_after();
          for (int cc = 0; cc < D / 2; cc += 16) {
            uint32_t o[16];
            tmem_ld16(tmem + lane_addr + C::kTmemO + cc, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st16(tmem + lane_addr + C::kTmemO + cc, o);
          }
          tmem_st_wait();
        }
      }
      uint8_t* prow = gP + s * C::kPBytes + hrow * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int chunk = 4 * half + i;
        uint4 v = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        *reinterpret_cast<uint4*>(prow + ((chunk ^ (hrow & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(1, 128);
      if (warp == 2 && lane == 0) {
        if (cta == 0) mbar_arrive(smem_u32(&bars.p_full[s]));   // leader: a local arrive
        else mbar_arrive_cluster(s ? lead_p1 : lead_p0);
      }
    }

    // ------------------------------ epilogue ------------------------------
    bars.red_sum[q][lane] = l_part;
    if (ntiles > 0) {
      const int tl = ntiles - 1;
      mbar_wait_spin(smem_u32(&bars.pv_done[tl & 1]), (uint32_t)(tl >> 1) & 1u, a.err, &failed);
    }
    const bool read_o = ntiles > 0 && !__any_sync(0xffffffffu, failed);
    named_bar_sync(1, 128);
    const float l_tot = l_part + bars.red_sum[q ^ 2][lane];
    const int head = kHeads * (int)cta + hrow;
    const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
    tc_fence_after();
    T* orow = reinterpret_cast<T*>(a.out) + ((size_t)row * a.N1 + min(head, a.N1 - 1)) * D;
    for (int j = 0; j < C::kNumPV; ++j) {
      const int dbase = j * C::kNPV + half * (C::kNPV / 2);
      for (int cc = 0; cc < C::kNPV / 2; cc += 32) {
        uint32_t o[32];
        if (read_o) {
          tmem_ld32(tmem + lane_addr + C::kTmemO + j * (C::kNPV / 2) + cc, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (head < a.N1 && a.splits > 1) {
          // split row: normalised fp32 partial for the combine kernel
          float4* dst = reinterpret_cast<float4*>(a.part_o + ((size_t)pair * a.N1 + head) * D + dbase + cc);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            dst[v] = make_float4(__uint_as_float(o[4 * v + 0]) * inv, __uint_as_float(o[4 * v + 1]) * inv,
                                 __uint_as_float(o[4 * v + 2]) * inv, __uint_as_float(o[4 * v + 3]) * inv);
        } else if (head < a.N1) {
          uint4* dst = reinterpret_cast<uint4*>(orow + dbase + cc);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = ElemTraits<T>::pack2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            dst[v] = w;
          }
        }
      }
    }
    if (head < a.N1 && half == 0 && a.splits > 1) {
      const bool any = ntiles > 0 && l_tot > 0.f;
      a.part_s[(size_t)pair * a.N1 + head] =
          make_float4(any ? m_ref : -INFINITY, any ? m_run : -INFINITY, any ? l_tot : 0.f, 0.f);
    } else if (head < a.N1 && half == 0 && a.smax != nullptr) {
      const bool any = ntiles > 0;
      a.smax[(size_t)row * a.N1 + head] = any ? m_run * a.scale : 0.f;
      a.ssum[(size_t)row * a.N1 + head] = any ? l_tot * ex2((m_ref - m_run) * c2) : 0.f;
    }
  }

  // ------------------------------ teardown ------------------------------
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, C::kTmemCols);
}

// Merge the key splits of each (row, head): weights w_s = l_s 2^((m_ref_s - M) c2) with
// M = the largest m_ref, O = sum_s w_s O_s / sum_s w_s (O_s normalised by l_s), and the
// statistics of the whole row: max = the largest m_run, sum = sum_s l_s 2^((m_ref_s - max) c2).
// One warp per (row, head); lane l owns columns 4l + 128i.
template <int D, typename T>
__global__ void __launch_bounds__(256) sfa_fwd_combine_kernel(const float* __restrict__ part_o,
                                                              const float4* __restrict__ part_s,
                                                              T* __restrict__ out, float* smax,
                                                              float* ssum, int num_rows, int n1,
                                                              int splits, float scale) {
  griddep_wait();   // launched as a programmatic dependent of the forward: its partials
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (gw >= num_rows * n1) return;
  const int row = gw / n1, h = gw - row * n1;
  const float c2 = scale * 1.4426950408889634f;
  float mref = -INFINITY, mrun = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) {
    const float4 st = __ldg(part_s + ((size_t)row * splits + sp) * n1 + h);
    if (st.z > 0.f) {
      mref = fmaxf(mref, st.x);
      mrun = fmaxf(mrun, st.y);
    }
  }
  constexpr int kV = D / 128;
  float4 acc[kV];
#pragma unroll
  for (int i = 0; i < kV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f, lsum = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    const size_t ps = ((size_t)row * splits + sp) * n1 + h;
    const float4 st = __ldg(part_s + ps);
    if (!(st.z > 0.f)) continue;
    const float w = st.z * ex2((st.x - mref) * c2);
    wsum += w;
    lsum += st.z * ex2((st.x - mrun) * c2);
    const float4* o = reinterpret_cast<const float4*>(part_o + ps * D);
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const float4 v = __ldg(o + lane + 32 * i);
      acc[i].x += w * v.x;
      acc[i].y += w * v.y;
      acc[i].z += w * v.z;
      acc[i].w += w * v.w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  T* orow = out + ((size_t)row * n1 + h) * D;
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    uint2 pk;
    pk.x = ElemTraits<T>::pack2(acc[i].x * inv, acc[i].y * inv);
    pk.y = ElemTraits<T>::pack2(acc[i].z * inv, acc[i].w * inv);
    *reinterpret_cast<uint2*>(orow + 4 * (lane + 32 * i)) = pk;
  }
  if (lane == 0 && smax != nullptr) {
    const bool any = wsum > 0.f;
    smax[(size_t)row * n1 + h] = any ? mrun * scale : 0.f;
    ssum[(size_t)row * n1 + h] = any ? lsum : 0.f;
  }
}

// Few query rows (decode) leave most SMs idle with one CTA pair per row; such rows are
// split into key ranges so that up to kSplitPairs pairs (one CTA per SM on 148 SMs) run at
// once, each with at least 4 tiles, when the workspace holds the partial results.
constexpr int kSplitPairs = 74;

inline int fwd_splits(int64_t num_rows, int64_t nent) {
  if (num_rows <= 0 || num_rows >= kSplitPairs) return 1;
  const int64_t ntiles = (nent + kTile - 1) / kTile;
  int64_t sp = kSplitPairs / num_rows;
  const int64_t cap = ntiles / 4 > 1 ? ntiles / 4 : 1;
  if (sp > cap) sp = cap;
  return sp > 1 ? (int)sp : 1;
}

inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// workspace layout: compaction (key rows, counts), then the split partials when split
inline int64_t compaction_bytes(int64_t num_rows, int64_t nent) { return 4 * (num_rows * nent + num_rows); }
inline int64_t partial_bytes(int64_t num_rows, int splits, int64_t n1, int64_t d) {
  return splits > 1 ? num_rows * splits * n1 * (d + 4) * 4 : 0;
}

template <int D>
constexpr int smem_bytes() { return Cfg<D>::kOffBars + (int)sizeof(Bars); }
static_assert(smem_bytes<512>() <= 232448, "D=512 smem budget (227 KiB per block)");

template <int D, typename T>
int launch(const DsaSfaFwdParams* p, cudaStream_t stream) {
  using C = Cfg<D>;
  const bool bf16 = ElemTraits<T>::kIsBf16;
  Maps maps;
  const uint64_t qrows = (uint64_t)p->num_rows * p->n1;
  if (!make_tmap_2d_16b(&maps.q, p->q, bf16, qrows, D, (uint64_t)D * 2, 64, 64) ||
      !make_tmap_2d_16b(&maps.qr, p->q_rope, bf16, qrows, 64, 128, 64, 64) ||
      !make_tmap_2d_16b(&maps.k, p->key, bf16, p->kv_rows, D, (uint64_t)D * 2, 64, 1) ||
      !make_tmap_2d_16b(&maps.kr, p->key_rope, bf16, p->kv_rows, 64, 128, 64, 1))
    return DSA_ERR_TMA_DESCRIPTOR;
  Args a;
  a.idx = p->sparse_indices;
  a.key = p->key;
  a.key_rope = p->key_rope;
  a.act_q = p->act_q;
  a.act_k = p->act_k;
  a.q_row_base = p->q_row_base;
  a.k_row_base = p->k_row_base;
  a.block_table = p->block_table;
  a.out = p->out;
  a.smax = p->softmax_max;
  a.ssum = p->softmax_sum;
  a.err = p->error_flag;
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
  a.ws_rows = static_cast<const int32_t*>(p->workspace);
  a.ws_count = static_cast<const int32_t*>(p->workspace) + (size_t)p->num_rows * p->topk * p->sparse_block_size;
  const int64_t nent = p->topk * p->sparse_block_size;
  int splits = fwd_splits(p->num_rows, nent);
  const int64_t part_off = align256(compaction_bytes(p->num_rows, nent));
  if (splits > 1 && p->workspace_bytes < part_off + partial_bytes(p->num_rows, splits, p->n1, D))
    splits = 1;   // the caller's workspace has no room for the partials: one pair per row
  a.splits = splits;
  a.part_o = splits > 1 ? reinterpret_cast<float*>(static_cast<char*>(p->workspace) + part_off) : nullptr;
  a.part_s = splits > 1 ? reinterpret_cast<float4*>(a.part_o + (size_t)p->num_rows * splits * p->n1 * D)
                        : nullptr;
  launch_prep(a, const_cast<int32_t*>(a.ws_rows), const_cast<int32_t*>(a.ws_count), p->num_rows,
              stream);
  auto kern = sfa_fwd_kernel<D, T>;
  constexpr int kSmem = smem_bytes<D>();
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return DSA_ERR_CUDA;
  // the forward and the split combine are programmatic dependents of the kernel before them
  // (each waits for its predecessor's results before reading them), so their launch and
  // set-up overlap the predecessor's tail; with few rows (decode) that latency is a
  // sizeable part of the call
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)(p->num_rows * splits));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, maps, a) != cudaSuccess) return DSA_ERR_CUDA;
  if (splits > 1) {
    const int64_t warps = p->num_rows * p->n1;
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3((unsigned)((warps + 7) / 8));
    cc.blockDim = dim3(256);
    cc.stream = stream;
    cc.attrs = pdl;
    cc.numAttrs = 1;
    if (cudaLaunchKernelEx(&cc, sfa_fwd_combine_kernel<D, T>, static_cast<const float*>(a.part_o),
                           static_cast<const float4*>(a.part_s), static_cast<T*>(p->out),
                           p->softmax_max, p->softmax_sum, (int)p->num_rows, (int)p->n1, splits,
                           p->scale) != cudaSuccess)
      return DSA_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

}  // namespace sfa_fwd
}  // namespace dsa

extern "C" int dsa_sfa_fwd(const DsaSfaFwdParams* p, void* stream_) {
  using namespace dsa::sfa_fwd;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!p) return DSA_ERR_INVALID_ARG;
  if (p->num_rows <= 0) return DSA_OK;
  if (p->n1 < 1 || p->n1 > 128 || p->batch < 1 || p->topk < 1 || p->sparse_block_size < 1 ||
      p->kv_rows < 1 || !p->q || !p->q_rope || !p->key || !p->key_rope || !p->sparse_indices ||
      !p->act_q || !p->act_k || !p->q_row_base || !p->out)
    return DSA_ERR_INVALID_ARG;
  if (!p->block_table && !p->k_row_base) return DSA_ERR_INVALID_ARG;
  if (!p->workspace || p->workspace_bytes < (int64_t)dsa_sfa_fwd_workspace_size(p->num_rows, p->topk, p->sparse_block_size))
    return DSA_ERR_INVALID_ARG;
  if (p->block_table && (p->page_size < 1 || p->max_blocks < 1)) return DSA_ERR_INVALID_ARG;
  if ((p->softmax_max == nullptr) != (p->softmax_sum == nullptr)) return DSA_ERR_INVALID_ARG;
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

extern "C" int64_t dsa_sfa_fwd_workspace_size(int64_t num_rows, int64_t topk, int64_t sparse_block_size) {
  if (num_rows < 0 || topk < 0 || sparse_block_size < 1) return -1;
  return dsa::sfa_fwd::compaction_bytes(num_rows, topk * sparse_block_size);
}

extern "C" int64_t dsa_sfa_fwd_fast_workspace_size(int64_t num_rows, int64_t n1, int64_t d, int64_t topk,
                                                   int64_t sparse_block_size) {
  using namespace dsa::sfa_fwd;
  if (num_rows < 0 || n1 < 1 || d < 1 || topk < 0 || sparse_block_size < 1) return -1;
  const int64_t nent = topk * sparse_block_size;
  const int splits = fwd_splits(num_rows, nent);
  if (splits <= 1) return compaction_bytes(num_rows, nent);
  return align256(compaction_bytes(num_rows, nent)) + partial_bytes(num_rows, splits, n1, d);
}

// ---------------------------------------------------------------------------------------
// dsa_sfa_fwd_noalloc: the forward for callers that cannot allocate device memory when
// they run attention (a serving runtime whose KV-cache pool took all free HBM at
// start-up, or a plain C/C++ host with no allocator of its own that may not call
// cudaMalloc on its hot path).  The only device memory dsa_sfa_fwd needs besides the
// caller's inputs and outputs is its workspace (the compaction, plus the key-split
// partials of few-row calls); here that workspace is the file-scope array below, so the
// call allocates nothing.
//
// The array lives in every GPU that loads this module, for as long as the process runs.
// Its name is only a host-side handle: the device address is looked up with
// cudaGetSymbolAddress, with the device current, by the first call in each CUDA context
// (a device's primary context, or a context a driver-API host made itself), and cached
// under that context's unique id -- an address is valid only in the context it was looked
// up in, and a context created later (after cudaDeviceReset, say) gets a new id and a new
// lookup.  That first call should therefore come before any stream capture.  All calls in
// a context share the array and it keeps the last call's contents.  It holds the
// compaction workspace and, for calls with few query rows (decode), the fp32 key-split
// partials when they fit (otherwise such calls run unsplit); no entry has to start at
// zero, because sfa_prep_kernel writes the count of every query row and the key rows below
// each count, and every split writes its whole partial, before anything reads them.
// Calls that overlap on the GPU (different streams, no ordering) race on the array.

static __device__ __align__(256) int32_t g_sfa_fwd_noalloc_scratch[DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES / 4];

namespace {

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct NoAllocEntry {
  unsigned long long ctx_id;
  void* addr;
};
constexpr int kNoAllocEntries = 64;
std::mutex g_noalloc_mu;
NoAllocEntry g_noalloc[kNoAllocEntries] = {};
int g_noalloc_next = 0;

// Unique id of the calling thread's current CUDA context (false if there is none or the
// driver does not provide the entry points).
bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool tried = false;
  if (!tried) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    tried = true;
  }
  CUcontext ctx = nullptr;
  if (!get_cur || !get_id || get_cur(&ctx) != CUDA_SUCCESS || !ctx) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of the scratch array in the current context (looked up on first use in
// that context; without a context id it is looked up on every call).
int noalloc_scratch_address(void** addr) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  unsigned long long id = 0;
  bool have_id = current_context_id(&id);
  if (have_id)
    for (const NoAllocEntry& e : g_noalloc)
      if (e.addr && e.ctx_id == id) {
        *addr = e.addr;
        return DSA_OK;
      }
  void* a = nullptr;
  if (cudaGetSymbolAddress(&a, g_sfa_fwd_noalloc_scratch) != cudaSuccess || !a) return DSA_ERR_CUDA;
  if (!have_id) have_id = current_context_id(&id);   // the lookup made the primary context current
  if (have_id) {
    g_noalloc[g_noalloc_next] = NoAllocEntry{id, a};
    g_noalloc_next = (g_noalloc_next + 1) % kNoAllocEntries;
  }
  *addr = a;
  return DSA_OK;
}

}  // namespace

extern "C" int dsa_sfa_fwd_noalloc(const DsaSfaFwdParams* p, void* stream) {
  if (!p) return DSA_ERR_INVALID_ARG;
  if (p->num_rows <= 0) return DSA_OK;
  const int64_t need = dsa_sfa_fwd_workspace_size(p->num_rows, p->topk, p->sparse_block_size);
  if (need < 0) return DSA_ERR_INVALID_ARG;
  if (need > DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES) return DSA_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const int rc = noalloc_scratch_address(&scratch);
  if (rc != DSA_OK) return rc;
  DsaSfaFwdParams q = *p;
  q.workspace = scratch;
  q.workspace_bytes = DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES;
  return dsa_sfa_fwd(&q, stream);
}
