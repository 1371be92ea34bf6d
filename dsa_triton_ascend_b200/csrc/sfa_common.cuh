// Index handling shared by the sparse flash attention kernels (forward and backward):
// query-row -> batch mapping, the per-entry key mask of the reference kernel, key-row
// translation (dense or paged) and the compaction pre-pass.  The functions are
// templates over the kernel's argument struct, which must provide the fields
// idx, act_q, act_k, q_row_base, k_row_base, block_table, num_rows, B, topk, block,
// kv_rows, page, max_blocks, s2_cap and sparse_mode.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sm100.cuh"

namespace dsa {
namespace sfa {

// Query row -> (batch, position) and the row's visible window.
struct RowInfo {
  int b, s1, aq, ak, threshold;
  bool active;
};

// Row information once the row's batch b is known.
template <class A>
__device__ __forceinline__ RowInfo row_info_in(const A& a, int row, int b) {
  RowInfo ri;
  ri.b = b;
  ri.s1 = row - __ldg(a.q_row_base + b);
  ri.aq = __ldg(a.act_q + b);
  ri.ak = __ldg(a.act_k + b);
  ri.threshold = a.sparse_mode == 0 ? ri.ak : ri.ak - ri.aq + ri.s1 + 1;
  ri.active = ri.s1 < ri.aq && ri.threshold > 0;
  return ri;
}

template <class A>
__device__ __forceinline__ RowInfo row_info(const A& a, int row) {
  int lo = 0, hi = a.B - 1;
  while (lo < hi) {  // last batch whose first row <= row
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(a.q_row_base + mid) <= row) lo = mid; else hi = mid - 1;
  }
  return row_info_in(a, row, lo);
}

// Entry j of the (block-expanded) index row -> key position, or -1 if masked.
// Mask rule: sparse_flash_attention_triton.py:264-266.
template <class A>
__device__ __forceinline__ int key_at(const A& a, const RowInfo& ri, const int32_t* row_idx, int j) {
  int blk = __ldg(row_idx + j / a.block);
  if (blk < 0) return -1;
  int t = blk * a.block + (j % a.block);
  if (t >= ri.threshold || t >= ri.ak || t >= a.s2_cap) return -1;
  if (a.block_table) {  // keys in unmapped pages are dropped (see key_row)
    int pb = __ldg(a.block_table + (size_t)ri.b * a.max_blocks + t / a.page);
    if (pb < 0 || (long long)pb * a.page >= a.kv_rows) return -1;
  }
  return t;
}

// Key position -> row of the key/key_rope matrices.
template <class A>
__device__ __forceinline__ int key_row(const A& a, int b, int t) {
  if (a.block_table) {
    int blk = __ldg(a.block_table + (size_t)b * a.max_blocks + t / a.page);
    return blk * a.page + t % a.page;
  }
  return __ldg(a.k_row_base + b) + t;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bar.sync is the aligned form: the whole warp must arrive converged, so converge it first
// (a lane that left a wait early, e.g. after a timeout, rejoins here)
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  __syncwarp();
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// One warp per query row: compact the row's valid key positions (block-expanded,
// masked as in sparse_flash_attention_triton.py:264-266) into key-matrix rows, in
// index order, plus their count.  The attention kernel then streams 64 rows per tile
// with one coalesced load and no per-tile scanning.
template <class A>
__global__ void __launch_bounds__(128) sfa_prep_kernel(const A a, int32_t* ws_rows, int32_t* ws_count) {
  griddep_launch_dependents();   // a forward launched as our dependent may start its set-up
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= a.num_rows) return;
  const RowInfo ri = row_info(a, row);
  const int nent = a.topk * a.block;
  int have = 0;
  if (ri.active) {
    const int32_t* row_idx = a.idx + (size_t)row * a.topk;
    int32_t* out = ws_rows + (size_t)row * nent;
    for (int base = 0; base < nent; base += 32) {
      const int j = base + lane;
      const int kp = j < nent ? key_at(a, ri, row_idx, j) : -1;
      const unsigned m = __ballot_sync(0xffffffffu, kp >= 0);
      if (kp >= 0) out[have + __popc(m & ((1u << lane) - 1u))] = key_row(a, ri.b, kp);
      have += __popc(m);
    }
  }
  if (lane == 0) ws_count[row] = have;
}


// The same compaction with one 512-thread block per query row, for calls with few rows
// (decode): the warp-per-row kernel would walk a 2048-entry row in 64 dependent steps
// (index, then page table) on a handful of SMs.  The block finds the row's batch with one
// parallel look at the row-base table (no dependent search), then each thread resolves
// kPrepPer consecutive entries at once (their loads in flight together) and one block
// scan of the per-thread counts places them in index order; rows longer than
// 512 * kPrepPer entries take several such rounds.
constexpr int kPrepBlockThreads = 512;
constexpr int kPrepPer = 8;

template <class A>
__global__ void __launch_bounds__(kPrepBlockThreads, 1) sfa_prep_block_kernel(const A a, int32_t* ws_rows,
                                                                           int32_t* ws_count) {
  constexpr int kWarps = kPrepBlockThreads / 32;
  __shared__ int warp_sums[kWarps];
  __shared__ int s_batch;
  griddep_launch_dependents();   // a forward launched as our dependent may start its set-up
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) s_batch = 0;
  __syncthreads();
  // the last batch whose first row <= row: the one with base <= row < next base
  for (int b = threadIdx.x; b < a.B; b += kPrepBlockThreads) {
    const int base = __ldg(a.q_row_base + b);
    const int next = b + 1 < a.B ? __ldg(a.q_row_base + b + 1) : 0x7fffffff;
    if (base <= row && row < next) s_batch = b;
  }
  __syncthreads();
  const RowInfo ri = row_info_in(a, row, s_batch);
  const int nent = ri.active ? a.topk * a.block : 0;
  const int32_t* row_idx = a.idx + (size_t)row * a.topk;
  int32_t* out = ws_rows + (size_t)row * a.topk * a.block;
  int done = 0;   // entries written by the previous rounds (uniform)
  for (int r0 = 0; r0 < nent; r0 += kPrepBlockThreads * kPrepPer) {
    const int j0 = r0 + threadIdx.x * kPrepPer;
    int kr[kPrepPer];
    int have = 0;
#pragma unroll
    for (int e = 0; e < kPrepPer; ++e) {
      const int kp = j0 + e < nent ? key_at(a, ri, row_idx, j0 + e) : -1;
      kr[e] = kp >= 0 ? key_row(a, ri.b, kp) : -1;
      have += kp >= 0;
    }
    // block exclusive scan of `have` (thread order = entry order)
    int x = have;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int v = warp_sums[w];
      before += w < warp ? v : 0;
      total += v;
    }
    int pos = done + before + x - have;
#pragma unroll
    for (int e = 0; e < kPrepPer; ++e)
      if (kr[e] >= 0) out[pos++] = kr[e];
    done += total;
    __syncthreads();   // warp_sums is rewritten by the next round
  }
  if (threadIdx.x == 0) ws_count[row] = done;
}

// Compaction pre-pass for `num_rows` rows: one block per row when there are few rows,
// one warp per row otherwise.
template <class A>
inline void launch_prep(const A& a, int32_t* ws_rows, int32_t* ws_count, int64_t num_rows,
                        cudaStream_t stream) {
  if (num_rows <= 1024)
    sfa_prep_block_kernel<A><<<dim3((unsigned)num_rows), dim3(kPrepBlockThreads), 0, stream>>>(
        a, ws_rows, ws_count);
  else
    sfa_prep_kernel<A><<<dim3((unsigned)((num_rows + 3) / 4)), dim3(128), 0, stream>>>(
        a, ws_rows, ws_count);
}

}  // namespace sfa
}  // namespace dsa
