// Dense lightning-indexer KL loss for sm_100a: the indexer loss over every visible key of a
// query row (no top-k).
//
// Replaces the reference's dense path (dense_loss_backward_triton.py): the index softmax
// statistics `_dense_indexer_stats_kernel` (:129-179), the loss `_dense_loss_kernel`
// (:263-320), dQueryIndex / dWeights `_dense_main_grad_kernel` (:182-260) and the dKeyIndex
// scatter `_dense_dkey_index_kernel` (:323-397).
//
//   I_k  = sum_g w_g ReLU(qi_g . ki_k)                       (index score of key k)
//   p_k  = (1/N1) sum_h exp(scale (q_h . k_k + qr_h . kr_k) - max_h) / (sum_h + 1e-8)
//   st_k = exp(I_k - max I) / max(sum I, 1e-8);  dI_k = st_k - p_k
//   loss += sum_k max(p,1e-8) (log max(p,1e-8) - log max(st,1e-8))
//   dW_g = sum_k dI_k ReLU(qi_g . ki_k);  dQI_g = sum_k dI_k w_g [qi_g . ki_k > 0] ki_k
//   dKI_k += sum_g dI_k w_g [qi_g . ki_k > 0] qi_g
//
// Kernels (256 threads, a warp per key or per index head; dot products are split over the
// lanes in 16-byte pieces and summed with shuffles):
//   dense_stats_kernel   one CTA per row: I_k of the visible keys, online max / sum.
//   dense_teacher_kernel one CTA per row: I_k, p_k, dI_k (kept in the workspace for the
//                        next kernel), the KL term and the key's dKeyIndex row (fp32
//                        reductions into an accumulator).
//   dense_qi_kernel      one CTA per (row, 8 index heads): dWeights and dQueryIndex.
//   dense_cast_kernel    dKeyIndex accumulator -> key_index dtype.
// No tensor cores: one query row against its keys is matrix-vector shaped, and the shapes the
// reference's tests exercise are small.  This is the first, correctness-first version of
// this path.

#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_b200.h"
#include "sm100.cuh"

namespace dsa {
namespace dense {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxNi = 128;        // index heads
constexpr int kMaxDi = 512;        // index head dim
constexpr int kCh = kMaxDi / 8 / 32;   // 16-byte pieces of an index row per lane
constexpr float kEps = 1e-8f;

struct Args {
  const void* q;      // [B*S1][N1][D]
  const void* k;      // [B*S2][N2][D]
  const void* qr;     // [B*S1][N1][dr] or NULL
  const void* kr;     // [B*S2][N2][dr] or NULL
  const void* qi;     // [B*S1][Ni][Di]
  const void* ki;     // [B*S2][Di]
  const void* w;      // [B*S1][Ni]
  const float* smax;  // [B][N2][S1][G]
  const float* ssum;
  float* imax;        // [B*S1]
  float* isum;
  const int32_t* act_q;
  const int32_t* act_k;
  float* di;          // [B*S1][S2] workspace
  float* dki_acc;     // [B*S2][Di] workspace
  void* dqi;          // [B*S1][Ni][Di]
  void* dki;          // [B*S2][Di]
  void* dw;           // [B*S1][Ni]
  float* loss;
  int B, S1, S2, N1, N2, D, dr, Ni, Di, w_dtype;
  float scale;
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = ElemTraits<T>::to_f(e[i]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x . y over n elements (n a multiple of 8, both 16-byte aligned), summed into every lane
template <typename T>
__device__ __forceinline__ float warp_dot(const T* x, const T* y, int n, int lane) {
  float acc = 0.f;
  for (int c = lane; c < n / 8; c += 32) {
    float a[8], b[8];
    load8(x + 8 * c, a);
    load8(y + 8 * c, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(a[i], b[i], acc);
  }
  return warp_sum(acc);
}

template <typename T>
__device__ __forceinline__ float load_w(const void* w, int dtype, size_t i) {
  if (dtype == DSA_DTYPE_FP32) return static_cast<const float*>(w)[i];
  return ElemTraits<T>::to_f(static_cast<const T*>(w)[i]);
}

// visible keys of a BSND row (s1 < act_q; s2 < min(max(act_k - act_q + s1 + 1, 0), S2))
__device__ __forceinline__ int visible(const Args& a, int row, int* b_out) {
  const int b = row / a.S1, s1 = row - b * a.S1;
  *b_out = b;
  const int aq = __ldg(a.act_q + b), ak = __ldg(a.act_k + b);
  if (s1 >= aq) return 0;
  return min(max(ak - aq + s1 + 1, 0), a.S2);
}

// the row's index queries (Ni x Di) into shared memory, weights as fp32
template <typename T>
__device__ __forceinline__ void stage_row(const Args& a, int row, T* qs, float* ws) {
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(a.qi) + (size_t)row * a.Ni * a.Di);
  uint4* dst = reinterpret_cast<uint4*>(qs);
  for (int i = threadIdx.x; i < a.Ni * a.Di / 8; i += kThreads) dst[i] = src[i];
  for (int g = threadIdx.x; g < a.Ni; g += kThreads) ws[g] = load_w<T>(a.w, a.w_dtype, (size_t)row * a.Ni + g);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) dense_stats_kernel(const Args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* qs = reinterpret_cast<T*>(smem_raw);
  float* ws = reinterpret_cast<float*>(qs + a.Ni * a.Di);
  __shared__ float wm[kWarps], wsum[kWarps];
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b;
  const int vis = visible(a, row, &b);
  stage_row<T>(a, row, qs, ws);
  __syncthreads();
  const T* ki = static_cast<const T*>(a.ki);
  float m = -INFINITY, s = 0.f;
  for (int key = warp; key < vis; key += kWarps) {
    const T* kk = ki + (size_t)(b * a.S2 + key) * a.Di;
    float I = 0.f;
    for (int g = 0; g < a.Ni; ++g) I = fmaf(ws[g], fmaxf(warp_dot(qs + g * a.Di, kk, a.Di, lane), 0.f), I);
    const float mn = fmaxf(m, I);
    s = s * expf(m - mn) + expf(I - mn);
    m = mn;
  }
  if (lane == 0) {
    wm[warp] = m;
    wsum[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int i = 0; i < kWarps; ++i) M = fmaxf(M, wm[i]);
    float S = 0.f;
    for (int i = 0; i < kWarps; ++i)
      if (wm[i] != -INFINITY) S += wsum[i] * expf(wm[i] - M);
    a.imax[row] = vis > 0 ? M : -INFINITY;
    a.isum[row] = vis > 0 ? S : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) dense_teacher_kernel(const Args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* qs = reinterpret_cast<T*>(smem_raw);
  float* ws = reinterpret_cast<float*>(qs + a.Ni * a.Di);
  float* dots = ws + kMaxNi;                    // [kWarps][kMaxNi]
  float* hm = dots + kWarps * kMaxNi;           // [N1] attention max of this row
  float* hs = hm + a.N1;                        // [N1] attention sum
  __shared__ float kls[kWarps];
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b;
  const int vis0 = visible(a, row, &b);
  const float im = a.imax[row], isu = a.isum[row];
  const int vis = (vis0 > 0 && isu > 0.f) ? vis0 : 0;   // rows without a student contribute 0
  const int G = a.N1 / a.N2, s1 = row - b * a.S1;
  stage_row<T>(a, row, qs, ws);
  for (int h = threadIdx.x; h < a.N1; h += kThreads) {
    const size_t si = ((size_t)(b * a.N2 + h / G) * a.S1 + s1) * G + h % G;
    hm[h] = a.smax[si];
    hs[h] = a.ssum[si];
  }
  __syncthreads();
  const T* q = static_cast<const T*>(a.q) + (size_t)row * a.N1 * a.D;
  const T* qr = a.dr > 0 ? static_cast<const T*>(a.qr) + (size_t)row * a.N1 * a.dr : nullptr;
  const T* kb = static_cast<const T*>(a.k);
  const T* krb = static_cast<const T*>(a.kr);
  const T* ki = static_cast<const T*>(a.ki);
  const float inv_isum = 1.f / fmaxf(isu, kEps);
  float* wd = dots + warp * kMaxNi;
  float kl = 0.f;
  for (int key = warp; key < vis; key += kWarps) {
    const size_t krow = (size_t)b * a.S2 + key;
    const T* kk = ki + krow * a.Di;
    float I = 0.f;
    for (int g = 0; g < a.Ni; ++g) {
      const float d = warp_dot(qs + g * a.Di, kk, a.Di, lane);
      if (lane == 0) wd[g] = d;
      I = fmaf(ws[g], fmaxf(d, 0.f), I);
    }
    float p = 0.f;
    for (int h = 0; h < a.N1; ++h) {
      const size_t kh = krow * a.N2 + h / G;
      float s = warp_dot(q + (size_t)h * a.D, kb + kh * a.D, a.D, lane);
      if (qr) s += warp_dot(qr + (size_t)h * a.dr, krb + kh * a.dr, a.dr, lane);
      p += expf(s * a.scale - hm[h]) / (hs[h] + kEps);
    }
    p *= 1.f / (float)a.N1;
    const float st = expf(I - im) * inv_isum;
    const float dI = st - p;
    if (lane == 0) {
      a.di[(size_t)row * a.S2 + key] = dI;
      const float pc = fmaxf(p, kEps), sc = fmaxf(st, kEps);
      kl += pc * (logf(pc) - logf(sc));
    }
    __syncwarp();
    // dKeyIndex row of this key: sum_g dI w_g [dot_g > 0] qi_g, lane-owned 16-byte pieces
    float acc[kCh][8];
#pragma unroll
    for (int j = 0; j < kCh; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[j][i] = 0.f;
    for (int g = 0; g < a.Ni; ++g) {
      if (!(wd[g] > 0.f)) continue;               // warp-uniform (one shared value)
      const float c = dI * ws[g];
#pragma unroll
      for (int j = 0; j < kCh; ++j) {
        const int ch = lane + 32 * j;
        if (ch < a.Di / 8) {
          float f[8];
          load8(qs + g * a.Di + 8 * ch, f);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[j][i] = fmaf(c, f[i], acc[j][i]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int ch = lane + 32 * j;
      if (ch < a.Di / 8) {
        float* dst = a.dki_acc + krow * a.Di + 8 * ch;
#pragma unroll
        for (int i = 0; i < 8; ++i) atomicAdd(dst + i, acc[j][i]);
      }
    }
    __syncwarp();
  }
  if (lane == 0) kls[warp] = kl;
  __syncthreads();
  if (threadIdx.x == 0 && vis > 0) {
    float t = 0.f;
    for (int i = 0; i < kWarps; ++i) t += kls[i];
    atomicAdd(a.loss, t);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) dense_qi_kernel(const Args a) {
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.y * kWarps + warp;
  if (g >= a.Ni) return;                          // whole warps; no block barrier below
  int b;
  const int vis0 = visible(a, row, &b);
  const int vis = (vis0 > 0 && a.isum[row] > 0.f) ? vis0 : 0;
  const T* qg = static_cast<const T*>(a.qi) + ((size_t)row * a.Ni + g) * a.Di;
  const T* ki = static_cast<const T*>(a.ki);
  const float wg = load_w<T>(a.w, a.w_dtype, (size_t)row * a.Ni + g);
  float qv[kCh][8], acc[kCh][8];
#pragma unroll
  for (int j = 0; j < kCh; ++j) {
    const int ch = lane + 32 * j;
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[j][i] = acc[j][i] = 0.f;
    if (ch < a.Di / 8) load8(qg + 8 * ch, qv[j]);
  }
  float dw = 0.f;
  for (int key = 0; key < vis; ++key) {
    const T* kk = ki + ((size_t)b * a.S2 + key) * a.Di;
    float kv[kCh][8];
    float part = 0.f;
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int ch = lane + 32 * j;
#pragma unroll
      for (int i = 0; i < 8; ++i) kv[j][i] = 0.f;
      if (ch < a.Di / 8) load8(kk + 8 * ch, kv[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) part = fmaf(qv[j][i], kv[j][i], part);
    }
    const float d = warp_sum(part);
    const float dI = a.di[(size_t)row * a.S2 + key];
    dw = fmaf(dI, fmaxf(d, 0.f), dw);
    if (d > 0.f) {
      const float c = dI * wg;
#pragma unroll
      for (int j = 0; j < kCh; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[j][i] = fmaf(c, kv[j][i], acc[j][i]);
    }
  }
  T* out = static_cast<T*>(a.dqi) + ((size_t)row * a.Ni + g) * a.Di;
#pragma unroll
  for (int j = 0; j < kCh; ++j) {
    const int ch = lane + 32 * j;
    if (ch < a.Di / 8) {
      uint4 u;
      u.x = ElemTraits<T>::pack2(acc[j][0], acc[j][1]);
      u.y = ElemTraits<T>::pack2(acc[j][2], acc[j][3]);
      u.z = ElemTraits<T>::pack2(acc[j][4], acc[j][5]);
      u.w = ElemTraits<T>::pack2(acc[j][6], acc[j][7]);
      *reinterpret_cast<uint4*>(out + 8 * ch) = u;
    }
  }
  if (lane == 0) {
    const size_t wi = (size_t)row * a.Ni + g;
    if (a.w_dtype == DSA_DTYPE_FP32) static_cast<float*>(a.dw)[wi] = dw;
    else static_cast<T*>(a.dw)[wi] = ElemTraits<T>::from_f(dw);
  }
}

template <typename T>
__global__ void dense_cast_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = ElemTraits<T>::from_f(src[i]);
}

inline int64_t di_bytes(int64_t rows, int64_t s2) { return (rows * s2 * 4 + 255) / 256 * 256; }

inline Args make_args(const DsaDenseIndexerParams* p) {
  Args a;
  a.q = p->query;
  a.k = p->key;
  a.qr = p->d_rope > 0 ? p->query_rope : nullptr;
  a.kr = p->d_rope > 0 ? p->key_rope : nullptr;
  a.qi = p->query_index;
  a.ki = p->key_index;
  a.w = p->weights;
  a.smax = p->softmax_max;
  a.ssum = p->softmax_sum;
  a.imax = p->index_max;
  a.isum = p->index_sum;
  a.act_q = p->act_q;
  a.act_k = p->act_k;
  a.di = static_cast<float*>(p->workspace);
  a.dki_acc = p->workspace
                  ? reinterpret_cast<float*>(static_cast<char*>(p->workspace) + di_bytes(p->batch * p->s1, p->s2))
                  : nullptr;
  a.dqi = p->d_query_index;
  a.dki = p->d_key_index;
  a.dw = p->d_weights;
  a.loss = p->loss;
  a.B = (int)p->batch;
  a.S1 = (int)p->s1;
  a.S2 = (int)p->s2;
  a.N1 = (int)p->n1;
  a.N2 = (int)p->n2;
  a.D = (int)p->d;
  a.dr = (int)p->d_rope;
  a.Ni = (int)p->n_index;
  a.Di = (int)p->d_index;
  a.w_dtype = p->weights_dtype;
  a.scale = p->scale;
  return a;
}

inline bool index_args_ok(const DsaDenseIndexerParams* p) {
  return p && p->query_index && p->key_index && p->weights && p->act_q && p->act_k &&
         p->index_max && p->index_sum && p->batch >= 1 && p->s1 >= 1 && p->s2 >= 1 &&
         p->n_index >= 1 && p->n_index <= kMaxNi && p->d_index >= 8 && p->d_index <= kMaxDi &&
         p->d_index % 8 == 0 && p->batch * p->s1 < (int64_t)1 << 31 &&
         p->batch * p->s2 < (int64_t)1 << 31 &&
         (p->dtype == DSA_DTYPE_BF16 || p->dtype == DSA_DTYPE_FP16) &&
         (p->weights_dtype == DSA_DTYPE_FP32 || p->weights_dtype == p->dtype);
}

template <typename T>
int launch_lse(const DsaDenseIndexerParams* p, cudaStream_t stream) {
  const Args a = make_args(p);
  const int smem = (int)(p->n_index * p->d_index * 2 + p->n_index * 4);
  if (cudaFuncSetAttribute(dense_stats_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return DSA_ERR_CUDA;
  dense_stats_kernel<T><<<dim3((unsigned)(p->batch * p->s1)), dim3(kThreads), smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

template <typename T>
int launch_grad(const DsaDenseIndexerParams* p, cudaStream_t stream) {
  const Args a = make_args(p);
  const int64_t rows = p->batch * p->s1;
  const int64_t nki = p->batch * p->s2 * p->d_index;
  if (cudaMemsetAsync(a.dki_acc, 0, (size_t)nki * 4, stream) != cudaSuccess ||
      cudaMemsetAsync(p->loss, 0, sizeof(float), stream) != cudaSuccess)
    return DSA_ERR_CUDA;
  const int smem = (int)(p->n_index * p->d_index * 2 + (kMaxNi + kWarps * kMaxNi + 2 * p->n1) * 4);
  if (cudaFuncSetAttribute(dense_teacher_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return DSA_ERR_CUDA;
  dense_teacher_kernel<T><<<dim3((unsigned)rows), dim3(kThreads), smem, stream>>>(a);
  dense_qi_kernel<T><<<dim3((unsigned)rows, (unsigned)((p->n_index + kWarps - 1) / kWarps)), dim3(kThreads), 0,
                       stream>>>(a);
  if (p->d_key_index)
    dense_cast_kernel<T><<<dim3(1184), dim3(256), 0, stream>>>(a.dki_acc, static_cast<T*>(p->d_key_index), nki);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

}  // namespace dense
}  // namespace dsa

extern "C" int64_t dsa_dense_indexer_workspace_size(int64_t batch, int64_t s1, int64_t s2, int64_t d_index) {
  if (batch < 0 || s1 < 0 || s2 < 0 || d_index < 0) return -1;
  return dsa::dense::di_bytes(batch * s1, s2) + batch * s2 * d_index * 4;
}

extern "C" int dsa_dense_indexer_softmax_lse(const DsaDenseIndexerParams* p, void* stream) {
  using namespace dsa::dense;
  if (!index_args_ok(p)) return DSA_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == DSA_DTYPE_BF16 ? launch_lse<__nv_bfloat16>(p, s) : launch_lse<__half>(p, s);
}

extern "C" int dsa_dense_indexer_grad_kl_loss(const DsaDenseIndexerParams* p, void* stream) {
  using namespace dsa::dense;
  if (!index_args_ok(p) || !p->query || !p->key || !p->softmax_max || !p->softmax_sum ||
      !p->d_query_index || !p->d_weights || !p->loss || !p->workspace)
    return DSA_ERR_INVALID_ARG;
  if (p->n1 < 1 || p->n2 < 1 || p->n1 % p->n2 != 0 || p->n1 > 1024 || p->d < 8 || p->d % 8 != 0 ||
      (p->d_rope != 0 && p->d_rope != 64) || (p->d_rope > 0 && (!p->query_rope || !p->key_rope)))
    return DSA_ERR_INVALID_ARG;
  if (p->workspace_bytes < dsa_dense_indexer_workspace_size(p->batch, p->s1, p->s2, p->d_index))
    return DSA_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == DSA_DTYPE_BF16 ? launch_grad<__nv_bfloat16>(p, s) : launch_grad<__half>(p, s);
}
