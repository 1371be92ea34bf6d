/*
 * dsa_b200.h -- C ABI of libdsa_b200.so, the sm_100a kernels of the DeepSeek Sparse
 * Attention hot path.
 *
 * Plain pointers and sizes only.  Every tensor argument is a device pointer to a
 * contiguous buffer; every entry point is asynchronous on `stream` (a cudaStream_t
 * passed as void*; NULL = legacy default stream) and returns DSA_OK or an error code
 * without synchronising.  Kernels that detect a problem on the device (a bounded
 * wait that gave up) set bits in `*error_flag` (may be NULL); callers read it after
 * synchronising.
 *
 * Each entry point replaces the launch layer of one reference operator of
 * 18851871668/dsa_triton_ascend (file:line of the reference project given below).
 * Layout normalisation (BSND / TND / PA_BSND), argument guards and output allocation
 * stay in the host wrapper (dsa_triton_ascend_b200/*.py), as in the reference.
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSA_OK 0
#define DSA_ERR_INVALID_ARG 1     /* bad size / null pointer / unsupported config */
#define DSA_ERR_CUDA 2            /* launch or attribute error from the CUDA runtime */
#define DSA_ERR_TMA_DESCRIPTOR 3  /* driver rejected a TMA tensor map (alignment) */
#define DSA_ERR_TOO_LARGE 4       /* request exceeds a fixed in-library scratch array */

#define DSA_DTYPE_BF16 0
#define DSA_DTYPE_FP16 1
#define DSA_DTYPE_FP32 2
#define DSA_DTYPE_FP8_E4M3 3      /* lightning indexer only (dsa_li_score_topk) */

/* Library version, (major << 16) | minor. */
int dsa_version(void);

/*
 * Sparse flash attention forward (MLA-absorb: value = key[..., :d]).
 * Replaces `_sfa_core` / `_sfa_kernel` (sparse_flash_attention_triton.py:445-477, :189-332).
 *
 * Query side is addressed by "query rows" r in [0, num_rows): one query token each.
 *   q           [num_rows][n1][d]      bf16/fp16, d in {128, 256, 512}
 *   q_rope      [num_rows][n1][64]
 *   sparse_indices [num_rows][topk]    int32 block ids (token ids when
 *                                      sparse_block_size == 1), -1 = padding
 *   q_row_base  [batch]                first query row of each batch (BSND: b*S1,
 *                                      TND: cumulative offsets); row r belongs to the
 *                                      last batch whose base <= r, position s1 = r - base
 *   act_q, act_k [batch]               valid query / key lengths
 * Key side: `kv_rows` rows of key [kv_rows][d] and key_rope [kv_rows][64].
 *   Dense (block_table == NULL): key position t of batch b is row k_row_base[b] + t.
 *   Paged (block_table != NULL, [batch][max_blocks]): row block_table[b][t / page_size]
 *     * page_size + t % page_size; keys in pages whose id is < 0 are skipped.
 * A key position t is attended iff t < threshold, t < act_k[b] and t < s2_cap, with
 * threshold = act_k[b] (sparse_mode 0) or act_k[b] - act_q[b] + s1 + 1 (sparse_mode 3);
 * rows with s1 >= act_q[b] or threshold <= 0 produce zeros.
 * Outputs: out [num_rows][n1][d] (query dtype); softmax_max / softmax_sum
 *   [num_rows][n1] fp32 (both NULL to skip): max of scaled scores and sum of
 *   exp(score - max); rows without keys get 0.
 */
typedef struct DsaSfaFwdParams {
  const void* q;
  const void* q_rope;
  const void* key;
  const void* key_rope;
  const int32_t* sparse_indices;
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  const int32_t* k_row_base;     /* dense layout only */
  const int32_t* block_table;    /* paged layout only, else NULL */
  void* out;
  float* softmax_max;
  float* softmax_sum;
  int* error_flag;
  void* workspace;               /* dsa_sfa_fwd_workspace_size() bytes, caller-owned */
  int64_t workspace_bytes;
  int64_t num_rows;
  int64_t batch;
  int64_t n1;
  int64_t d;
  int64_t topk;
  int64_t sparse_block_size;
  int64_t kv_rows;
  int64_t page_size;
  int64_t max_blocks;
  int64_t s2_cap;                /* exclusive upper bound on key positions */
  float scale;
  int32_t sparse_mode;           /* 0 or 3 */
  int32_t dtype;                 /* DSA_DTYPE_* of q/q_rope/key/key_rope/out */
} DsaSfaFwdParams;

int dsa_sfa_fwd(const DsaSfaFwdParams* params, void* stream);

/* Workspace of dsa_sfa_fwd: the compacted key rows of every query row (int32
 * [num_rows][topk * sparse_block_size]) and their counts (int32 [num_rows]).
 * Returns -1 for invalid sizes. */
int64_t dsa_sfa_fwd_workspace_size(int64_t num_rows, int64_t topk, int64_t sparse_block_size);

/* Workspace with which dsa_sfa_fwd may split the keys of few-row calls (fewer query rows
 * than CTA pairs the GPU runs at once, e.g. decode) over several CTA pairs per row and
 * merge their fp32 partial results in a second kernel: dsa_sfa_fwd_workspace_size() plus
 * room for the partials (num_rows * splits * n1 * (d + 4) floats) when it would split,
 * else exactly dsa_sfa_fwd_workspace_size().  dsa_sfa_fwd accepts any workspace of at
 * least dsa_sfa_fwd_workspace_size() bytes and splits only when the partials fit.
 * Returns -1 for invalid sizes. */
int64_t dsa_sfa_fwd_fast_workspace_size(int64_t num_rows, int64_t n1, int64_t d, int64_t topk,
                                        int64_t sparse_block_size);

/*
 * Sparse flash attention forward that allocates nothing.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when they run
 * attention -- a serving runtime that has handed all free HBM to its KV-cache pool
 * at start-up, or a host program that owns no allocator of its own (no torch, no
 * pool) and may not call cudaMalloc on its hot path.
 *
 * Same parameters and results as dsa_sfa_fwd, except that `workspace` and
 * `workspace_bytes` are ignored: the workspace is a fixed array of
 * DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads
 * the library's forward module holds until the process exits.  It holds the
 * compaction of the index rows and, for calls with few query rows (decode), the fp32
 * partial results of the key splits, up to DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES in all; a
 * few-row call whose partials do not fit beside the compaction runs unsplit instead.
 *   - Calls whose dsa_sfa_fwd_workspace_size(num_rows, topk, sparse_block_size)
 *     exceeds DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES return DSA_ERR_TOO_LARGE and launch
 *     nothing (split the query rows into several calls, or use dsa_sfa_fwd).
 *   - The first call in a CUDA context looks up that context's copy of the array (with
 *     the device current) and caches its address under the context's unique id; the
 *     address is valid only in that context, so a new context (after cudaDeviceReset,
 *     or one a driver-API host creates) gets its own lookup.  Make that first call
 *     before any stream capture begins.
 *   - Every call in a context shares the one array and it keeps the last call's
 *     contents.  Nothing in it has to start at zero (each call writes every entry it
 *     later reads), but calls that overlap on the GPU -- on different streams without
 *     ordering between them -- race on it (compaction and partials alike) and give
 *     wrong results.
 * Calls no cudaMalloc, cudaFree or other allocating routine.
 */
#define DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES (16LL << 20)
int dsa_sfa_fwd_noalloc(const DsaSfaFwdParams* params, void* stream);

/*
 * Sparse flash attention backward (MLA-absorb).
 * Replaces `_sfa_grad_core` / `_sfa_grad_kernel` (sparse_flash_attention_grad_triton.py:334-376,
 * :158-308).  Query/key addressing as in DsaSfaFwdParams.  Inputs: q, q_rope, key, key_rope,
 * d_out and out ([num_rows][n1][d]), softmax_max / softmax_sum ([num_rows][n1], the forward's
 * statistics).  Outputs: dq [num_rows][n1][d], dqr [num_rows][n1][64] (query dtype); the key
 * gradients are accumulated in caller-provided fp32 buffers dk_acc [kv_rows][d],
 * dkr_acc [kv_rows][64], dv_acc [kv_rows][d] (zeroed by the call unless accumulate is set) and, unless defer_cast is
 * set, cast into dk / dkr / dv (key dtype, NULL to skip).  With defer_cast a caller (e.g. a
 * multi-GPU one that all-reduces the fp32 buffers) finishes with dsa_sfa_bwd_cast().
 * The key gradients are scatter-added with fp32 vector reductions, so their summation order
 * is not deterministic (as in the reference, which rejects deterministic=True).
 * Merged key gradient: with dv_acc = NULL (and dv = NULL) the call is for key == value (one
 * latent tensor, MLA-absorb) and accumulates dK + dV into dk_acc (cast into dk), the sum the
 * reference's bprop forms for that tensor; half the scattered bytes of separate dK and dV.
 */
typedef struct DsaSfaBwdParams {
  const void* q;
  const void* q_rope;
  const void* key;
  const void* key_rope;
  const void* d_out;
  const void* out;
  const float* softmax_max;
  const float* softmax_sum;
  const int32_t* sparse_indices;
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  const int32_t* k_row_base;
  const int32_t* block_table;
  void* dq;
  void* dqr;
  void* dk;
  void* dkr;
  void* dv;
  float* dk_acc;
  float* dkr_acc;
  float* dv_acc;
  int* error_flag;
  void* workspace;               /* dsa_sfa_bwd_workspace_size() bytes, caller-owned,
                                    256-byte aligned (DSA_ERR_INVALID_ARG otherwise) */
  int64_t workspace_bytes;
  int64_t num_rows;
  int64_t batch;
  int64_t n1;
  int64_t d;
  int64_t topk;
  int64_t sparse_block_size;
  int64_t kv_rows;
  int64_t page_size;
  int64_t max_blocks;
  int64_t s2_cap;
  float scale;
  int32_t sparse_mode;
  int32_t dtype;
  int32_t defer_cast;            /* 1: leave the key gradients in the fp32 buffers */
  int32_t accumulate;            /* 1: add into dk_acc / dkr_acc / dv_acc instead of zeroing
                                    them first (query rows processed in several calls) */
  float* teacher;                /* NULL, or fp32 [num_rows][topk], zeroed by the caller: the
                                    call adds (1/n1) sum_h P[row, key, h] of each valid entry
                                    at its place among the row's valid entries -- the
                                    attention distribution the indexer KL loss takes as its
                                    teacher (see DsaSliParams.teacher).  sparse_block_size 1. */
} DsaSfaBwdParams;

int dsa_sfa_bwd(const DsaSfaBwdParams* params, void* stream);

/* Cast dk_acc / dkr_acc / dv_acc into dk / dkr / dv (the tail of dsa_sfa_bwd). */
int dsa_sfa_bwd_cast(const DsaSfaBwdParams* params, void* stream);

/* Workspace of dsa_sfa_bwd: compacted key rows and counts, bf16/fp16 scratch for P and
 * dS ([num_rows][keys padded to 256][128 heads] each) and fp32 rowsum(dO * O) per (row, head)
 * ([num_rows][128]).  Returns -1 for invalid sizes. */
int64_t dsa_sfa_bwd_workspace_size(int64_t num_rows, int64_t topk, int64_t sparse_block_size);

/*
 * Lightning indexer: scores + top-k.
 * Replaces `_lightning_indexer_score_core` / `_lightning_indexer_score_kernel` and
 * `_stable_topk` (lightning_indexer_triton.py:382-413, :147-280, :339-357).
 *   query [q_rows][n1][d], key [kv_rows][n2][d] (bf16/fp16, d multiple of 8, <= 256),
 *   weights [q_rows][n1] (bf16/fp16/fp32, weights_dtype).
 *   score[r][n2][s2] = sum over the n1/n2 query heads g of group n2 of
 *                      ReLU(query[r][g] . key[k_row_base[b] + s2][n2]) * weights[r][g]
 *   for s2 < visible(r) (sparse_mode 3: min(act_k, clamp(act_k - act_q + s1 + 1, 0, s2_cap));
 *   mode 0: min(act_k, s2_cap); 0 for s1 >= act_q), -inf elsewhere.
 * Outputs: out_indices [q_rows][n2][sparse_count] int32 ordered by (score desc, index asc),
 * -1 where the score is -inf; out_values (query dtype, NULL to skip) the matching scores.
 * Query rows: q_row_base[b] is batch b's first row; a BSND caller passes q_len_dense = S1
 * (rows s1 >= act_q exist but see nothing); a TND caller passes q_len_dense = 0 (a batch has
 * act_q rows).  q_len_max = largest row count of a batch.  s2_row = length of a score row
 * (>= sparse_count, <= 131072).  Workspace: dsa_li_workspace_size() bytes (the fp32 score matrix).
 * Paged keys (no counterpart in the reference, whose indexer rejects block_table at
 * lightning_indexer_triton.py:497-498): with block_table != NULL, key is a block pool
 * [kv_rows = blocks * page_size][n2][d] and key position s2 of batch b is pool row
 * block_table[b * max_blocks + s2 / page_size] * page_size + s2 % page_size (k_row_base is
 * not read).  page_size is a multiple of 128 or divides 128 and is at least 8.  Blocks past
 * a row's visible keys are never read for its scores; a negative id reads zeros.
 * FP8 indexer (no counterpart in the reference): dtype DSA_DTYPE_FP8_E4M3 takes e4m3 query
 * and key (d 128 or 256) and key_scale [kv_rows][n2] (positive fp32, laid out
 * like the key rows, paged or not); score = key_scale * sum_g ReLU(q_g . k) * w_g, and
 * out_values are fp32.
 */
typedef struct DsaLiParams {
  const void* query;
  const void* key;
  const void* weights;
  const int32_t* act_q;
  const int32_t* act_k;
  const int32_t* q_row_base;
  const int32_t* k_row_base;
  int32_t* out_indices;
  void* out_values;
  int* error_flag;
  void* workspace;
  int64_t workspace_bytes;
  int64_t q_rows;
  int64_t batch;
  int64_t n1;
  int64_t n2;
  int64_t d;
  int64_t kv_rows;
  int64_t sparse_count;
  int64_t s2_row;
  int64_t s2_cap;
  int64_t q_len_max;
  int64_t q_len_dense;
  int32_t sparse_mode;
  int32_t dtype;
  int32_t weights_dtype;
  const int32_t* block_table;   /* NULL: dense keys at k_row_base; else [batch][max_blocks] */
  int64_t page_size;
  int64_t max_blocks;
  const float* key_scale;       /* dtype DSA_DTYPE_FP8_E4M3 only: [kv_rows][n2] fp32 > 0 */
} DsaLiParams;

int dsa_li_score_topk(const DsaLiParams* params, void* stream);
int64_t dsa_li_workspace_size(int64_t q_rows, int64_t n2, int64_t s2_row);

/*
 * Sparse lightning-indexer KL-loss gradient (BSND, sparse_mode 3).
 * Replaces `_sparse_lightning_indexer_grad_kl_loss_core` and its kernels
 * (sparse_lightning_indexer_grad_kl_loss_triton.py:355-464, :39-327).
 *   query [batch*s1][n1][d], query_rope [batch*s1][n1][64], key [batch*s2][d],
 *   key_rope [batch*s2][64], query_index [batch*s1][n_index][128], key_index [batch*s2][128],
 *   weights [batch*s1][n_index] (weights_dtype), sparse_indices [batch*s1][topk] int32,
 *   softmax_max / softmax_sum [batch*s1][n1] fp32, act_q / act_k [batch].
 * Outputs: d_query_index (query_index dtype), d_weights (weights dtype), loss [1] fp32 (sum
 * over rows, zeroed by the call), dki_acc [batch*s2][128] fp32 (zeroed by the call) and, if
 * d_key_index != NULL, its cast to the key_index dtype.  n_index <= 64, n1 <= 128.
 * Workspace: dsa_sli_workspace_size() bytes (the teacher distribution, fp32).
 */
typedef struct DsaSliParams {
  const void* query;
  const void* key;
  const void* query_rope;
  const void* key_rope;
  const void* query_index;
  const void* key_index;
  const void* weights;
  const int32_t* sparse_indices;
  const float* softmax_max;
  const float* softmax_sum;
  const int32_t* act_q;
  const int32_t* act_k;
  void* d_query_index;
  void* d_key_index;
  void* d_weights;
  float* dki_acc;
  float* loss;
  int* error_flag;
  void* workspace;
  int64_t workspace_bytes;
  int64_t batch;
  int64_t s1;
  int64_t s2;
  int64_t n1;
  int64_t d;
  int64_t n_index;
  int64_t d_index;
  int64_t topk;
  float scale;
  int32_t dtype;
  int32_t weights_dtype;
  const float* teacher;          /* NULL, or the teacher distribution p [batch*s1][topk] fp32
                                    (as dsa_sfa_bwd's teacher output gives it): the call then
                                    skips its own teacher pass, reads p from here and needs
                                    no workspace.  Valid when each row's valid entries come
                                    first in sparse_indices (an indexer top-k row is so). */
} DsaSliParams;

int dsa_sli_grad(const DsaSliParams* params, void* stream);

/* Cast dki_acc into d_key_index (key_index dtype): the tail of dsa_sli_grad, for a caller
 * that passed d_key_index = NULL there and summed dki_acc (and loss) over the GPUs that
 * hold disjoint query rows first.  Sharding support; the reference has no counterpart
 * (its scatter-and-cast is one call, sparse_lightning_indexer_grad_kl_loss_triton.py:268-327). */
int dsa_sli_cast(const DsaSliParams* params, void* stream);
int64_t dsa_sli_workspace_size(int64_t batch, int64_t s1, int64_t topk);

/*
 * Dense lightning-indexer KL loss: the indexer loss over every visible key of a query row
 * (BSND, sparse_mode 3).  Replaces the reference's dense path: `_dense_index_stats_core` and
 * `_dense_loss_backward_core` / `_dense_loss_backward_with_index_core` with their kernels
 * (dense_loss_backward_triton.py:129-397, :410-646).
 *   query [batch*s1][n1][d], key [batch*s2][n2][d], query_rope / key_rope [..][64] or NULL
 *   (d_rope 0 / 64), query_index [batch*s1][n_index][d_index], key_index [batch*s2][d_index],
 *   weights [batch*s1][n_index] (query dtype or fp32), softmax_max / softmax_sum
 *   [batch][n2][s1][n1/n2] fp32 (statistics of the full attention), act_q / act_k [batch].
 * dsa_dense_indexer_softmax_lse writes index_max / index_sum [batch*s1] (max of the index
 * scores over the visible keys and the sum of exp(score - max); -inf / 0 for a row without
 * visible keys).  dsa_dense_indexer_grad_kl_loss reads them and writes d_query_index
 * (query_index dtype), d_weights (weights dtype), loss [1] fp32 (sum over rows, zeroed by the
 * call) and, if d_key_index != NULL, the key_index gradient in its dtype.  n_index <= 128,
 * d_index <= 512 (multiples of 8).  Workspace: dsa_dense_indexer_workspace_size() bytes.
 */
typedef struct DsaDenseIndexerParams {
  const void* query;
  const void* key;
  const void* query_rope;
  const void* key_rope;
  const void* query_index;
  const void* key_index;
  const void* weights;
  const float* softmax_max;
  const float* softmax_sum;
  float* index_max;
  float* index_sum;
  const int32_t* act_q;
  const int32_t* act_k;
  void* d_query_index;
  void* d_key_index;
  void* d_weights;
  float* loss;
  void* workspace;
  int64_t workspace_bytes;
  int64_t batch;
  int64_t s1;
  int64_t s2;
  int64_t n1;
  int64_t n2;
  int64_t d;
  int64_t d_rope;
  int64_t n_index;
  int64_t d_index;
  float scale;
  int32_t dtype;
  int32_t weights_dtype;
} DsaDenseIndexerParams;

int dsa_dense_indexer_softmax_lse(const DsaDenseIndexerParams* params, void* stream);
int dsa_dense_indexer_grad_kl_loss(const DsaDenseIndexerParams* params, void* stream);
int64_t dsa_dense_indexer_workspace_size(int64_t batch, int64_t s1, int64_t s2, int64_t d_index);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H_ */
