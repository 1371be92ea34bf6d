"""lightning_indexer_triton: drop-in lightning indexer (score + top-k) on B200.

Same name, argument order, defaults and guards as the reference
``lightning_indexer_triton`` (lightning_indexer_triton.py:462-550) and its
``LightningIndexerTriton`` cell (:416-459).  BSND / TND layouts are addressed in place.
The score matrix is computed by a tcgen05 kernel and reduced by a radix-select top-k
kernel (``dsa_li_score_topk``).  Ties are broken by ascending key index (the reference's
default ``mint.topk`` leaves their order unspecified, :349-351).
"""
from __future__ import annotations

import torch

from . import _host as H
from ._lib import LiParams, DSA_DTYPE_FP32, DSA_DTYPE_FP8_E4M3, check, error_flag, lib, ptr, stream_ptr

INT64_MAX = H.INT64_MAX
MAX_SCORE_ROW = 1 << 17   # keys in one score row (the top-k kernel's packed counts)


def _check_row_length(s2):
    if s2 > MAX_SCORE_ROW:
        raise ValueError(f"key length {s2} exceeds the {MAX_SCORE_ROW} keys a score row may hold")


def _weights_code(w: torch.Tensor) -> int:
    if w.dtype == torch.float32:
        return DSA_DTYPE_FP32
    return H.dtype_code(w)


def lightning_indexer_triton(
    query: torch.Tensor,
    key: torch.Tensor,
    weights: torch.Tensor,
    actual_seq_lengths_query=None,
    actual_seq_lengths_key=None,
    block_table=None,
    layout_query="BSND",
    layout_key="BSND",
    sparse_count=2048,
    sparse_mode=3,
    pre_tokens=INT64_MAX,
    next_tokens=INT64_MAX,
    return_value=False,
):
    """Lightning indexer: returns (sparse_indices int32 [.., N2, sparse_count], values in the
    query dtype (zeros unless ``return_value``)).  ``pre_tokens``/``next_tokens`` are
    ignored, as in the reference."""
    if block_table is not None:   # lightning_indexer_triton.py:497-498
        raise ValueError("PA_BSND / block_table not supported in triton lightning_indexer")
    if sparse_mode not in (0, 3):
        raise ValueError("Only sparse_mode 0 (full) / 3 (rightDownCausal) supported")
    H.require_cuda(query, key, weights)
    dev = query.device
    is_tnd = layout_query == "TND"
    if is_tnd:
        cum_q = H.cumulative(actual_seq_lengths_query, dev)
        cum_k = H.cumulative(actual_seq_lengths_key, dev)
        B = cum_q.numel()
        q_base, act_q = H.tnd_offsets(cum_q)
        _, act_k = H.tnd_offsets(cum_k)
        T1, N1, D = query.shape
        q_rows = T1
        q_len_max = int(act_q.max().item()) if B > 0 else 0
        q_len_dense = 0
        if layout_key == "TND":
            k_base, _ = H.tnd_offsets(cum_k)
            kv_rows, N2 = key.shape[0], key.shape[1]
            s2 = int(act_k.max().item()) if B > 0 else 0
        else:
            kv_rows, N2 = key.shape[0] * key.shape[1], key.shape[2]
            s2 = key.shape[1]
            k_base = H.row_bases(B, s2, dev)
    else:
        B, S1, N1, D = query.shape
        _, S2, N2, _ = key.shape
        q_rows, q_len_max, q_len_dense = B * S1, S1, S1
        q_base = H.row_bases(B, S1, dev)
        k_base = H.row_bases(B, S2, dev)
        act_q = H.lens_tensor(actual_seq_lengths_query, B, S1, dev)
        act_k = H.lens_tensor(actual_seq_lengths_key, B, S2, dev)
        kv_rows, s2 = B * S2, S2
    if N1 % N2 != 0:              # lightning_indexer_triton.py:520-521
        raise ValueError(f"N1({N1}) must be divisible by N2({N2})")
    if key.shape[-1] != D or key.dtype != query.dtype:
        raise ValueError("query and key must share dtype and head dim")
    _check_row_length(s2)
    k_eff = min(int(sparse_count), s2)
    if k_eff != int(sparse_count):
        # the reference reshapes min(k, S2) results into sparse_count columns and fails
        raise ValueError(f"sparse_count ({sparse_count}) exceeds the key length ({s2})")
    q = query.contiguous()
    k = key.contiguous()
    w = weights.contiguous()
    K = int(sparse_count)
    out_shape = (q_rows, N2, K) if is_tnd else (B, S1, N2, K)
    indices = torch.empty(out_shape, dtype=torch.int32, device=dev)
    values = (torch.empty(out_shape, dtype=query.dtype, device=dev) if return_value
              else torch.zeros(out_shape, dtype=query.dtype, device=dev))
    ws_bytes = lib().dsa_li_workspace_size(q_rows, N2, s2)
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    p = LiParams()
    p.query, p.key, p.weights = ptr(q), ptr(k), ptr(w)
    p.act_q, p.act_k, p.q_row_base, p.k_row_base = ptr(act_q), ptr(act_k), ptr(q_base), ptr(k_base)
    p.out_indices = ptr(indices)
    p.out_values = ptr(values) if return_value else 0
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.q_rows, p.batch, p.n1, p.n2, p.d, p.kv_rows = q_rows, B, N1, N2, D, kv_rows
    p.sparse_count, p.s2_row, p.s2_cap = K, s2, s2
    p.q_len_max, p.q_len_dense = q_len_max, q_len_dense
    p.sparse_mode = int(sparse_mode)
    p.dtype = H.dtype_code(query)
    p.weights_dtype = _weights_code(w)
    check(lib().dsa_li_score_topk(p, stream_ptr(dev)), "dsa_li_score_topk")
    return indices, values


def lightning_indexer_paged(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    weights: torch.Tensor,
    block_table: torch.Tensor,
    actual_seq_lengths_query=None,
    actual_seq_lengths_key=None,
    layout_query="BSND",
    sparse_count=2048,
    sparse_mode=3,
    return_value=False,
):
    """Lightning indexer over a paged key cache (the decode-time indexer).

    No counterpart in the reference, whose indexer rejects ``block_table``
    (lightning_indexer_triton.py:497-498); the scores, masks, tie order and outputs are those
    of ``lightning_indexer_triton``.  ``key_cache`` is a block pool [num_blocks, page_size,
    N2, D]; ``block_table`` [B, max_blocks] int32 maps position s2 of batch b to block
    ``block_table[b, s2 // page_size]``, row ``s2 % page_size``.  ``actual_seq_lengths_key``
    gives each batch's key length (default: max_blocks * page_size, which is also the length
    of a score row).  ``query`` is BSND [B, S1, N1, D] or TND [T1, N1, D] with cumulative
    ``actual_seq_lengths_query``.  page_size is a multiple of 128, or divides 128 and is at
    least 8.  Rows longer than about 50k keys are selected from the score matrix in global
    memory instead of shared memory.
    """
    if sparse_mode not in (0, 3):
        raise ValueError("Only sparse_mode 0 (full) / 3 (rightDownCausal) supported")
    if key_cache.dim() != 4:
        raise ValueError("key_cache must be [num_blocks, page_size, N2, D]")
    if block_table.dim() != 2 or block_table.dtype != torch.int32:
        raise ValueError("block_table must be an int32 [B, max_blocks] tensor")
    nblocks, page, N2, Dk = key_cache.shape
    if page < 8 or (page % 128 != 0 and 128 % page != 0):
        raise ValueError(f"page_size ({page}) must be a multiple of 128 or divide 128 (>= 8)")
    _check_row_length(block_table.shape[1] * page)
    H.require_cuda(query, key_cache, weights, block_table)
    dev = query.device
    B, max_blocks = block_table.shape
    s2 = max_blocks * page
    if layout_query == "TND":
        cum_q = H.cumulative(actual_seq_lengths_query, dev)
        if cum_q.numel() != B:
            raise ValueError("actual_seq_lengths_query must have one entry per block_table row")
        q_base, act_q = H.tnd_offsets(cum_q)
        T1, N1, D = query.shape
        q_rows, q_len_dense = T1, 0
        q_len_max = int(act_q.max().item()) if B > 0 else 0
        out_shape = (T1, N2, int(sparse_count))
    else:
        Bq, S1, N1, D = query.shape
        if Bq != B:
            raise ValueError("query batch and block_table rows differ")
        q_rows, q_len_max, q_len_dense = B * S1, S1, S1
        q_base = H.row_bases(B, S1, dev)
        act_q = H.lens_tensor(actual_seq_lengths_query, B, S1, dev)
        out_shape = (B, S1, N2, int(sparse_count))
    act_k = H.lens_tensor(actual_seq_lengths_key, B, s2, dev)
    if N1 % N2 != 0:
        raise ValueError(f"N1({N1}) must be divisible by N2({N2})")
    if Dk != D or key_cache.dtype != query.dtype:
        raise ValueError("query and key_cache must share dtype and head dim")
    K = int(sparse_count)
    if K > s2:
        raise ValueError(f"sparse_count ({K}) exceeds the block table's capacity ({s2})")
    q = query.contiguous()
    k = key_cache.contiguous()
    w = weights.contiguous()
    bt = block_table.contiguous()
    indices = torch.empty(out_shape, dtype=torch.int32, device=dev)
    values = (torch.empty(out_shape, dtype=query.dtype, device=dev) if return_value
              else torch.zeros(out_shape, dtype=query.dtype, device=dev))
    ws_bytes = lib().dsa_li_workspace_size(q_rows, N2, s2)
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    p = LiParams()
    p.query, p.key, p.weights = ptr(q), ptr(k), ptr(w)
    p.act_q, p.act_k, p.q_row_base, p.k_row_base = ptr(act_q), ptr(act_k), ptr(q_base), 0
    p.out_indices = ptr(indices)
    p.out_values = ptr(values) if return_value else 0
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.q_rows, p.batch, p.n1, p.n2, p.d, p.kv_rows = q_rows, B, N1, N2, D, nblocks * page
    p.sparse_count, p.s2_row, p.s2_cap = K, s2, s2
    p.q_len_max, p.q_len_dense = q_len_max, q_len_dense
    p.sparse_mode = int(sparse_mode)
    p.dtype = H.dtype_code(query)
    p.weights_dtype = _weights_code(w)
    p.block_table, p.page_size, p.max_blocks = ptr(bt), page, max_blocks
    check(lib().dsa_li_score_topk(p, stream_ptr(dev)), "dsa_li_score_topk")
    return indices, values


def lightning_indexer_fp8(
    query: torch.Tensor,
    key: torch.Tensor,
    key_scale: torch.Tensor,
    weights: torch.Tensor,
    actual_seq_lengths_query=None,
    actual_seq_lengths_key=None,
    block_table=None,
    sparse_count=2048,
    sparse_mode=3,
    return_value=False,
):
    """FP8 lightning indexer: e4m3 query and key with a per-key scale.

    No counterpart in the reference (its indexer is bf16 / fp16); DeepSeek-V3.2 runs the
    indexer in FP8.  score[s2] = key_scale[s2] * sum_g ReLU(q_g . k_s2) * w_g, with any
    per-query scale folded into ``weights`` by the caller; masks, top-k and tie order are
    those of ``lightning_indexer_triton``.  ``query`` [B, S1, N1, D] and ``key`` are
    ``torch.float8_e4m3fn`` (D 128 or 256); ``key`` is [B, S2, N2, D] with
    ``key_scale`` [B, S2, N2], or, with ``block_table`` [B, max_blocks] int32, a block pool
    [num_blocks, page_size, N2, D] with ``key_scale`` [num_blocks, page_size, N2] (paging as
    in ``lightning_indexer_paged``).  ``key_scale`` is fp32 and positive.  Returns (indices
    int32 [B, S1, N2, sparse_count], values fp32; zeros unless ``return_value``).
    """
    if sparse_mode not in (0, 3):
        raise ValueError("Only sparse_mode 0 (full) / 3 (rightDownCausal) supported")
    if query.dtype != torch.float8_e4m3fn or key.dtype != torch.float8_e4m3fn:
        raise ValueError("query and key must be torch.float8_e4m3fn")
    if key_scale.dtype != torch.float32 or tuple(key_scale.shape) != tuple(key.shape[:3]):
        raise ValueError("key_scale must be float32 with the key's shape without D")
    if query.dim() != 4 or key.dim() != 4:
        raise ValueError("query and key must be 4-D")
    _check_row_length(key.shape[1] if block_table is None else block_table.shape[1] * key.shape[1])
    H.require_cuda(query, key, key_scale, weights, block_table)
    B, S1, N1, D = query.shape
    dev = query.device
    if block_table is None:
        if key.shape[0] != B:
            raise ValueError("key batch differs from query batch")
        S2, N2 = key.shape[1], key.shape[2]
        kv_rows, page, max_blocks, bt = B * S2, 0, 0, None
        k_base = H.row_bases(B, S2, dev)
    else:
        if block_table.dim() != 2 or block_table.dtype != torch.int32 or block_table.shape[0] != B:
            raise ValueError("block_table must be an int32 [B, max_blocks] tensor")
        nblocks, page, N2 = key.shape[0], key.shape[1], key.shape[2]
        if page < 8 or (page % 128 != 0 and 128 % page != 0):
            raise ValueError(f"page_size ({page}) must be a multiple of 128 or divide 128 (>= 8)")
        max_blocks = block_table.shape[1]
        S2, kv_rows = max_blocks * page, nblocks * page
        bt = block_table.contiguous()
        k_base = None
    if key.shape[3] != D or D not in (128, 256):
        raise ValueError("query and key must share a head dim of 128 or 256")
    if N1 % N2 != 0:
        raise ValueError(f"N1({N1}) must be divisible by N2({N2})")
    K = int(sparse_count)
    if K > S2:
        raise ValueError(f"sparse_count ({K}) exceeds the key length ({S2})")
    q_base = H.row_bases(B, S1, dev)
    act_q = H.lens_tensor(actual_seq_lengths_query, B, S1, dev)
    act_k = H.lens_tensor(actual_seq_lengths_key, B, S2, dev)
    q, k, ks, w = query.contiguous(), key.contiguous(), key_scale.contiguous(), weights.contiguous()
    out_shape = (B, S1, N2, K)
    indices = torch.empty(out_shape, dtype=torch.int32, device=dev)
    values = (torch.empty(out_shape, dtype=torch.float32, device=dev) if return_value
              else torch.zeros(out_shape, dtype=torch.float32, device=dev))
    ws_bytes = lib().dsa_li_workspace_size(B * S1, N2, S2)
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    p = LiParams()
    p.query, p.key, p.weights = ptr(q), ptr(k), ptr(w)
    p.act_q, p.act_k, p.q_row_base = ptr(act_q), ptr(act_k), ptr(q_base)
    p.k_row_base = ptr(k_base) if k_base is not None else 0
    p.out_indices = ptr(indices)
    p.out_values = ptr(values) if return_value else 0
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.q_rows, p.batch, p.n1, p.n2, p.d, p.kv_rows = B * S1, B, N1, N2, D, kv_rows
    p.sparse_count, p.s2_row, p.s2_cap = K, S2, S2
    p.q_len_max, p.q_len_dense = S1, S1
    p.sparse_mode = int(sparse_mode)
    p.dtype = DSA_DTYPE_FP8_E4M3
    p.weights_dtype = _weights_code(w)
    p.block_table = ptr(bt) if bt is not None else 0
    p.page_size, p.max_blocks = page, max_blocks
    p.key_scale = ptr(ks)
    check(lib().dsa_li_score_topk(p, stream_ptr(dev)), "dsa_li_score_topk")
    return indices, values


class LightningIndexerTriton(torch.nn.Module):
    """Module wrapper (reference cell: lightning_indexer_triton.py:416-459)."""

    def __init__(self, sparse_count=2048, sparse_mode=3, layout_query="BSND", layout_key="BSND",
                 return_value=False, pre_tokens=INT64_MAX, next_tokens=INT64_MAX):
        super().__init__()
        self.sparse_count = sparse_count
        self.sparse_mode = sparse_mode
        self.layout_query = layout_query
        self.layout_key = layout_key
        self.return_value = return_value
        self.pre_tokens = pre_tokens
        self.next_tokens = next_tokens

    def forward(self, query, key, weights, actual_seq_lengths_query=None,
                actual_seq_lengths_key=None, block_table=None):
        return lightning_indexer_triton(
            query, key, weights, actual_seq_lengths_query=actual_seq_lengths_query,
            actual_seq_lengths_key=actual_seq_lengths_key, block_table=block_table,
            layout_query=self.layout_query, layout_key=self.layout_key,
            sparse_count=self.sparse_count, sparse_mode=self.sparse_mode,
            pre_tokens=self.pre_tokens, next_tokens=self.next_tokens,
            return_value=self.return_value)
