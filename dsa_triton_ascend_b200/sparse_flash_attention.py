"""sparse_flash_attention_triton: drop-in forward of the reference operator on B200.

Same name, argument order, defaults and guards as the reference
``sparse_flash_attention_triton`` (sparse_flash_attention_triton.py:483-641) and its
``SparseFlashAttentionTriton`` cell (:644-695), with ``mindspore.Tensor`` replaced by
CUDA ``torch.Tensor``.  The computation runs in ``libdsa_b200.so`` (``dsa_sfa_fwd``);
layouts are not copied into padded BSND buffers but addressed in place:

* BSND query [B,S1,N1,D] / TND query [T1,N1,D] (cumulative ``actual_seq_lengths_query``)
* BSND key [B,S2,1,D] / TND key [T2,1,D] / PA_BSND cache [blocks,block_size,1,D] with
  ``block_table`` [B,max_blocks] (resolved inside the kernel, no de-paging copy)

MLA-absorb: ``value`` is ignored (value = key[..., :D]).
"""
from __future__ import annotations

import torch

from . import _host as H
from ._lib import SfaFwdParams, check, error_flag, lib, ptr, stream_ptr

INT64_MAX = H.INT64_MAX
_VALID_D = (128, 256, 512)
_D_ROPE = 64
_VALID_N1 = (1, 2, 4, 8, 16, 32, 64, 128)


def sparse_flash_attention_triton(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    sparse_indices: torch.Tensor,
    scale_value: float = 1.0,
    block_table=None,
    actual_seq_lengths_query=None,
    actual_seq_lengths_kv=None,
    query_rope=None,
    key_rope=None,
    sparse_block_size: int = 1,
    layout_query: str = "BSND",
    layout_kv: str = "BSND",
    sparse_mode: int = 0,
    pre_tokens: int = INT64_MAX,
    next_tokens: int = INT64_MAX,
    attention_mode: int = 2,
    return_softmax_lse: bool = False,
    block_size: int = 0,
):
    """Sparse flash attention forward (MLA-absorb, MQA).  Returns
    (attention_out, softmax_max, softmax_sum); softmax stats are (B,1,S1,N1) for BSND
    and (1,T1,N1) for TND, zeros when ``return_softmax_lse`` is False."""
    # guards: sparse_flash_attention_triton.py:529-539
    if attention_mode != 2:
        raise ValueError("Only attention_mode=2 (MLA-absorb) is supported")
    if pre_tokens != INT64_MAX or next_tokens != INT64_MAX:
        raise ValueError("pre_tokens/next_tokens only support default INT64_MAX")
    if sparse_mode not in (0, 3):
        raise ValueError("Only sparse_mode 0 (full) / 3 (rightDownCausal) supported")
    if query_rope is None or key_rope is None:
        raise ValueError("query_rope and key_rope are required (no empty rope)")
    if not H.is_pow2_block(int(sparse_block_size)):
        raise ValueError("sparse_block_size must be a power of 2 in [1,128]")
    if layout_query not in ("BSND", "TND"):
        raise ValueError(f"unsupported layout_query {layout_query}")
    if layout_kv not in ("BSND", "TND", "PA_BSND"):
        raise ValueError(f"unsupported layout_kv {layout_kv}")
    H.require_cuda(query, key, query_rope, key_rope, sparse_indices)
    dev = query.device
    is_tnd_q = layout_query == "TND"

    # ---- query side ----
    if is_tnd_q:
        if query.dim() != 3:
            raise ValueError("TND query must be [T1, N1, D]")
        cum_q = H.cumulative(actual_seq_lengths_query, dev)
        B = cum_q.numel()
        q_base, act_q = H.tnd_offsets(cum_q)
        T1, N1, D = query.shape
        num_rows, S1 = T1, None
    else:
        if query.dim() != 4:
            raise ValueError("BSND query must be [B, S1, N1, D]")
        B, S1, N1, D = query.shape
        num_rows = B * S1
        q_base = H.row_bases(B, S1, dev)
        act_q = H.lens_tensor(actual_seq_lengths_query, B, S1, dev)
    D_ROPE = query_rope.shape[-1]

    # ---- key side ----
    page, max_blocks, bt = 0, 0, None
    if layout_kv == "PA_BSND":
        if block_table is None:
            raise ValueError("PA_BSND requires block_table")
        if actual_seq_lengths_kv is None:
            raise ValueError("PA_BSND requires actual_seq_lengths_kv")
        if key.dim() != 4:
            raise ValueError("PA_BSND key must be [block_num, block_size, 1, D]")
        page = int(block_size) or key.shape[1]
        if page != key.shape[1]:
            raise ValueError(f"block_size {page} does not match the cache block dim {key.shape[1]}")
        H.require_cuda(block_table)
        bt = block_table.to(dtype=torch.int32).contiguous()
        if bt.dim() != 2 or bt.shape[0] != B:
            raise ValueError("block_table must be [B, max_blocks]")
        max_blocks = bt.shape[1]
        kv_rows = key.shape[0] * page
        n2 = key.shape[2]
        s2_cap = max_blocks * page
        act_k = H.lens_tensor(actual_seq_lengths_kv, B, s2_cap, dev)
        k_base = None
    elif layout_kv == "TND":
        if key.dim() != 3:
            raise ValueError("TND key must be [T2, 1, D]")
        cum_k = H.cumulative(actual_seq_lengths_kv, dev)
        if cum_k.numel() != B:
            raise ValueError("query and key TND lengths disagree on the batch size")
        k_base, act_k = H.tnd_offsets(cum_k)
        kv_rows, n2 = key.shape[0], key.shape[1]
        s2_cap = kv_rows
    else:
        if key.dim() != 4 or key.shape[0] != B:
            raise ValueError("BSND key must be [B, S2, 1, D]")
        S2, n2 = key.shape[1], key.shape[2]
        kv_rows = B * S2
        k_base = H.row_bases(B, S2, dev)
        act_k = H.lens_tensor(actual_seq_lengths_kv, B, S2, dev)
        s2_cap = S2

    # validation: sparse_flash_attention_triton.py:579-586
    if D not in _VALID_D:
        raise ValueError(f"D must be one of {_VALID_D}, got {D}")
    if D_ROPE != _D_ROPE:
        raise ValueError(f"rope dim must be {_D_ROPE}, got {D_ROPE}")
    if n2 != 1:
        raise ValueError("Only N2=1 (MQA) is supported")
    if N1 not in _VALID_N1:
        raise ValueError(f"N1 must be one of {_VALID_N1}, got {N1}")
    if key.shape[-1] != D or key.dtype != query.dtype or key_rope.dtype != query.dtype \
            or query_rope.dtype != query.dtype:
        raise ValueError("query/key/rope tensors must share dtype and latent dim")

    topk = sparse_indices.shape[-1]
    si = sparse_indices.reshape(num_rows, topk)
    if si.dtype != torch.int32:
        si = si.to(torch.int32)
    si = si.contiguous()
    q = query.contiguous()
    qr = query_rope.contiguous()
    k = key.contiguous()
    kr = key_rope.contiguous()

    out = torch.empty(query.shape, dtype=query.dtype, device=dev)
    # the kernel writes every statistic (zeros for rows without keys); zeros are only
    # needed when they are not requested
    alloc = torch.empty if return_softmax_lse else torch.zeros
    if is_tnd_q:
        smax = alloc((1, num_rows, N1), dtype=torch.float32, device=dev)
    else:
        smax = alloc((B, 1, S1, N1), dtype=torch.float32, device=dev)
    ssum = alloc(smax.shape, dtype=torch.float32, device=dev)

    # room for the split partials too: few-row calls (decode) then spread over more SMs
    ws_bytes = lib().dsa_sfa_fwd_fast_workspace_size(num_rows, N1, D, topk, int(sparse_block_size))
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)

    p = SfaFwdParams()
    p.q, p.q_rope, p.key, p.key_rope = ptr(q), ptr(qr), ptr(k), ptr(kr)
    p.sparse_indices, p.act_q, p.act_k = ptr(si), ptr(act_q), ptr(act_k)
    p.q_row_base, p.k_row_base, p.block_table = ptr(q_base), ptr(k_base), ptr(bt)
    p.out = ptr(out)
    p.softmax_max = ptr(smax) if return_softmax_lse else 0
    p.softmax_sum = ptr(ssum) if return_softmax_lse else 0
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.num_rows, p.batch, p.n1, p.d, p.topk = num_rows, B, N1, D, topk
    p.sparse_block_size = int(sparse_block_size)
    p.kv_rows, p.page_size, p.max_blocks, p.s2_cap = kv_rows, page, max_blocks, s2_cap
    p.scale = float(scale_value)
    p.sparse_mode = int(sparse_mode)
    p.dtype = H.dtype_code(query)
    check(lib().dsa_sfa_fwd(p, stream_ptr(dev)), "dsa_sfa_fwd")
    return out, smax, ssum


class SparseFlashAttentionTriton(torch.nn.Module):
    """Module wrapper around :func:`sparse_flash_attention_triton`
    (reference cell: sparse_flash_attention_triton.py:644-695)."""

    def __init__(self, scale_value=1.0, sparse_block_size=1, layout_query="BSND",
                 layout_kv="BSND", sparse_mode=0, attention_mode=2, return_softmax_lse=False,
                 pre_tokens=INT64_MAX, next_tokens=INT64_MAX, block_size=0):
        super().__init__()
        self.scale_value = scale_value
        self.sparse_block_size = sparse_block_size
        self.layout_query = layout_query
        self.layout_kv = layout_kv
        self.sparse_mode = sparse_mode
        self.attention_mode = attention_mode
        self.return_softmax_lse = return_softmax_lse
        self.pre_tokens = pre_tokens
        self.next_tokens = next_tokens
        self.block_size = block_size

    def forward(self, query, key, value, sparse_indices, query_rope=None, key_rope=None,
                actual_seq_lengths_query=None, actual_seq_lengths_kv=None, block_table=None):
        return sparse_flash_attention_triton(
            query, key, value, sparse_indices, scale_value=self.scale_value,
            block_table=block_table, actual_seq_lengths_query=actual_seq_lengths_query,
            actual_seq_lengths_kv=actual_seq_lengths_kv, query_rope=query_rope,
            key_rope=key_rope, sparse_block_size=self.sparse_block_size,
            layout_query=self.layout_query, layout_kv=self.layout_kv,
            sparse_mode=self.sparse_mode, pre_tokens=self.pre_tokens,
            next_tokens=self.next_tokens, attention_mode=self.attention_mode,
            return_softmax_lse=self.return_softmax_lse, block_size=self.block_size)
