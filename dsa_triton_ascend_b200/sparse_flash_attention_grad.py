"""sparse_flash_attention_grad_triton: drop-in backward of the reference operator on B200.

Same name, argument order, defaults and guards as the reference
``sparse_flash_attention_grad_triton`` (sparse_flash_attention_grad_triton.py:382-541)
and its ``SparseFlashAttentionGradTriton`` cell (:544-586).  Layouts BSND / TND are
addressed in place (no padded copies).  Returns (d_query, d_key, d_value, d_query_rope,
d_key_rope): d_key (Q K^T path) and d_value (P dO path) are separate, as in the
reference; a caller sharing key == value sums them.  The key gradients are scatter-added
in fp32 (non-deterministic summation order, like the reference's atomics), so
``deterministic=True`` is rejected exactly as the reference does.
"""
from __future__ import annotations

import torch

from . import _host as H
from ._lib import SfaBwdParams, check, error_flag, lib, ptr, stream_ptr

INT64_MAX = H.INT64_MAX
_VALID_D = (128, 256, 512)
_D_ROPE = 64
_VALID_N1 = (1, 2, 4, 8, 16, 32, 64, 128)


def _sfa_grad(query, key, value, sparse_indices, d_out, out, softmax_max, softmax_sum,
              scale_value, query_rope, key_rope, actual_seq_lengths_query,
              actual_seq_lengths_kv, sparse_block_size, layout, sparse_mode, pre_tokens,
              next_tokens, deterministic, defer_cast, accumulators=None, merged=False,
              teacher=None, workspace=None):
    # guards: sparse_flash_attention_grad_triton.py:428-438
    if pre_tokens != INT64_MAX or next_tokens != INT64_MAX:
        raise ValueError("pre_tokens/next_tokens only support default INT64_MAX")
    if sparse_mode not in (0, 3):
        raise ValueError("Only sparse_mode 0 (full) / 3 (rightDownCausal) supported")
    if query_rope is None or key_rope is None:
        raise ValueError("query_rope and key_rope are required (no empty rope)")
    if deterministic:
        raise ValueError("deterministic=True is not supported (scatter-add path)")
    if not H.is_pow2_block(int(sparse_block_size)):
        raise ValueError("sparse_block_size must be a power of 2 in [1,128]")
    if layout not in ("BSND", "TND"):
        raise ValueError(f"unsupported layout {layout}")
    H.require_cuda(query, key, query_rope, key_rope, sparse_indices, d_out, out,
                   softmax_max, softmax_sum)
    dev = query.device
    is_tnd = layout == "TND"
    if is_tnd:
        if query.dim() != 3 or key.dim() != 3:
            raise ValueError("TND tensors must be [T, N, D]")
        cum_q = H.cumulative(actual_seq_lengths_query, dev)
        cum_k = H.cumulative(actual_seq_lengths_kv, dev)
        B = cum_q.numel()
        if cum_k.numel() != B:
            raise ValueError("query and key TND lengths disagree on the batch size")
        q_base, act_q = H.tnd_offsets(cum_q)
        k_base, act_k = H.tnd_offsets(cum_k)
        T1, N1, D = query.shape
        num_rows = T1
        kv_rows, n2 = key.shape[0], key.shape[1]
        s2_cap = kv_rows
    else:
        if query.dim() != 4 or key.dim() != 4:
            raise ValueError("BSND tensors must be [B, S, N, D]")
        B, S1, N1, D = query.shape
        S2, n2 = key.shape[1], key.shape[2]
        num_rows, kv_rows, s2_cap = B * S1, B * S2, S2
        q_base = H.row_bases(B, S1, dev)
        k_base = H.row_bases(B, S2, dev)
        act_q = H.lens_tensor(actual_seq_lengths_query, B, S1, dev)
        act_k = H.lens_tensor(actual_seq_lengths_kv, B, S2, dev)
    D_ROPE = query_rope.shape[-1]
    # validation: sparse_flash_attention_grad_triton.py:471-478
    if D not in _VALID_D:
        raise ValueError(f"D must be one of {_VALID_D}, got {D}")
    if D_ROPE != _D_ROPE:
        raise ValueError(f"rope dim must be {_D_ROPE}, got {D_ROPE}")
    if n2 != 1:
        raise ValueError("Only N2=1 (MQA) is supported")
    if N1 not in _VALID_N1:
        raise ValueError(f"N1 must be one of {_VALID_N1}, got {N1}")
    for t in (key, key_rope, query_rope, d_out, out):
        if t.dtype != query.dtype:
            raise ValueError("query/key/rope/d_out/out must share one dtype")

    topk = sparse_indices.shape[-1]
    si = sparse_indices.reshape(num_rows, topk).to(torch.int32).contiguous()
    q, qr, k, kr = (t.contiguous() for t in (query, query_rope, key, key_rope))
    do, o = d_out.contiguous(), out.contiguous()
    smax = softmax_max.reshape(-1).to(torch.float32).contiguous()
    ssum = softmax_sum.reshape(-1).to(torch.float32).contiguous()
    if smax.numel() != num_rows * N1:
        raise ValueError("softmax_max/softmax_sum must hold one value per (query row, head)")

    dq = torch.empty_like(q)
    dqr = torch.empty_like(qr)
    flat = None
    if accumulators is None:
        # one contiguous fp32 buffer [dk | dkr | dv] ([dk + dv | dkr] when merged), so a
        # multi-GPU caller can sum the key gradients of all ranks with a single all-reduce
        nacc = D + D_ROPE + (0 if merged else D)
        flat = torch.empty(kv_rows * nacc, dtype=torch.float32, device=dev)
        dk_acc = flat[: kv_rows * D].view(kv_rows, D)
        dkr_acc = flat[kv_rows * D: kv_rows * (D + D_ROPE)].view(kv_rows, D_ROPE)
        dv_acc = None if merged else flat[kv_rows * (D + D_ROPE):].view(kv_rows, D)
    else:
        dk_acc, dkr_acc, dv_acc = (tuple(accumulators) + (None,))[:3]
        if merged:
            dv_acc = None
        for t, n in ((dk_acc, D), (dkr_acc, D_ROPE), (dv_acc, D)):
            if t is None and merged:
                continue
            if (t is None or t.dtype != torch.float32 or not t.is_contiguous() or t.device != dev
                    or t.numel() != kv_rows * n):
                raise ValueError("accumulators must be contiguous fp32 [kv_rows, dim] on the "
                                 "query's device")
    kshape = key.shape
    dk = torch.empty(kshape, dtype=key.dtype, device=dev)
    dv = None if merged else torch.empty(
        kshape, dtype=value.dtype if value is not None else key.dtype, device=dev)
    dkr = torch.empty(key_rope.shape, dtype=key_rope.dtype, device=dev)
    ws_bytes = lib().dsa_sfa_bwd_workspace_size(num_rows, topk, int(sparse_block_size))
    if workspace is None:
        ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    else:   # caller-owned (a test reads the key lists and row-pair runs back from it)
        if workspace.dtype != torch.uint8 or workspace.numel() < ws_bytes or workspace.device != dev:
            raise ValueError(f"workspace must be a uint8 tensor of >= {ws_bytes} bytes on the query's device")
        ws = workspace

    p = SfaBwdParams()
    p.q, p.q_rope, p.key, p.key_rope = ptr(q), ptr(qr), ptr(k), ptr(kr)
    p.d_out, p.out, p.softmax_max, p.softmax_sum = ptr(do), ptr(o), ptr(smax), ptr(ssum)
    p.sparse_indices, p.act_q, p.act_k = ptr(si), ptr(act_q), ptr(act_k)
    p.q_row_base, p.k_row_base, p.block_table = ptr(q_base), ptr(k_base), 0
    # merged: dv and dv_acc NULL; the kernels add dS^T Q + P^T dO into dk_acc
    p.dq, p.dqr, p.dk, p.dkr = ptr(dq), ptr(dqr), ptr(dk), ptr(dkr)
    p.dv = 0 if merged else ptr(dv)
    p.dk_acc, p.dkr_acc = ptr(dk_acc), ptr(dkr_acc)
    p.dv_acc = 0 if merged else ptr(dv_acc)
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.num_rows, p.batch, p.n1, p.d, p.topk = num_rows, B, N1, D, topk
    p.sparse_block_size = int(sparse_block_size)
    p.kv_rows, p.page_size, p.max_blocks, p.s2_cap = kv_rows, 0, 0, s2_cap
    p.scale = float(scale_value)
    p.sparse_mode = int(sparse_mode)
    p.dtype = H.dtype_code(query)
    p.defer_cast = 1 if defer_cast else 0
    p.accumulate = 0 if accumulators is None else 1
    if teacher is not None:
        # fp32 [num_rows, topk], zeroed: K1 adds (1/N1) sum_h P of each valid entry
        if (teacher.dtype != torch.float32 or not teacher.is_contiguous()
                or teacher.numel() != num_rows * topk or int(sparse_block_size) != 1):
            raise ValueError("teacher must be a contiguous fp32 [rows, topk] buffer (block size 1)")
        p.teacher = ptr(teacher)
    check(lib().dsa_sfa_bwd(p, stream_ptr(dev)), "dsa_sfa_bwd")
    if defer_cast:
        def finish():
            check(lib().dsa_sfa_bwd_cast(p, stream_ptr(dev)), "dsa_sfa_bwd_cast")
            return (dq, dk, dqr, dkr) if merged else (dq, dk, dv, dqr, dkr)
        finish.query_grads = (dq, dqr)   # ready before the cast (they need no reduction)
        # the accumulators as one contiguous fp32 tensor (None when the caller passed its
        # own accumulators)
        finish.key_grad_buffer = flat
        return ((dk_acc, dkr_acc) if merged else (dk_acc, dkr_acc, dv_acc)), finish
    return (dq, dk, dqr, dkr) if merged else (dq, dk, dv, dqr, dkr)


def sparse_flash_attention_grad_triton(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    sparse_indices: torch.Tensor,
    d_out: torch.Tensor,
    out: torch.Tensor,
    softmax_max: torch.Tensor,
    softmax_sum: torch.Tensor,
    scale_value: float = 1.0,
    query_rope=None,
    key_rope=None,
    actual_seq_lengths_query=None,
    actual_seq_lengths_kv=None,
    sparse_block_size: int = 1,
    layout: str = "BSND",
    sparse_mode: int = 3,
    pre_tokens: int = INT64_MAX,
    next_tokens: int = INT64_MAX,
    deterministic: bool = False,
):
    """SparseFlashAttentionGrad (MLA-absorb, MQA): returns
    (d_query, d_key, d_value, d_query_rope, d_key_rope)."""
    return _sfa_grad(query, key, value, sparse_indices, d_out, out, softmax_max, softmax_sum,
                     scale_value, query_rope, key_rope, actual_seq_lengths_query,
                     actual_seq_lengths_kv, sparse_block_size, layout, sparse_mode, pre_tokens,
                     next_tokens, deterministic, defer_cast=False)


def sparse_flash_attention_grad_merged(query, key, sparse_indices, d_out, out, softmax_max,
                                       softmax_sum, scale_value=1.0, **kw):
    """Backward for key == value (MLA-absorb: one latent tensor is both): returns
    (d_query, d_key, d_query_rope, d_key_rope) with d_key = dK + dV, the gradient the
    reference's bprop hands back for the shared tensor (sparse_flash_attention_grad_triton.py:66).

    Same arguments as :func:`sparse_flash_attention_grad_triton` without ``value``.  The
    kernels accumulate dS^T Q + P^T dO into one fp32 buffer, which halves the scattered
    key-gradient bytes (4 (D + 64) per valid pair instead of 4 (2 D + 64))."""
    args = dict(query_rope=None, key_rope=None, actual_seq_lengths_query=None,
                actual_seq_lengths_kv=None, sparse_block_size=1, layout="BSND", sparse_mode=3,
                pre_tokens=INT64_MAX, next_tokens=INT64_MAX, deterministic=False)
    args.update(kw)
    return _sfa_grad(query, key, key, sparse_indices, d_out, out, softmax_max, softmax_sum,
                     scale_value, defer_cast=False, merged=True, **args)


def sparse_flash_attention_grad_partial(query, key, value, sparse_indices, d_out, out,
                                        softmax_max, softmax_sum, scale_value=1.0,
                                        merge_key_grads=False, **kw):
    """Backward for a caller that reduces the key gradients itself (e.g. across GPUs).

    Same arguments as :func:`sparse_flash_attention_grad_triton`, plus ``accumulators``:
    optional fp32 ``(dk_acc, dkr_acc, dv_acc)`` to add this call's key gradients into
    (query rows processed in several calls); without it they are fresh and zeroed.
    Returns ``((dk_acc, dkr_acc, dv_acc), finish)``: the fp32 key-gradient accumulators,
    which the caller may all-reduce in place, and ``finish()`` which casts them to the key
    dtype and returns the usual 5-tuple.  Fresh accumulators are views of one contiguous
    buffer, ``finish.key_grad_buffer``, so one all-reduce of it sums all three.

    ``merge_key_grads=True`` (key == value): the accumulators are ``(dkv_acc, dkr_acc)``
    with dkv = dK + dV, and ``finish()`` returns (d_query, d_key, d_query_rope, d_key_rope)
    as :func:`sparse_flash_attention_grad_merged` does.
    """
    args = dict(query_rope=None, key_rope=None, actual_seq_lengths_query=None,
                actual_seq_lengths_kv=None, sparse_block_size=1, layout="BSND", sparse_mode=3,
                pre_tokens=INT64_MAX, next_tokens=INT64_MAX, deterministic=False,
                accumulators=None)
    args.update(kw)
    return _sfa_grad(query, key, value, sparse_indices, d_out, out, softmax_max, softmax_sum,
                     scale_value, defer_cast=True, merged=bool(merge_key_grads), **args)


class SparseFlashAttentionGradTriton(torch.nn.Module):
    """Module wrapper (reference cell: sparse_flash_attention_grad_triton.py:544-586)."""

    def __init__(self, scale_value=1.0, sparse_block_size=1, layout="BSND", sparse_mode=3,
                 pre_tokens=INT64_MAX, next_tokens=INT64_MAX, deterministic=False):
        super().__init__()
        self.scale_value = scale_value
        self.sparse_block_size = sparse_block_size
        self.layout = layout
        self.sparse_mode = sparse_mode
        self.pre_tokens = pre_tokens
        self.next_tokens = next_tokens
        self.deterministic = deterministic

    def forward(self, query, key, value, sparse_indices, d_out, out, softmax_max, softmax_sum,
                query_rope=None, key_rope=None, actual_seq_lengths_query=None,
                actual_seq_lengths_kv=None):
        return sparse_flash_attention_grad_triton(
            query, key, value, sparse_indices, d_out, out, softmax_max, softmax_sum,
            scale_value=self.scale_value, query_rope=query_rope, key_rope=key_rope,
            actual_seq_lengths_query=actual_seq_lengths_query,
            actual_seq_lengths_kv=actual_seq_lengths_kv,
            sparse_block_size=self.sparse_block_size, layout=self.layout,
            sparse_mode=self.sparse_mode, pre_tokens=self.pre_tokens,
            next_tokens=self.next_tokens, deterministic=self.deterministic)
