"""sparse_lightning_indexer_grad_kl_loss_triton: drop-in indexer KL-loss gradient on B200.

Same name, argument order, defaults and guards as the reference
``sparse_lightning_indexer_grad_kl_loss_triton``
(sparse_lightning_indexer_grad_kl_loss_triton.py:520-556) and its
``SparseLightningIndexerGradKLLossTriton`` cell (:467-516).  Returns
(dQueryIndex, dKeyIndex, dWeights, loss); loss is the KL divergence summed over all
query rows (not averaged), fp32 [1].  Computed by ``dsa_sli_grad`` (two tcgen05 kernels,
no gathered copies).
"""
from __future__ import annotations

import torch

from . import _host as H
from ._lib import SliParams, DSA_DTYPE_FP32, check, error_flag, lib, ptr, stream_ptr

INT64_MAX = H.INT64_MAX


def sparse_lightning_indexer_grad_kl_loss_triton(
    query: torch.Tensor, key: torch.Tensor,
    query_index: torch.Tensor, key_index: torch.Tensor,
    weights: torch.Tensor, sparse_indices: torch.Tensor,
    softmax_max: torch.Tensor, softmax_sum: torch.Tensor,
    query_rope: torch.Tensor = None, key_rope: torch.Tensor = None,
    actual_seq_qlen=None, actual_seq_klen=None,
    scale_value: float = 1.0,
    layout: str = "BSND", sparse_mode: int = 3,
    pre_tokens: int = INT64_MAX,
    next_tokens: int = INT64_MAX,
    deterministic: bool = False,
):
    """Drop-in replacement for aclnnSparseLightningIndexerGradKLLoss (BSND, mode 3)."""
    return _sli(query, key, query_index, key_index, weights, sparse_indices, softmax_max,
                softmax_sum, query_rope, key_rope, actual_seq_qlen, actual_seq_klen, scale_value,
                layout, sparse_mode, defer_cast=False)


def sparse_lightning_indexer_grad_kl_loss_partial(
    query, key, query_index, key_index, weights, sparse_indices, softmax_max, softmax_sum,
    query_rope=None, key_rope=None, actual_seq_qlen=None, actual_seq_klen=None,
    scale_value=1.0, layout="BSND", sparse_mode=3):
    """The indexer KL-loss gradient for a caller that sums it over GPUs itself.

    Same arguments as :func:`sparse_lightning_indexer_grad_kl_loss_triton` (a contiguous
    causal row range [r0, r1) of a BSND batch is passed as its own query with
    ``actual_seq_qlen = S1 - r0``, see ``sharding.py``).  Returns ``((dki_acc, loss),
    finish)``: the fp32 dKeyIndex accumulator [B*S2, 128] and this call's loss [1], both
    views of one contiguous buffer ``finish.key_grad_buffer`` (one all-reduce sums both),
    and ``finish()``, which casts the (reduced) accumulator to the key_index dtype and
    returns (dQueryIndex, dKeyIndex, dWeights, loss)."""
    return _sli(query, key, query_index, key_index, weights, sparse_indices, softmax_max,
                softmax_sum, query_rope, key_rope, actual_seq_qlen, actual_seq_klen, scale_value,
                layout, sparse_mode, defer_cast=True)


def _sli(query, key, query_index, key_index, weights, sparse_indices, softmax_max, softmax_sum,
         query_rope, key_rope, actual_seq_qlen, actual_seq_klen, scale_value, layout,
         sparse_mode, defer_cast, teacher=None):
    # guards: sparse_lightning_indexer_grad_kl_loss_triton.py:534-538
    if layout != "BSND":
        raise ValueError("Only BSND layout is supported in triton path")
    if sparse_mode != 3:
        raise ValueError("Only sparse_mode=3 (rightDownCausal) is supported")
    assert sparse_indices.shape[2] == 1, "Nidx2 must be 1 (MQA constraint)"
    H.require_cuda(query, key, query_index, key_index, weights, sparse_indices, softmax_max,
                   softmax_sum)
    dev = query.device
    B, S1, N1, D = query.shape
    S2, N2 = key.shape[1], key.shape[2]
    Ni, Di = query_index.shape[2], query_index.shape[3]
    topk = sparse_indices.shape[3]
    if N2 != 1 or key_index.shape[2] != 1:
        raise ValueError("key / key_index must have one head (MQA)")
    if D not in (128, 256, 512) or Di != 128 or Ni > 64 or N1 > 128:
        raise ValueError("supported: D in (128, 256, 512), D_idx == 128, Nidx1 <= 64, N1 <= 128")
    # absent rope contributes nothing (the reference zero-fills it, :543-546)
    if query_rope is None:
        query_rope = torch.zeros((B, S1, N1, 64), dtype=query.dtype, device=dev)
    if key_rope is None:
        key_rope = torch.zeros((B, S2, N2, 64), dtype=key.dtype, device=dev)
    if query_rope.shape[-1] != 64 or key_rope.shape[-1] != 64:
        raise ValueError("rope dim must be 64")
    for t in (key, query_rope, key_rope, query_index, key_index):
        if t.dtype != query.dtype:
            raise ValueError("query/key/rope/index tensors must share one dtype")
    act_q = H.lens_tensor(actual_seq_qlen, B, S1, dev)
    act_k = H.lens_tensor(actual_seq_klen, B, S2, dev)
    q, k, qr, kr, qi, ki = (t.contiguous() for t in (query, key, query_rope, key_rope,
                                                      query_index, key_index))
    w = weights.contiguous()
    si = sparse_indices.reshape(B * S1, topk).to(torch.int32).contiguous()
    smax = softmax_max.reshape(-1).to(torch.float32).contiguous()
    ssum = softmax_sum.reshape(-1).to(torch.float32).contiguous()
    d_qi = torch.empty_like(qi)
    d_ki = torch.empty_like(ki)
    d_w = torch.empty_like(w)
    # [dKeyIndex accumulator | loss | pad]: one buffer, so that a sharded caller sums both
    # with a single all-reduce
    nk = B * S2 * Di
    flat = torch.empty(nk + 4, dtype=torch.float32, device=dev)
    dki_acc = flat[:nk].view(B * S2, Di)
    loss = flat[nk:nk + 1]
    if teacher is not None:
        # the attention backward's (1/N1) sum_h P per entry: no teacher pass, no workspace
        if (teacher.dtype != torch.float32 or not teacher.is_contiguous()
                or teacher.numel() != B * S1 * topk):
            raise ValueError("teacher must be a contiguous fp32 [B*S1, topk] buffer")
        ws_bytes = 0
        ws = torch.empty(4, dtype=torch.uint8, device=dev)
    else:
        ws_bytes = lib().dsa_sli_workspace_size(B, S1, topk)
        ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    p = SliParams()
    p.query, p.key, p.query_rope, p.key_rope = ptr(q), ptr(k), ptr(qr), ptr(kr)
    p.query_index, p.key_index, p.weights = ptr(qi), ptr(ki), ptr(w)
    p.sparse_indices, p.softmax_max, p.softmax_sum = ptr(si), ptr(smax), ptr(ssum)
    p.act_q, p.act_k = ptr(act_q), ptr(act_k)
    p.d_query_index, p.d_key_index, p.d_weights = ptr(d_qi), 0 if defer_cast else ptr(d_ki), ptr(d_w)
    p.dki_acc, p.loss = ptr(dki_acc), ptr(loss)
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.teacher = ptr(teacher) if teacher is not None else 0
    p.batch, p.s1, p.s2, p.n1, p.d = B, S1, S2, N1, D
    p.n_index, p.d_index, p.topk = Ni, Di, topk
    p.scale = float(scale_value)
    p.dtype = H.dtype_code(query)
    p.weights_dtype = DSA_DTYPE_FP32 if w.dtype == torch.float32 else H.dtype_code(w)
    check(lib().dsa_sli_grad(p, stream_ptr(dev)), "dsa_sli_grad")
    if defer_cast:
        p.d_key_index = ptr(d_ki)

        def finish():
            check(lib().dsa_sli_cast(p, stream_ptr(dev)), "dsa_sli_cast")
            return d_qi, d_ki, d_w, loss
        finish.key_grad_buffer = flat
        finish.keep_alive = (q, k, qr, kr, qi, ki, w, si, smax, ssum, act_q, act_k, ws)
        return (dki_acc, loss), finish
    return d_qi, d_ki, d_w, loss


class SparseLightningIndexerGradKLLossTriton(torch.nn.Module):
    """Module wrapper (reference cell: sparse_lightning_indexer_grad_kl_loss_triton.py:467-516)."""

    def __init__(self, scale_value=1.0, layout="BSND", sparse_mode=3, pre_tokens=INT64_MAX,
                 next_tokens=INT64_MAX, deterministic=False):
        super().__init__()
        self.scale_value = scale_value
        self.layout = layout
        self.sparse_mode = sparse_mode
        self.pre_tokens = pre_tokens
        self.next_tokens = next_tokens
        self.deterministic = deterministic

    def forward(self, query, key, query_index, key_index, weights, sparse_indices, softmax_max,
                softmax_sum, query_rope=None, key_rope=None, actual_seq_qlen=None,
                actual_seq_klen=None):
        return sparse_lightning_indexer_grad_kl_loss_triton(
            query, key, query_index, key_index, weights, sparse_indices, softmax_max, softmax_sum,
            query_rope=query_rope, key_rope=key_rope, actual_seq_qlen=actual_seq_qlen,
            actual_seq_klen=actual_seq_klen, scale_value=self.scale_value, layout=self.layout,
            sparse_mode=self.sparse_mode, pre_tokens=self.pre_tokens,
            next_tokens=self.next_tokens, deterministic=self.deterministic)
