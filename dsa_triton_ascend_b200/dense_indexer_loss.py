"""Dense lightning-indexer KL loss on B200: the indexer loss over every visible key.

Same names, argument order, defaults and guards as the reference's dense path
(``dense_loss_backward_triton.py``): ``dense_loss_backward_triton`` (:752-814),
``npu_dense_lightning_indexer_softmax_lse_triton`` / ``dense_lightning_indexer_softmax_lse_triton``
(:817-865), ``dense_lightning_indexer_grad_kl_loss_triton`` /
``npu_dense_lightning_indexer_grad_kl_loss_triton`` (:868-930) and the cells
``DenseLightningIndexerSoftmaxLseTriton``, ``DenseLossBackwardTriton``,
``DenseLightningIndexerGradKLLossTriton`` (:933-1002).  The reference raises ``TypeError`` for
wrong dtypes and ``ValueError`` for wrong shapes and options; so does this module.  Computed
by ``dsa_dense_indexer_softmax_lse`` and ``dsa_dense_indexer_grad_kl_loss`` (csrc/dense.cu).
"""
from __future__ import annotations

import torch

from . import _host as H
from ._lib import DenseIndexerParams, DSA_DTYPE_FP32, check, lib, ptr, stream_ptr

INT64_MAX = H.INT64_MAX
SUPPORTED_D = (128, 256, 512)        # dense_loss_backward_triton.py:12-13
SUPPORTED_NIDX1 = (32, 64, 128)


def _check_in(name, value, supported):
    if value not in supported:
        raise ValueError(f"{name}={value} is not supported; supported values: {supported}")


def _validate_index_inputs(query_index, key_index, weights, layout, sparse_mode,
                           pre_tokens=INT64_MAX, next_tokens=INT64_MAX):
    """dense_loss_backward_triton.py:649-672"""
    if layout != "BSND":
        raise ValueError("Only BSND layout is supported")
    if sparse_mode != 3:
        raise ValueError("Only sparse_mode=3 (rightDownCausal) is supported")
    if pre_tokens != INT64_MAX or next_tokens != INT64_MAX:
        raise ValueError("pre_tokens/next_tokens only support the official default value")
    if query_index.dim() != 4 or key_index.dim() != 4:
        raise ValueError("query_index and key_index must be 4D BSND tensors")
    if weights.dim() != 3:
        raise ValueError("weights must be [B, S1, Nidx1]")
    B, S1, Nidx1, D_idx = query_index.shape
    if key_index.shape[0] != B or key_index.shape[2] != 1:
        raise ValueError("key_index must be [B, S2, 1, D_idx]")
    if tuple(weights.shape) != (B, S1, Nidx1):
        raise ValueError("weights must be [B, S1, Nidx1]")
    if key_index.shape[3] != D_idx:
        raise ValueError("query_index and key_index must share D_idx")
    _check_in("Nidx1", Nidx1, SUPPORTED_NIDX1)
    _check_in("D_idx", D_idx, SUPPORTED_D)


def _validate_inputs(query, key, query_index, key_index, weights, softmax_max, softmax_sum,
                     layout, sparse_mode, query_rope, key_rope, pre_tokens, next_tokens):
    """dense_loss_backward_triton.py:675-739; returns the rope dim (0 without rope)"""
    if query.dim() != 4 or key.dim() != 4:
        raise ValueError("query and key must be 4D BSND tensors")
    _validate_index_inputs(query_index, key_index, weights, layout, sparse_mode,
                           pre_tokens, next_tokens)
    if query.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"query dtype must be float16 or bfloat16, got {query.dtype}")
    if key.dtype != query.dtype or query_index.dtype != query.dtype or key_index.dtype != query.dtype:
        raise TypeError("query, key, query_index, and key_index must share dtype")
    if weights.dtype not in (query.dtype, torch.float32):
        raise TypeError("weights dtype must match query dtype or be float32")
    if softmax_max.dtype != torch.float32 or softmax_sum.dtype != torch.float32:
        raise TypeError("softmax_max and softmax_sum must be float32")
    B, S1, N1, D = query.shape
    if key.shape[0] != B or key.shape[3] != D:
        raise ValueError("key must be [B, S2, N2, D_attn]")
    N2 = key.shape[2]
    if N2 <= 0 or N1 % N2 != 0:
        raise ValueError("query N1 must be divisible by key N2")
    if query_index.shape[0] != B or query_index.shape[1] != S1:
        raise ValueError("query_index must share B and S1 with query")
    if key_index.shape[1] != key.shape[1]:
        raise ValueError("key_index S2 must match key S2")
    softmax_shape = (B, N2, S1, N1 // N2)
    if tuple(softmax_max.shape) != softmax_shape or tuple(softmax_sum.shape) != softmax_shape:
        raise ValueError(f"softmax_max and softmax_sum must be [B, N2, S1, G], got {tuple(softmax_max.shape)}")
    _check_in("D_attn", D, SUPPORTED_D)
    if (query_rope is None) != (key_rope is None):
        raise ValueError("query_rope and key_rope must be both provided or both omitted")
    if query_rope is None:
        return 0
    if query_rope.dim() != 4 or key_rope.dim() != 4:
        raise ValueError("query_rope and key_rope must be 4D BSND tensors")
    if tuple(query_rope.shape[:3]) != tuple(query.shape[:3]):
        raise ValueError("query_rope must share [B, S1, N1] with query")
    if tuple(key_rope.shape[:3]) != tuple(key.shape[:3]):
        raise ValueError("key_rope must share [B, S2, N2] with key")
    if query_rope.shape[3] != key_rope.shape[3]:
        raise ValueError("query_rope and key_rope must share Drope")
    if query_rope.shape[3] != 64:
        raise ValueError("Only Drope=64 is supported for query_rope/key_rope")
    if query_rope.dtype != query.dtype or key_rope.dtype != key.dtype:
        raise TypeError("query_rope/key_rope dtype must match query/key dtype")
    return 64


def _reshape_index_stat(stat, B, S1, name):
    """dense_loss_backward_triton.py:742-749"""
    if tuple(stat.shape) in ((B, S1), (B * S1,), (B, 1, S1), (B, 1, S1, 1)):
        return stat.reshape(B * S1).contiguous()
    raise ValueError(f"{name} must have shape [B,S1], [B*S1], [B,1,S1], or [B,1,S1,1], "
                     f"got {tuple(stat.shape)}")


def _index_params(query_index, key_index, weights, act_q, act_k, imax, isum):
    B, S1, Ni, Di = query_index.shape
    p = DenseIndexerParams()
    p.query_index, p.key_index, p.weights = ptr(query_index), ptr(key_index), ptr(weights)
    p.act_q, p.act_k = ptr(act_q), ptr(act_k)
    p.index_max, p.index_sum = ptr(imax), ptr(isum)
    p.batch, p.s1, p.s2, p.n_index, p.d_index = B, S1, key_index.shape[1], Ni, Di
    p.dtype = H.dtype_code(query_index)
    p.weights_dtype = DSA_DTYPE_FP32 if weights.dtype == torch.float32 else H.dtype_code(weights)
    return p


def _lse(query_index, key_index, weights, act_q, act_k):
    B, S1 = query_index.shape[0], query_index.shape[1]
    dev = query_index.device
    imax = torch.empty(B * S1, dtype=torch.float32, device=dev)
    isum = torch.empty(B * S1, dtype=torch.float32, device=dev)
    p = _index_params(query_index, key_index, weights, act_q, act_k, imax, isum)
    check(lib().dsa_dense_indexer_softmax_lse(p, stream_ptr(dev)), "dsa_dense_indexer_softmax_lse")
    return imax, isum


def npu_dense_lightning_indexer_softmax_lse_triton(
    query_index, key_index, weights, actual_seq_qlen=None, actual_seq_klen=None,
    layout="BSND", sparse_mode=3, pre_tokens=INT64_MAX, next_tokens=INT64_MAX,
):
    """Index softmax statistics over the visible keys: (softmax_max_index,
    softmax_sum_index), each fp32 [B, 1, S1] (dense_loss_backward_triton.py:817-845)."""
    _validate_index_inputs(query_index, key_index, weights, layout, sparse_mode,
                           pre_tokens, next_tokens)
    H.require_cuda(query_index, key_index, weights)
    B, S1 = query_index.shape[0], query_index.shape[1]
    dev = query_index.device
    act_q = H.lens_tensor(actual_seq_qlen, B, S1, dev)
    act_k = H.lens_tensor(actual_seq_klen, B, key_index.shape[1], dev)
    imax, isum = _lse(query_index.contiguous(), key_index.contiguous(), weights.contiguous(),
                      act_q, act_k)
    return imax.reshape(B, 1, S1), isum.reshape(B, 1, S1)


def dense_lightning_indexer_softmax_lse_triton(
    query_index, key_index, weights, actual_seq_qlen=None, actual_seq_klen=None,
    layout="BSND", sparse_mode=3, pre_tokens=INT64_MAX, next_tokens=INT64_MAX,
):
    return npu_dense_lightning_indexer_softmax_lse_triton(
        query_index, key_index, weights, actual_seq_qlen=actual_seq_qlen,
        actual_seq_klen=actual_seq_klen, layout=layout, sparse_mode=sparse_mode,
        pre_tokens=pre_tokens, next_tokens=next_tokens)


# MQA calls (one key head) whose shapes the SLI kernels take run through them: the dense
# KL loss over every visible key is the sparse one with the index set 0..S2-1, since the
# SLI's window keeps the first min(topK, act_k - act_q + s1 + 1) entries of a row
# (sparse_lightning_indexer_grad_kl_loss_triton.py:74-110) -- exactly the keys the dense
# reference sees (dense_loss_backward_triton.py:182-397) -- and the student softmax it
# forms over that set is the one the dense index statistics describe.  The tensor-core
# kernels then do the work; other shapes use the kernels of csrc/dense.cu.
_SLI_MAX_KEYS = 8192


def _full_query_lengths(actual_seq_qlen, S1):
    """True when no query row lies past its batch's actual length (the SLI window does not
    drop such rows; the dense loss gives them nothing)."""
    if actual_seq_qlen is None:
        return True
    if isinstance(actual_seq_qlen, int):
        return actual_seq_qlen == S1
    if isinstance(actual_seq_qlen, (list, tuple)):
        return all(int(x) == S1 for x in actual_seq_qlen)
    return False


def _sli_route_ok(query, key, query_index, N2, D, N1, actual_seq_qlen):
    Ni, Di = query_index.shape[2], query_index.shape[3]
    return (N2 == 1 and Di == 128 and Ni <= 64 and N1 <= 128 and D in (128, 256, 512)
            and key.shape[1] <= _SLI_MAX_KEYS and query.dtype in (torch.bfloat16, torch.float16)
            and _full_query_lengths(actual_seq_qlen, query.shape[1]))


def _dense_via_sli(query, key, query_index, key_index, weights, softmax_max, softmax_sum,
                   scale_value, query_rope, key_rope, act_q, act_k):
    from .sparse_lightning_indexer_grad_kl_loss import sparse_lightning_indexer_grad_kl_loss_triton
    B, S1 = query.shape[0], query.shape[1]
    S2 = key.shape[1]
    ids = torch.arange(S2, dtype=torch.int32, device=query.device)
    si = ids.view(1, 1, 1, S2).expand(B, S1, 1, S2)
    return sparse_lightning_indexer_grad_kl_loss_triton(
        query, key, query_index, key_index, weights, si, softmax_max, softmax_sum,
        query_rope=query_rope, key_rope=key_rope, actual_seq_qlen=act_q, actual_seq_klen=act_k,
        scale_value=scale_value, layout="BSND", sparse_mode=3)


def dense_loss_backward_triton(
    query, key, query_index, key_index, weights, softmax_max, softmax_sum,
    softmax_max_index=None, softmax_sum_index=None, scale_value=1.0,
    query_rope=None, key_rope=None, actual_seq_qlen=None, actual_seq_klen=None,
    layout="BSND", sparse_mode=3, pre_tokens=INT64_MAX, next_tokens=INT64_MAX,
):
    """Dense indexer KL-loss backward: (dQueryIndex, dKeyIndex, dWeights, loss [1] fp32, the
    KL divergence summed over query rows).  Without softmax_max_index / softmax_sum_index the
    index statistics are computed first (dense_loss_backward_triton.py:752-814).  MQA calls
    within the SLI kernels' limits run on them (tensor cores); they form the index softmax
    over the visible keys themselves, which given statistics of the same inputs describe."""
    d_rope = _validate_inputs(query, key, query_index, key_index, weights, softmax_max,
                              softmax_sum, layout, sparse_mode, query_rope, key_rope,
                              pre_tokens, next_tokens)
    if (softmax_max_index is None) != (softmax_sum_index is None):
        raise ValueError("softmax_max_index and softmax_sum_index must be both provided or both omitted")
    H.require_cuda(query, key, query_index, key_index, weights, softmax_max, softmax_sum,
                   query_rope, key_rope, softmax_max_index, softmax_sum_index)
    B, S1, N1, D = query.shape
    S2, N2 = key.shape[1], key.shape[2]
    Di = query_index.shape[3]
    dev = query.device
    if _sli_route_ok(query, key, query_index, N2, D, N1, actual_seq_qlen):
        if softmax_max_index is not None and (softmax_max_index.dtype != torch.float32
                                              or softmax_sum_index.dtype != torch.float32):
            raise TypeError("softmax_max_index and softmax_sum_index must be float32")
        return _dense_via_sli(query, key, query_index, key_index, weights, softmax_max,
                              softmax_sum, scale_value, query_rope, key_rope, actual_seq_qlen,
                              actual_seq_klen)
    act_q = H.lens_tensor(actual_seq_qlen, B, S1, dev)
    act_k = H.lens_tensor(actual_seq_klen, B, S2, dev)
    q, k, qi, ki, w = (t.contiguous() for t in (query, key, query_index, key_index, weights))
    qr = query_rope.contiguous() if d_rope else None
    kr = key_rope.contiguous() if d_rope else None
    if softmax_max_index is not None:
        if softmax_max_index.dtype != torch.float32 or softmax_sum_index.dtype != torch.float32:
            raise TypeError("softmax_max_index and softmax_sum_index must be float32")
        imax = _reshape_index_stat(softmax_max_index, B, S1, "softmax_max_index")
        isum = _reshape_index_stat(softmax_sum_index, B, S1, "softmax_sum_index")
    else:
        imax, isum = _lse(qi, ki, w, act_q, act_k)
    smax = softmax_max.contiguous()
    ssum = softmax_sum.contiguous()
    d_qi = torch.empty_like(qi)
    d_ki = torch.empty_like(ki)
    d_w = torch.empty_like(w)
    loss = torch.empty((1,), dtype=torch.float32, device=dev)
    ws_bytes = lib().dsa_dense_indexer_workspace_size(B, S1, S2, Di)
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    p = _index_params(qi, ki, w, act_q, act_k, imax, isum)
    p.query, p.key = ptr(q), ptr(k)
    p.query_rope, p.key_rope = (ptr(qr), ptr(kr)) if d_rope else (0, 0)
    p.softmax_max, p.softmax_sum = ptr(smax), ptr(ssum)
    p.d_query_index, p.d_key_index, p.d_weights, p.loss = ptr(d_qi), ptr(d_ki), ptr(d_w), ptr(loss)
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.n1, p.n2, p.d, p.d_rope = N1, N2, D, d_rope
    p.scale = float(scale_value)
    check(lib().dsa_dense_indexer_grad_kl_loss(p, stream_ptr(dev)), "dsa_dense_indexer_grad_kl_loss")
    return d_qi, d_ki, d_w, loss


def dense_lightning_indexer_grad_kl_loss_triton(
    query, key, query_index, key_index, weights, softmax_max, softmax_sum,
    softmax_max_index, softmax_sum_index, scale_value, query_rope=None, key_rope=None,
    actual_seq_qlen=None, actual_seq_klen=None, layout="BSND", sparse_mode=3,
    pre_tokens=INT64_MAX, next_tokens=INT64_MAX,
):
    """dense_loss_backward_triton.py:868-898"""
    return dense_loss_backward_triton(
        query, key, query_index, key_index, weights, softmax_max, softmax_sum,
        softmax_max_index, softmax_sum_index, scale_value, query_rope=query_rope,
        key_rope=key_rope, actual_seq_qlen=actual_seq_qlen, actual_seq_klen=actual_seq_klen,
        layout=layout, sparse_mode=sparse_mode, pre_tokens=pre_tokens, next_tokens=next_tokens)


npu_dense_lightning_indexer_grad_kl_loss_triton = dense_lightning_indexer_grad_kl_loss_triton


class DenseLightningIndexerSoftmaxLseTriton(torch.nn.Module):
    """Module wrapper (reference cell: dense_loss_backward_triton.py:933-952)."""

    def __init__(self, layout="BSND", sparse_mode=3, pre_tokens=INT64_MAX, next_tokens=INT64_MAX):
        super().__init__()
        self.layout, self.sparse_mode = layout, sparse_mode
        self.pre_tokens, self.next_tokens = pre_tokens, next_tokens

    def forward(self, query_index, key_index, weights, actual_seq_qlen=None, actual_seq_klen=None):
        return npu_dense_lightning_indexer_softmax_lse_triton(
            query_index, key_index, weights, actual_seq_qlen=actual_seq_qlen,
            actual_seq_klen=actual_seq_klen, layout=self.layout, sparse_mode=self.sparse_mode,
            pre_tokens=self.pre_tokens, next_tokens=self.next_tokens)


class DenseLossBackwardTriton(torch.nn.Module):
    """Module wrapper (reference cell: dense_loss_backward_triton.py:955-984)."""

    def __init__(self, scale_value=1.0, layout="BSND", sparse_mode=3, pre_tokens=INT64_MAX,
                 next_tokens=INT64_MAX):
        super().__init__()
        self.scale_value, self.layout, self.sparse_mode = scale_value, layout, sparse_mode
        self.pre_tokens, self.next_tokens = pre_tokens, next_tokens

    def forward(self, query, key, query_index, key_index, weights, softmax_max, softmax_sum,
                softmax_max_index=None, softmax_sum_index=None, scale_value=None,
                query_rope=None, key_rope=None, actual_seq_qlen=None, actual_seq_klen=None):
        scale = self.scale_value if scale_value is None else scale_value
        return dense_loss_backward_triton(
            query, key, query_index, key_index, weights, softmax_max, softmax_sum,
            softmax_max_index, softmax_sum_index, scale, query_rope=query_rope,
            key_rope=key_rope, actual_seq_qlen=actual_seq_qlen, actual_seq_klen=actual_seq_klen,
            layout=self.layout, sparse_mode=self.sparse_mode, pre_tokens=self.pre_tokens,
            next_tokens=self.next_tokens)


class DenseLightningIndexerGradKLLossTriton(DenseLossBackwardTriton):
    """dense_loss_backward_triton.py:987-988"""
