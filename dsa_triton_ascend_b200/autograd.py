"""Autograd integration: the DSA operators as differentiable torch functions.

The reference wires its backward operators into the framework's autodiff by hand (the
bprop attached to the forward in sparse_flash_attention_grad_triton.py:30-70): d(out)
feeds sparse_flash_attention_grad, and since MLA-absorb uses one latent tensor as both
key and value, the key gradient handed back is dk + dv.  This module does the same for
torch:

* :class:`SparseFlashAttentionFunction` -- forward with softmax statistics, backward
  through the B200 kernels; returns the merged key gradient.
* :class:`IndexerKLLossFunction` -- the lightning indexer's KL loss against the attention
  distribution; the SLI kernel computes the loss and its gradients (dQueryIndex,
  dKeyIndex, dWeights) in one pass, and backward scales them by d(loss).
* :class:`SparseAttentionWithIndexer` -- lightning indexer (top-k, not differentiated)
  -> sparse attention -> indexer KL loss, the training-time composition of a DSA layer
  (cf. dsa_torch.py:111-151).
"""
from __future__ import annotations

import torch

from . import _host as H

from .lightning_indexer import lightning_indexer_triton
from .sparse_flash_attention import sparse_flash_attention_triton
from .sparse_flash_attention_grad import sparse_flash_attention_grad_merged
from .sparse_lightning_indexer_grad_kl_loss import sparse_lightning_indexer_grad_kl_loss_triton


class SparseFlashAttentionFunction(torch.autograd.Function):
    """out, softmax_max, softmax_sum = f(query, key, query_rope, key_rope, sparse_indices).

    BSND or TND query, BSND/TND key (value = key[..., :D]); the statistics are returned
    for the indexer loss and carry no gradient.  Gradients: query, key (dk + dv),
    query_rope, key_rope."""

    @staticmethod
    def forward(ctx, query, key, query_rope, key_rope, sparse_indices, scale_value=1.0,
                sparse_mode=3, actual_seq_lengths_query=None, actual_seq_lengths_kv=None,
                sparse_block_size=1, layout="BSND"):
        out, smax, ssum = sparse_flash_attention_triton(
            query, key, key, sparse_indices, scale_value,
            actual_seq_lengths_query=actual_seq_lengths_query,
            actual_seq_lengths_kv=actual_seq_lengths_kv, query_rope=query_rope,
            key_rope=key_rope, sparse_block_size=sparse_block_size, layout_query=layout,
            layout_kv=layout, sparse_mode=sparse_mode, return_softmax_lse=True)
        ctx.save_for_backward(query, key, query_rope, key_rope, sparse_indices, out, smax, ssum)
        ctx.cfg = (scale_value, sparse_mode, actual_seq_lengths_query, actual_seq_lengths_kv,
                   sparse_block_size, layout)
        ctx.mark_non_differentiable(smax, ssum)
        return out, smax, ssum

    @staticmethod
    def backward(ctx, d_out, _d_smax, _d_ssum):
        query, key, query_rope, key_rope, sparse_indices, out, smax, ssum = ctx.saved_tensors
        scale, mode, aq, ak, block, layout = ctx.cfg
        # key == value: the merged kernels accumulate dK + dV directly
        dq, dkv, dqr, dkr = sparse_flash_attention_grad_merged(
            query, key, sparse_indices, d_out.contiguous(), out, smax, ssum, scale,
            query_rope=query_rope, key_rope=key_rope, actual_seq_lengths_query=aq,
            actual_seq_lengths_kv=ak, sparse_block_size=block, layout=layout, sparse_mode=mode)
        return dq, dkv, dqr, dkr, None, None, None, None, None, None, None


class IndexerKLLossFunction(torch.autograd.Function):
    """loss = f(query_index, key_index, weights; attention tensors and statistics).

    The attention side (query, key, ropes, softmax statistics) is the teacher and gets no
    gradient; the indexer side gets dQueryIndex, dKeyIndex and dWeights times d(loss)."""

    @staticmethod
    def forward(ctx, query_index, key_index, weights, query, key, query_rope, key_rope,
                sparse_indices, softmax_max, softmax_sum, scale_value=1.0):
        d_qi, d_ki, d_w, loss = sparse_lightning_indexer_grad_kl_loss_triton(
            query, key, query_index, key_index, weights, sparse_indices, softmax_max,
            softmax_sum, query_rope=query_rope, key_rope=key_rope, scale_value=scale_value)
        ctx.save_for_backward(d_qi, d_ki, d_w)
        return loss.reshape(())

    @staticmethod
    def backward(ctx, d_loss):
        d_qi, d_ki, d_w = ctx.saved_tensors
        g = d_loss.to(torch.float32)
        scale = lambda t: (t.float() * g).to(t.dtype)
        return (scale(d_qi), scale(d_ki), scale(d_w), None, None, None, None, None, None, None,
                None)


class _AttentionWithIndexerLoss(torch.autograd.Function):
    """(out, loss) = f(query, key, query_rope, key_rope, query_index, key_index, weights;
    sparse_indices) with the indexer KL loss formed in backward.

    The loss's teacher is the attention distribution (1/N1) sum_h P over each row's
    selected keys; the attention backward's first kernel forms exactly these P, so it adds
    them up for the loss on the way (`teacher` in DsaSfaBwdParams) and the loss kernel runs
    without its own pass over the keys (`teacher` in DsaSliParams).  The loss value exists
    only once the backward has run: the tensor returned by forward holds 0 until then and
    is filled in place (read it after backward())."""

    @staticmethod
    def forward(ctx, query, key, query_rope, key_rope, query_index, key_index, weights,
                sparse_indices, scale_value):
        out, smax, ssum = sparse_flash_attention_triton(
            query, key, key, sparse_indices, scale_value, query_rope=query_rope,
            key_rope=key_rope, sparse_mode=3, return_softmax_lse=True)
        loss = torch.zeros((), dtype=torch.float32, device=query.device)
        ctx.save_for_backward(query, key, query_rope, key_rope, query_index, key_index, weights,
                              sparse_indices, out, smax, ssum)
        ctx.loss = loss
        ctx.scale = scale_value
        return out, loss

    @staticmethod
    def backward(ctx, d_out, d_loss):
        from .sparse_flash_attention_grad import _sfa_grad
        from .sparse_lightning_indexer_grad_kl_loss import _sli
        (query, key, query_rope, key_rope, query_index, key_index, weights, sparse_indices,
         out, smax, ssum) = ctx.saved_tensors
        B, S1 = query.shape[0], query.shape[1]
        topk = sparse_indices.shape[-1]
        teacher = torch.zeros(B * S1 * topk, dtype=torch.float32, device=query.device)
        if d_out is None:
            d_out = torch.zeros_like(out)
        dq, dkv, dqr, dkr = _sfa_grad(
            query, key, key, sparse_indices, d_out.contiguous(), out, smax, ssum, ctx.scale,
            query_rope, key_rope, None, None, 1, "BSND", 3, H.INT64_MAX, H.INT64_MAX, False,
            defer_cast=False, merged=True, teacher=teacher)
        d_qi, d_ki, d_w, loss = _sli(
            query, key, query_index, key_index, weights, sparse_indices, smax, ssum, query_rope,
            key_rope, None, None, ctx.scale, "BSND", 3, defer_cast=False, teacher=teacher)
        ctx.loss.copy_(loss.reshape(()))
        g = (d_loss if d_loss is not None else torch.ones((), device=query.device)).to(torch.float32)
        return (dq, dkv, dqr, dkr, (d_qi.float() * g).to(d_qi.dtype),
                (d_ki.float() * g).to(d_ki.dtype), (d_w.float() * g).to(d_w.dtype), None, None)


class SparseAttentionWithIndexer(torch.nn.Module):
    """Lightning indexer -> sparse flash attention -> indexer KL loss (BSND, causal).

    forward(query, key, query_rope, key_rope, query_index, key_index, weights) returns
    (attention_out, indexer_loss); attention_out is differentiable in the attention
    inputs, indexer_loss in the indexer inputs (query_index, key_index, weights).  The
    top-k selection itself has no gradient, as in the reference's training setup."""

    def __init__(self, scale_value: float, sparse_count: int = 2048,
                 teacher_from_backward: bool = False):
        """``teacher_from_backward=True``: the indexer loss is formed in backward from the
        attention backward's probabilities (no second pass over the keys for the teacher);
        the returned loss then holds its value only after backward() has run."""
        super().__init__()
        self.scale_value = scale_value
        self.sparse_count = sparse_count
        self.teacher_from_backward = teacher_from_backward

    def forward(self, query, key, query_rope, key_rope, query_index, key_index, weights):
        with torch.no_grad():
            sparse_indices, _ = lightning_indexer_triton(
                query_index.detach(), key_index.detach(), weights.detach(),
                sparse_count=self.sparse_count, sparse_mode=3)
        if self.teacher_from_backward:
            return _AttentionWithIndexerLoss.apply(
                query, key, query_rope, key_rope, query_index, key_index, weights,
                sparse_indices, self.scale_value)
        out, smax, ssum = SparseFlashAttentionFunction.apply(
            query, key, query_rope, key_rope, sparse_indices, self.scale_value, 3)
        loss = IndexerKLLossFunction.apply(
            query_index, key_index, weights, query.detach(), key.detach(), query_rope.detach(),
            key_rope.detach(), sparse_indices, smax, ssum, self.scale_value)
        return out, loss
