"""Autograd functions and the indexer -> attention -> KL-loss module vs direct calls (GPU)."""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import OUT_ATOL, OUT_RTOL

pytestmark = pytest.mark.gpu

bf16 = torch.bfloat16


def _t(x, grad=False, dt=bf16):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dt)
    return t.requires_grad_(grad)


def test_sfa_function_grads_match_grad_operator():
    import dsa_triton_ascend_b200 as dsa
    c = I.sfa_case(1, 64, 256, 16, 512, 96, 1, 3, "bf16", seed=41)
    q, k, qr, kr = (_t(c[n], True) for n in ("q", "k", "qr", "kr"))
    si = torch.from_numpy(np.ascontiguousarray(c["si"], np.int32)).cuda()
    g = _t(c["dout"])
    out, smax, ssum = dsa.SparseFlashAttentionFunction.apply(q, k, qr, kr, si, c["scale"], 3)
    (out.float() * g.float()).sum().backward()
    (dk_acc, _, dv_acc), finish = dsa.sparse_flash_attention_grad_partial(
        q.detach(), k.detach(), k.detach(), si, g, out.detach(), smax, ssum, c["scale"],
        query_rope=qr.detach(), key_rope=kr.detach(), sparse_mode=3)
    dkv = (dk_acc + dv_acc).to(k.dtype).view(k.shape)   # key = value: dk + dv rounded once
    dq, dk, dv, dqr, dkr = finish()
    tol = dict(rtol=OUT_RTOL, atol=OUT_ATOL)
    torch.testing.assert_close(q.grad.float(), dq.float(), **tol)
    torch.testing.assert_close(k.grad.float(), dkv.float(), **tol)
    torch.testing.assert_close(qr.grad.float(), dqr.float(), **tol)
    torch.testing.assert_close(kr.grad.float(), dkr.float(), **tol)


def test_indexer_kl_loss_function_matches_operator():
    import dsa_triton_ascend_b200 as dsa
    c = I.sli_case(1, 64, 256, 16, 512, 64, 128, 64, "causal_random", "bf16", seed=42)
    from oracle import sli
    smx, ssm = sli.softmax_stats_full(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
    qi, ki = _t(c["qi"], True), _t(c["ki"], True)
    w = torch.from_numpy(np.ascontiguousarray(c["w"], np.float32)).cuda().requires_grad_(True)
    q, k, qr, kr = (_t(c[n]) for n in ("q", "k", "qr", "kr"))
    si = torch.from_numpy(np.ascontiguousarray(c["si"], np.int32)).cuda()
    mx = torch.from_numpy(smx.astype(np.float32)).cuda()
    sm = torch.from_numpy(ssm.astype(np.float32)).cuda()
    loss = dsa.IndexerKLLossFunction.apply(qi, ki, w, q, k, qr, kr, si, mx, sm, c["scale"])
    (2.0 * loss).backward()
    d_qi, d_ki, d_w, ref_loss = dsa.sparse_lightning_indexer_grad_kl_loss_triton(
        q, k, qi.detach(), ki.detach(), w.detach(), si, mx, sm, query_rope=qr, key_rope=kr,
        scale_value=c["scale"])
    torch.testing.assert_close(loss.detach().reshape(1), ref_loss, rtol=1e-4, atol=1e-6)
    tol = dict(rtol=OUT_RTOL, atol=OUT_ATOL)
    torch.testing.assert_close(qi.grad.float(), 2.0 * d_qi.float(), **tol)
    torch.testing.assert_close(ki.grad.float(), 2.0 * d_ki.float(), **tol)
    torch.testing.assert_close(w.grad.float(), 2.0 * d_w.float(), **tol)


def test_sparse_attention_with_indexer_trains():
    """One step of the composed layer: finite output and loss, gradients on both sides."""
    import dsa_triton_ascend_b200 as dsa
    c = I.sli_case(1, 128, 512, 16, 512, 64, 128, 64, "causal_random", "bf16", seed=43)
    q, k, qr, kr = (_t(c[n], True) for n in ("q", "k", "qr", "kr"))
    qi, ki = _t(c["qi"], True), _t(c["ki"], True)
    w = torch.from_numpy(np.ascontiguousarray(c["w"], np.float32)).cuda().requires_grad_(True)
    layer = dsa.SparseAttentionWithIndexer(scale_value=c["scale"], sparse_count=64)
    out, loss = layer(q, k, qr, kr, qi, ki, w)
    (out.float().square().mean() + loss).backward()
    torch.cuda.synchronize()
    dsa.check_device_errors()
    assert torch.isfinite(out.float()).all() and torch.isfinite(loss)
    assert float(loss.detach()) > 0
    for t in (q, k, qr, kr, qi, ki, w):
        assert t.grad is not None and torch.isfinite(t.grad.float()).all()
        assert float(t.grad.float().abs().sum()) > 0


@pytest.mark.parametrize("S,topk", [(128, 64), (512, 256)])
def test_indexer_teacher_from_attention_backward_matches(S, topk):
    """teacher_from_backward: the loss formed in backward from the attention backward's P
    (no teacher pass) equals the standard path's loss within the loss tolerance, and every
    gradient agrees; the output is the same call."""
    import dsa_triton_ascend_b200 as dsa
    c = I.sli_case(1, S, S, 16, 512, 64, 128, topk, "causal_random", "bf16", seed=44)
    res = []
    for fused in (False, True):
        q, k, qr, kr = (_t(c[n], True) for n in ("q", "k", "qr", "kr"))
        qi, ki = _t(c["qi"], True), _t(c["ki"], True)
        w = torch.from_numpy(np.ascontiguousarray(c["w"], np.float32)).cuda().requires_grad_(True)
        layer = dsa.SparseAttentionWithIndexer(scale_value=c["scale"], sparse_count=topk,
                                               teacher_from_backward=fused)
        out, loss = layer(q, k, qr, kr, qi, ki, w)
        g = torch.from_numpy(np.ascontiguousarray(c["dout"])).cuda().to(bf16) if "dout" in c else None
        obj = (out.float() * (g.float() if g is not None else 1.0)).sum() + 0.5 * loss
        obj.backward()
        torch.cuda.synchronize()
        dsa.check_device_errors()
        res.append((out.detach(), float(loss.detach()), [t.grad.float() for t in (q, k, qr, kr, qi, ki, w)]))
    (o0, l0, g0), (o1, l1, g1) = res
    torch.testing.assert_close(o1, o0, rtol=0, atol=0)
    assert l0 > 0 and abs(l1 - l0) <= 1e-4 * abs(l0) + 1e-6
    names = ("q", "k", "qr", "kr", "qi", "ki", "w")
    for a, b, n in zip(g1, g0, names):
        # attention gradients: the merged key gradient is the same sum rounded once; index
        # gradients: the same loss kernel fed a teacher summed in another order
        torch.testing.assert_close(a, b, rtol=OUT_RTOL, atol=OUT_ATOL * max(1.0, float(b.abs().max())),
                                   msg=lambda m: f"{n}: {m}")
