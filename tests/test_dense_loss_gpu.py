"""Dense lightning-indexer KL loss (``dense_loss_backward_triton`` and its softmax-LSE
helper) on the B200 vs the numpy oracle ``oracle/dense.py`` (GPU).

Shapes are the reference's own test matrix (``test_dense_loss_backward_triton.py:19-50``:
B=1, S1=2..4, S2=64..128, N1=N2=32, every D_attn / Nidx1 / D_idx of the supported sets for
the statistics, the grad configurations), plus an MQA case with actual lengths, on seeded
fp16 / bf16 inputs. Tolerance: the reference test's (atol 1e-2, rtol 1e-4, :12-13), plus one
unit in the last place of the output's dtype where the operator returns fp16 / bf16 (the
gradients come back in the input dtypes, as in the reference, while the oracle is float64).
"""
import numpy as np
import pytest
import torch

import inputs as I
from oracle import dense

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 1e-4
SUP = (128, 256, 512)
LSE_CASES = [(1, 2, 64, 32, 32, d, ni, di) for d in SUP for ni in (32, 64, 128) for di in SUP] + [
    (1, 3, 96, 32, 32, 128, 32, 128), (1, 4, 128, 32, 32, 128, 32, 128)]
GRAD_CASES = [
    (1, 2, 64, 32, 32, 128, 32, 128),
    (1, 2, 64, 32, 32, 128, 64, 128),
    (1, 3, 96, 32, 32, 128, 32, 128),
    (1, 4, 128, 32, 32, 128, 32, 128),
    (1, 2, 64, 32, 32, 512, 128, 512),
]


def _inputs(B, S1, S2, N1, N2, D, Ni, Di, dt="fp16", seed=42):
    rng = np.random.default_rng(seed)
    q = I.randn(rng, (B, S1, N1, D), dt)
    k = I.randn(rng, (B, S2, N2, D), dt)
    qr = I.randn(rng, (B, S1, N1, 64), dt)
    kr = I.randn(rng, (B, S2, N2, 64), dt)
    qi = I.randn(rng, (B, S1, Ni, Di), dt)
    ki = I.randn(rng, (B, S2, 1, Di), dt)
    w = np.abs(I.randn(rng, (B, S1, Ni), dt))
    return q, k, qr, kr, qi, ki, w


def _t(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", {"fp16": torch.float16,
                                                                 "bf16": torch.bfloat16,
                                                                 "fp32": torch.float32}[dt])


ULP = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7, torch.float32: 0.0}


def _close(got, ref, what):
    ulp = ULP[got.dtype]
    got = got.float().cpu().numpy().reshape(np.shape(ref))
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL + ulp, err_msg=what)


@pytest.mark.parametrize("B,S1,S2,N1,N2,D,Ni,Di", LSE_CASES)
def test_dense_softmax_lse(B, S1, S2, N1, N2, D, Ni, Di):
    import dsa_triton_ascend_b200 as dsa
    _, _, _, _, qi, ki, w = _inputs(B, S1, S2, N1, N2, D, Ni, Di)
    mx, sm = dsa.DenseLightningIndexerSoftmaxLseTriton()(_t(qi, "fp16"), _t(ki, "fp16"), _t(w, "fp16"))
    assert mx.shape == (B, 1, S1) and mx.dtype == torch.float32
    rmx, rsm = dense.dense_lse(qi, ki, w)
    _close(mx, rmx, "softmax_max_index")
    _close(sm, rsm, "softmax_sum_index")


@pytest.mark.parametrize("B,S1,S2,N1,N2,D,Ni,Di", GRAD_CASES)
def test_dense_grad_kl_loss(B, S1, S2, N1, N2, D, Ni, Di):
    """Two-stage path (statistics from the LSE helper) and the path that computes them."""
    import dsa_triton_ascend_b200 as dsa
    q, k, qr, kr, qi, ki, w = _inputs(B, S1, S2, N1, N2, D, Ni, Di)
    scale = 1.0 / np.sqrt(D + 64)
    smax, ssum = dense.attention_stats(q, k, qr, kr, scale)
    imax, isum = dense.dense_lse(qi, ki, w)
    rdqi, rdki, rdw, rloss = dense.dense_grad(q, k, qr, kr, qi, ki, w, smax, ssum, imax, isum, scale)
    tq, tk, tqr, tkr, tqi, tki, tw = (_t(x, "fp16") for x in (q, k, qr, kr, qi, ki, w))
    tsm, tss = _t(smax, "fp32"), _t(ssum, "fp32")
    mx, sm = dsa.dense_lightning_indexer_softmax_lse_triton(tqi, tki, tw)
    cell = dsa.DenseLightningIndexerGradKLLossTriton(scale_value=scale)
    outs = [cell(tq, tk, tqi, tki, tw, tsm, tss, mx, sm, query_rope=tqr, key_rope=tkr),
            dsa.dense_loss_backward_triton(tq, tk, tqi, tki, tw, tsm, tss, scale_value=scale,
                                           query_rope=tqr, key_rope=tkr)]
    torch.cuda.synchronize()
    for dqi, dki, dw, loss in outs:
        assert dqi.dtype == tqi.dtype and dki.dtype == tki.dtype and dw.dtype == tw.dtype
        assert loss.shape == (1,) and loss.dtype == torch.float32
        _close(dqi, rdqi, "dQueryIndex")
        _close(dki, rdki, "dKeyIndex")
        _close(dw, rdw, "dWeights")
        _close(loss, np.array([rloss]), "loss")
    assert abs(rloss) > 0 and float(np.abs(rdqi).max()) > 1e-3


def test_dense_grad_mqa_bf16_actual_lengths_fp32_weights():
    """One key head (the DSA shape), bf16, fp32 weights, no rope, actual lengths with a row
    past act_q (zeros) and a batch whose keys end early."""
    import dsa_triton_ascend_b200 as dsa
    B, S1, S2, N1, N2, D, Ni, Di = 2, 3, 80, 16, 1, 256, 32, 128
    q, k, _, _, qi, ki, w = _inputs(B, S1, S2, N1, N2, D, Ni, Di, dt="bf16", seed=7)
    w = I.randn(np.random.default_rng(8), (B, S1, Ni), "fp32", scale=0.5)
    act_q, act_k = [3, 2], [80, 40]
    scale = 1.0 / np.sqrt(D)
    smax, ssum = dense.attention_stats(q, k, None, None, scale, act_q, act_k)
    imax, isum = dense.dense_lse(qi, ki, w, act_q, act_k)
    rdqi, rdki, rdw, rloss = dense.dense_grad(q, k, None, None, qi, ki, w, smax, ssum, imax, isum,
                                              scale, act_q, act_k)
    dqi, dki, dw, loss = dsa.dense_loss_backward_triton(
        _t(q, "bf16"), _t(k, "bf16"), _t(qi, "bf16"), _t(ki, "bf16"), _t(w, "fp32"),
        _t(smax, "fp32"), _t(ssum, "fp32"), scale_value=scale, actual_seq_qlen=act_q,
        actual_seq_klen=act_k)
    torch.cuda.synchronize()
    assert dw.dtype == torch.float32
    _close(dqi, rdqi, "dQueryIndex")
    _close(dki, rdki, "dKeyIndex")
    _close(dw, rdw, "dWeights")
    _close(loss, np.array([rloss]), "loss")
    assert float(dqi[1, 2].abs().max()) == 0.0


@pytest.mark.parametrize("D,Ni,dt,rope", [(512, 64, "bf16", True), (128, 32, "fp16", False)])
def test_dense_grad_mqa_tensor_core_route(D, Ni, dt, rope):
    """MQA with the SLI kernels' shapes (one key head, D_idx 128, at most 64 index heads):
    the call runs on the tensor-core SLI kernels over the index set 0..S2-1; it must equal
    the dense oracle and the CUDA-core dense kernels, with given and with computed index
    statistics, and with a batch whose keys end early."""
    import dsa_triton_ascend_b200 as dsa
    import dsa_triton_ascend_b200.dense_indexer_loss as dil
    B, S1, S2, N1, N2, Di = 2, 24, 160, 32, 1, 128
    q, k, qr, kr, qi, ki, w = _inputs(B, S1, S2, N1, N2, D, Ni, Di, dt=dt, seed=11)
    w = I.randn(np.random.default_rng(12), (B, S1, Ni), "fp32", scale=0.5)
    if not rope:
        qr = kr = None
    act_k = [S2, 150]
    scale = 1.0 / np.sqrt(D + (64 if rope else 0))
    smax, ssum = dense.attention_stats(q, k, qr, kr, scale, None, act_k)
    imax, isum = dense.dense_lse(qi, ki, w, None, act_k)
    ref = dense.dense_grad(q, k, qr, kr, qi, ki, w, smax, ssum, imax, isum, scale, None, act_k)
    tq, tk, tqi, tki = (_t(x, dt) for x in (q, k, qi, ki))
    tw, tsm, tss = _t(w, "fp32"), _t(smax, "fp32"), _t(ssum, "fp32")
    kw = dict(scale_value=scale, actual_seq_klen=act_k)
    if rope:
        kw.update(query_rope=_t(qr, dt), key_rope=_t(kr, dt))
    assert dil._sli_route_ok(tq, tk, tqi, 1, D, N1, None)
    mx, sm = dsa.dense_lightning_indexer_softmax_lse_triton(tqi, tki, tw, actual_seq_klen=act_k)
    got = [dsa.dense_loss_backward_triton(tq, tk, tqi, tki, tw, tsm, tss, **kw),
           dsa.dense_loss_backward_triton(tq, tk, tqi, tki, tw, tsm, tss, mx, sm, **kw)]
    saved = dil._SLI_MAX_KEYS
    try:
        dil._SLI_MAX_KEYS = 0           # the CUDA-core kernels for the same call
        cuda_core = dsa.dense_loss_backward_triton(tq, tk, tqi, tki, tw, tsm, tss, **kw)
    finally:
        dil._SLI_MAX_KEYS = saved
    torch.cuda.synchronize()
    for out in got + [cuda_core]:
        for g, r, name in zip(out, ref, ("dQueryIndex", "dKeyIndex", "dWeights", "loss")):
            _close(g, np.atleast_1d(r), name)
    for g, c in zip(got[0], cuda_core):
        torch.testing.assert_close(g.float(), c.float(), rtol=2e-2, atol=2e-3)
