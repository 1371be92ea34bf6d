"""The dense indexer KL-loss oracle against the pinned sparse one (CPU).

With an index set that lists every visible key of a row (in order), the sparse KL-loss
gradient of ``sparse_lightning_indexer_grad_kl_loss_triton.py`` and the dense one of
``dense_loss_backward_triton.py`` are the same function (their student normalisations
differ by 1e-8 in the denominator), so ``oracle/dense.py`` is checked against
``oracle/sli.py``, which is pinned to the reference's numpy golden.
"""
import numpy as np
import pytest

import inputs as I
from oracle import dense, sli


@pytest.mark.parametrize("B,S1,S2,N1,Ni,act_q,act_k", [
    (1, 4, 64, 16, 8, None, None),
    (2, 3, 40, 8, 4, [3, 2], [40, 25]),
])
def test_dense_oracle_equals_sparse_oracle_on_full_index_sets(B, S1, S2, N1, Ni, act_q, act_k):
    rng = np.random.default_rng(3)
    D, Di = 128, 128
    q = I.randn(rng, (B, S1, N1, D), "bf16")
    k = I.randn(rng, (B, S2, 1, D), "bf16")
    qr = I.randn(rng, (B, S1, N1, 64), "bf16")
    kr = I.randn(rng, (B, S2, 1, 64), "bf16")
    qi = I.randn(rng, (B, S1, Ni, Di), "bf16")
    ki = I.randn(rng, (B, S2, 1, Di), "bf16")
    w = I.randn(rng, (B, S1, Ni), "fp32", scale=0.125)
    scale = 1 / np.sqrt(D + 64)
    smax, ssum = dense.attention_stats(q, k, qr, kr, scale, act_q, act_k)
    imax, isum = dense.dense_lse(qi, ki, w, act_q, act_k)
    dqi, dki, dw, loss = dense.dense_grad(q, k, qr, kr, qi, ki, w, smax, ssum, imax, isum, scale,
                                          act_q, act_k)
    si = np.broadcast_to(np.arange(S2, dtype=np.int32), (B, S1, 1, S2)).copy()
    ref = sli.sli_grad(q, k, qr, kr, qi, ki, w, si, smax.reshape(B, 1, S1, N1),
                       ssum.reshape(B, 1, S1, N1), scale, act_q, act_k)
    np.testing.assert_allclose(dqi, ref["dQueryIndex"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(dki, ref["dKeyIndex"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(dw, ref["dWeights"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(loss, float(np.asarray(ref["loss"]).reshape(-1)[0]), rtol=1e-5)
    assert abs(loss) > 0


def test_dense_lse_formula():
    rng = np.random.default_rng(5)
    qi = I.randn(rng, (1, 3, 4, 128), "bf16")
    ki = I.randn(rng, (1, 10, 1, 128), "bf16")
    w = np.abs(I.randn(rng, (1, 3, 4), "fp32"))
    mx, sm = dense.dense_lse(qi, ki, w, act_q=[3], act_k=[10])
    for s1 in range(3):
        vis = 10 - 3 + s1 + 1
        I_ = (w[0, s1, :, None] * np.maximum(qi[0, s1].astype(np.float64) @ ki[0, :vis, 0].T, 0)).sum(0)
        assert np.isclose(mx[0, 0, s1], I_.max(), rtol=1e-6)
        assert np.isclose(sm[0, 0, s1], np.exp(I_ - I_.max()).sum(), rtol=1e-6)
    mx2, sm2 = dense.dense_lse(qi, ki, w, act_q=[1], act_k=[10])
    assert mx2[0, 0, 1] == -np.inf and sm2[0, 0, 1] == 0
