"""Pin the CPU oracle against the reference's own numpy goldens (CPU only).

The fixtures were produced by ``tests/golden/gen_golden.py`` from the unmodified
reference goldens; the inputs are regenerated here from the same seeds.
"""
import numpy as np
import pytest

import inputs as I
from gen_golden import SFA_FWD_CASES, SFA_BWD_CASES, SLI_CASES, CONFIG1_ROWS, LI_SCORE_CASES
from golden_io import load, from_bits16
from oracle import sfa, sli, li


def _close(a, b, rtol, atol):
    np.testing.assert_allclose(np.asarray(a, np.float32), np.asarray(b, np.float32),
                               rtol=rtol, atol=atol)


@pytest.mark.parametrize("case", SFA_FWD_CASES, ids=[c[0] for c in SFA_FWD_CASES])
def test_sfa_fwd_oracle_matches_golden(case):
    name, B, S1, S2, N1, D, cnt, blk, mode, dt, seed = case
    c = I.sfa_case(B, S1, S2, N1, D, cnt, blk, mode, dt, seed)
    g = load(name)
    tok = sfa.expand_block_indices(c["si"], blk)
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["scale"],
                              sparse_mode=mode, dtype=dt)
    # same arithmetic as the golden up to summation order: bf16/fp16 output ulp level
    _close(out, from_bits16(g["out"], dt), rtol=1e-2, atol=1e-3)
    _close(mx, g["softmax_max"], rtol=1e-6, atol=1e-6)
    _close(sm, g["softmax_sum"], rtol=1e-5, atol=1e-6)


def test_sfa_fwd_oracle_config1_rows():
    c = I.config1()
    g = load("config1")
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              sparse_mode=3, dtype="bf16")
    _close(out[:, CONFIG1_ROWS], from_bits16(g["out_rows"], "bf16"), rtol=1e-2, atol=1e-3)
    _close(mx, g["softmax_max"], rtol=1e-6, atol=1e-6)
    _close(sm, g["softmax_sum"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", SFA_BWD_CASES, ids=[c[0] for c in SFA_BWD_CASES])
def test_sfa_bwd_oracle_matches_golden(case):
    name, B, S1, S2, N1, D, cnt, blk, mode, dt, seed = case
    c = I.sfa_case(B, S1, S2, N1, D, cnt, blk, mode, dt, seed)
    g = load(name)
    tok = sfa.expand_block_indices(c["si"], blk)
    out = from_bits16(g["out"], dt)
    res = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["dout"], out,
                      g["softmax_max"], g["softmax_sum"], c["scale"], sparse_mode=mode, dtype=dt)
    for got, key in zip(res, ("dq", "dk", "dv", "dqr", "dkr")):
        _close(got, from_bits16(g[key], dt), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("case", SLI_CASES, ids=[c[0] for c in SLI_CASES])
def test_sli_oracle_matches_golden(case):
    name, B, S1, S2, N1, D, Nidx1, Di, topK, pat, seed = case
    c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, topK, pat, "fp16", seed)
    g = load(name)
    r = sli.sli_grad(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"], c["w"], c["si"],
                     g["softmax_max"], g["softmax_sum"], c["scale"], emulate_fp16=True)
    _close(r["dQueryIndex"], g["dQueryIndex"], rtol=1e-4, atol=1e-5)
    _close(r["dKeyIndex"], g["dKeyIndex"], rtol=1e-4, atol=1e-5)
    _close(r["dWeights"], g["dW"], rtol=1e-4, atol=1e-5)
    _close(r["loss"], g["loss"], rtol=1e-5, atol=1e-6)


def test_sli_fp32_mode_close_to_golden():
    """The kernel-faithful fp32 mode stays within the reference test's 1e-2 band."""
    name, B, S1, S2, N1, D, Nidx1, Di, topK, pat, seed = SLI_CASES[0]
    c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, topK, pat, "fp16", seed)
    g = load(name)
    r = sli.sli_grad(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"], c["w"], c["si"],
                     g["softmax_max"], g["softmax_sum"], c["scale"])
    _close(r["dWeights"], g["dW"], rtol=1e-2, atol=1e-2)
    _close(r["loss"], g["loss"], rtol=1e-2, atol=1e-2)


def test_li_oracle_known_answers():
    """Hand-computed cases (no reference golden exists for the indexer)."""
    q = np.zeros((1, 3, 2, 4), np.float32)
    k = np.zeros((1, 4, 1, 4), np.float32)
    w = np.ones((1, 3, 2), np.float32)
    k[0, :, 0, 0] = [1.0, 2.0, -1.0, 2.0]
    q[0, :, 0, 0] = 1.0                       # head 0 sees +k
    q[0, :, 1, 0] = -1.0                      # head 1 sees -k (ReLU kills positives)
    w[0, :, 1] = 0.5
    s = li.li_score(q, k, w, sparse_mode=3, act_q=[3], act_k=[4])
    # row s1 sees keys < act_k - act_q + s1 + 1 = s1 + 2
    exp_full = np.array([1.0, 2.0, 0.5, 2.0], np.float32)
    for s1 in range(3):
        lim = s1 + 2
        np.testing.assert_array_equal(s[0, s1, 0, :lim], exp_full[:lim])
        assert np.all(np.isneginf(s[0, s1, 0, lim:]))
    idx, val = li.li_topk(s, 4)
    # ties (score 2.0 at ids 1 and 3) resolve by ascending index; -inf -> -1
    np.testing.assert_array_equal(idx[0, 2, 0], [1, 3, 0, 2])
    np.testing.assert_array_equal(idx[0, 0, 0], [1, 0, -1, -1])
    s0 = li.li_score(q, k, w, sparse_mode=0, act_q=[2], act_k=[3])
    assert np.all(np.isneginf(s0[0, 2]))                     # inactive row
    np.testing.assert_array_equal(s0[0, 0, 0, :3], exp_full[:3])
    assert np.isneginf(s0[0, 0, 0, 3])


def test_li_topk_ragged_and_short():
    sc = np.array([[3.0, -np.inf, 3.0, 1.0, -np.inf]], np.float32)
    idx, val = li.li_topk(sc, 5)
    np.testing.assert_array_equal(idx[0], [0, 2, 3, -1, -1])
    idx2, _ = li.li_topk(sc, 2)
    np.testing.assert_array_equal(idx2[0], [0, 2])


@pytest.mark.parametrize("case", LI_SCORE_CASES, ids=[c[0] for c in LI_SCORE_CASES])
def test_li_score_oracle_matches_sli_golden_stage1(case):
    """The indexer's score arithmetic, pinned to the reference's own golden.

    The SLI golden's stage 1 (sli_grad_kl_loss_numpy.py:64-76) computes
    I = sum_g w_g ReLU(qi_g . ki) for the keys listed in each index row.  With rows that
    list every visible key in order (causal_continuous, topK = S2) that is the indexer's
    score of every visible key under sparse_mode 3 (lightning_indexer_triton.py:202-280).
    The golden rounds its inputs and every dot product to fp16; so does the oracle here.
    """
    name, B, S1, S2, N1, D, Nidx1, Di, seed = case
    c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, S2, "causal_continuous", "fp16", seed)
    g = load(name)["I_scores"]                                   # [B, S1, topK = S2]
    sc = li.li_score(c["qi"], c["ki"], c["w"], sparse_mode=3, emulate_fp16=True)
    for s1 in range(S1):
        vis = S2 - S1 + s1 + 1
        assert np.all(np.isneginf(sc[0, s1, 0, vis:]))
        # fp32 summation order differs (one fp16 ulp of a dot product at most)
        _close(sc[0, s1, 0, :vis], g[0, s1, :vis], rtol=1e-4, atol=2e-3)
    # the same scores without fp16 emulation stay within the fp16 rounding band
    sc32 = li.li_score(c["qi"], c["ki"], c["w"], sparse_mode=3)
    vis = S2 - S1 + 1
    _close(sc32[0, 0, 0, :vis], g[0, 0, :vis], rtol=2e-2, atol=2e-2)
