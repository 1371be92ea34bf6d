"""Lightning indexer (score + top-k) on the B200 vs the numpy oracle (GPU).

The reference ships no golden for this operator, so the checks are against the oracle
restatement with the build contract's rule for top-k: indices bit-exact except where the
fp32 score lies within 1e-5 relative of the k-th score.
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import cuda, icuda, host
from oracle import li

pytestmark = pytest.mark.gpu


def check_topk(idx, val, scores, K, what=""):
    """idx/val [..., K] from the GPU, scores [..., S2] from the oracle."""
    idx = idx.reshape(-1, K)
    val = val.reshape(-1, K)
    sc = scores.reshape(-1, scores.shape[-1]).astype(np.float64)
    for r in range(sc.shape[0]):
        s = sc[r]
        finite = np.isfinite(s)
        nfin = int(finite.sum())
        g = idx[r]
        assert np.all(g[min(nfin, K):] == -1), f"{what} row {r}: -1 padding"
        gv = g[:min(nfin, K)]
        assert np.all(gv >= 0) and len(set(gv.tolist())) == len(gv), f"{what} row {r}: bad ids"
        if nfin == 0:
            continue
        srt = np.sort(s[finite])[::-1]
        kth = srt[min(K, nfin) - 1]
        tol = 1e-5 * abs(kth) + 1e-6
        assert np.all(s[gv] >= kth - tol), f"{what} row {r}: selected a score below the k-th"
        must = np.nonzero(finite & (s > kth + tol))[0]
        assert set(must.tolist()) <= set(gv.tolist()), f"{what} row {r}: missed a top score"
        ordered = s[gv]
        d = ordered[1:] - ordered[:-1]
        assert np.all(d <= 1e-5 * np.abs(ordered[:-1]) + 1e-6), f"{what} row {r}: not sorted"
        np.testing.assert_allclose(val[r, :len(gv)], s[gv], rtol=8e-3, atol=1e-3,
                                   err_msg=f"{what} row {r}: values")


def _run(c, K, mode, act_q=None, act_k=None, w_dtype="fp32", dt="bf16"):
    from dsa_triton_ascend_b200 import lightning_indexer_triton, check_device_errors
    w = torch.from_numpy(c["w"]).to("cuda", {"fp32": torch.float32, "bf16": torch.bfloat16,
                                             "fp16": torch.float16}[w_dtype])
    idx, val = lightning_indexer_triton(cuda(c["q"], dt), cuda(c["k"], dt), w,
                                        actual_seq_lengths_query=act_q,
                                        actual_seq_lengths_key=act_k, sparse_count=K,
                                        sparse_mode=mode, return_value=True)
    check_device_errors()
    return idx.cpu().numpy(), host(val), w.float().cpu().numpy()


# shapes of the reference's own test matrix (test_li_triton.py:42-52), S1 reduced for the
# oracle, plus the config-2 geometry (N1=64, D=128, N2=1) at reduced length
CASES = [
    (1, 1, 128, 8, 1, 128, 32),
    (2, 4, 256, 7, 1, 96, 32),
    (3, 8, 128, 16, 2, 64, 64),
    (1, 3, 256, 12, 4, 256, 32),
    (2, 64, 512, 64, 1, 128, 256),
    (1, 16, 300, 128, 1, 128, 128),
]


@pytest.mark.parametrize("mode", [0, 3])
@pytest.mark.parametrize("B,S1,S2,N1,N2,D,K", CASES)
def test_li_matches_oracle(B, S1, S2, N1, N2, D, K, mode):
    c = I.li_case(B, S1, S2, N1, N2, D, "bf16", seed=S1 * 7 + N1)
    idx, val, w = _run(c, K, mode)
    sc = li.li_score(c["q"], c["k"], w, sparse_mode=mode)
    check_topk(idx, val, sc, K, what=f"mode{mode}")


def test_li_actual_lengths_fp16_weights():
    c = I.li_case(3, 10, 200, 64, 1, 128, "fp16", seed=5)
    aq, ak = [10, 6, 8], [200, 120, 3]
    idx, val, w = _run(c, 64, 3, act_q=aq, act_k=ak, w_dtype="fp16", dt="fp16")
    sc = li.li_score(c["q"], c["k"], w, act_q=aq, act_k=ak, sparse_mode=3)
    check_topk(idx, val, sc, 64, what="lens")
    assert np.all(idx[1, 6:] == -1)


def test_li_exact_ties_ascending_index():
    """Duplicated key rows give exactly equal scores: ascending index must win."""
    c = I.li_case(1, 4, 256, 16, 1, 128, "bf16", seed=9)
    k = c["k"].copy()
    k[0, 1::2] = k[0, 0::2]          # keys 2j and 2j+1 identical
    c["k"] = k
    idx, val, w = _run(c, 64, 0)
    sc = li.li_score(c["q"], c["k"], w, sparse_mode=0)
    ref_idx, _ = li.li_topk(sc, 64)
    np.testing.assert_array_equal(idx, ref_idx)


def test_li_tnd_layout():
    from dsa_triton_ascend_b200 import lightning_indexer_triton, check_device_errors
    lq, lk = [5, 9], [150, 260]
    c = I.li_case(2, 9, 260, 32, 1, 128, "bf16", seed=3)
    cat = lambda x, l: np.concatenate([x[b, :l[b]] for b in range(2)])
    idx, val = lightning_indexer_triton(
        cuda(cat(c["q"], lq)), cuda(cat(c["k"], lk)),
        torch.from_numpy(cat(c["w"], lq)).cuda(),
        actual_seq_lengths_query=list(np.cumsum(lq)), actual_seq_lengths_key=list(np.cumsum(lk)),
        layout_query="TND", layout_key="TND", sparse_count=128, sparse_mode=3, return_value=True)
    check_device_errors()
    assert idx.shape == (14, 1, 128)
    for b in range(2):
        sc = li.li_score(c["q"][b:b + 1, :lq[b]], c["k"][b:b + 1, :lk[b]], c["w"][b:b + 1, :lq[b]],
                         sparse_mode=3)
        off = sum(lq[:b])
        # TND pads key rows to the longest batch: scores past lk[b] are -inf there
        scp = np.full(sc.shape[:-1] + (max(lk),), -np.inf, np.float32)
        scp[..., :lk[b]] = sc
        check_topk(idx[off:off + lq[b]].cpu().numpy(), host(val[off:off + lq[b]]), scp, 128,
                   what=f"tnd b{b}")


def test_li_scores_match_reference_golden_stage1():
    """Indexer scores of every visible key against the reference's own golden numbers.

    The fixtures hold the SLI golden's stage-1 scores I = sum_g w_g ReLU(qi_g . ki)
    (sli_grad_kl_loss_numpy.py:64-76) for index rows listing every visible key, i.e. the
    indexer's score row.  The golden rounds each dot product to fp16 and the kernel keeps
    it in fp32, and the returned values are in the query dtype (fp16 here), so the bound is
    a few fp16 ulps of the largest term.
    """
    from golden_io import load
    from gen_golden import LI_SCORE_CASES
    for name, B, S1, S2, N1, D, Nidx1, Di, seed in LI_SCORE_CASES:
        c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, S2, "causal_continuous", "fp16", seed)
        g = load(name)["I_scores"]
        c2 = dict(q=c["qi"], k=c["ki"], w=c["w"])
        idx, val, _ = _run(c2, S2, 3, dt="fp16")
        for s1 in range(S1):
            vis = S2 - S1 + s1 + 1
            got = np.full(S2, np.nan, np.float32)
            ids = idx[0, s1, 0, :vis]
            assert np.all(ids >= 0) and np.all(idx[0, s1, 0, vis:] == -1), f"{name} row {s1}"
            got[ids] = val[0, s1, 0, :vis]
            ref = g[0, s1, :vis]
            bound = 4e-3 * np.abs(ref) + 2e-3 * np.abs(ref).max()
            assert np.all(np.abs(got[:vis] - ref) <= bound), (
                f"{name} row {s1}: max err {np.nanmax(np.abs(got[:vis] - ref)):.3g}")
