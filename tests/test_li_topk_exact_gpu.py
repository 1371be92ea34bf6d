"""Lightning-indexer top-k, bit-exact (GPU).

The fp32 scores the score kernel wrote are read back from the caller's workspace, and the
top-k of each row must equal a stable sort of exactly those scores by (score desc, index
asc) over the row's visible keys (the reference's ``_stable_topk`` order,
lightning_indexer_triton.py:339-357), with -1 past the visible keys.  The cases cover the
bucket path (spread-out scores, with and without exact ties) and the radix path (one
outlier score that crowds the others into a few buckets, all-equal scores, negative
scores only), at the config-2 row length.
"""
import numpy as np
import pytest
import torch

from dsa_triton_ascend_b200 import _host as H
from dsa_triton_ascend_b200 import check_device_errors
from dsa_triton_ascend_b200._lib import LiParams, check, error_flag, lib, ptr, stream_ptr
from dsa_triton_ascend_b200.lightning_indexer import _weights_code

pytestmark = pytest.mark.gpu


def _score_topk(q, k, w, K, mode):
    """dsa_li_score_topk on BSND inputs with a workspace of our own; returns the indices,
    values and the fp32 score rows [B*S1, N2, S2]."""
    B, S1, N1, D = q.shape
    S2, N2 = k.shape[1], k.shape[2]
    dev = q.device
    idx = torch.empty((B, S1, N2, K), dtype=torch.int32, device=dev)
    val = torch.empty((B, S1, N2, K), dtype=q.dtype, device=dev)
    ws_bytes = lib().dsa_li_workspace_size(B * S1, N2, S2)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    act_q = H.lens_tensor(None, B, S1, dev)
    act_k = H.lens_tensor(None, B, S2, dev)
    q_base, k_base = H.row_bases(B, S1, dev), H.row_bases(B, S2, dev)
    p = LiParams()
    p.query, p.key, p.weights = ptr(q), ptr(k), ptr(w)
    p.act_q, p.act_k, p.q_row_base, p.k_row_base = ptr(act_q), ptr(act_k), ptr(q_base), ptr(k_base)
    p.out_indices, p.out_values = ptr(idx), ptr(val)
    p.error_flag = ptr(error_flag(dev))
    p.workspace, p.workspace_bytes = ptr(ws), ws_bytes
    p.q_rows, p.batch, p.n1, p.n2, p.d, p.kv_rows = B * S1, B, N1, N2, D, B * S2
    p.sparse_count, p.s2_row, p.s2_cap = K, S2, S2
    p.q_len_max, p.q_len_dense = S1, S1
    p.sparse_mode = mode
    p.dtype = H.dtype_code(q)
    p.weights_dtype = _weights_code(w)
    check(lib().dsa_li_score_topk(p, stream_ptr(dev)), "dsa_li_score_topk")
    torch.cuda.synchronize()
    check_device_errors()
    scores = ws.view(torch.float32).view(B * S1, N2, S2)
    return idx.view(B * S1, N2, K).cpu().numpy(), val.view(B * S1, N2, K), scores.cpu().numpy()


def _expected(scores, S1, S2, K, mode):
    rows, N2, _ = scores.shape
    ar = np.arange(S2)
    out = np.full((rows, N2, K), -1, np.int32)
    vals = np.zeros((rows, N2, K), np.float32)
    for r in range(rows):
        s1 = r % S1
        lim = min(max(S2 - S1 + s1 + 1, 0), S2) if mode == 3 else S2
        for h in range(N2):
            s = scores[r, h, :lim].astype(np.float64)
            order = np.lexsort((ar[:lim], -s))[:K]
            out[r, h, :len(order)] = order
            vals[r, h, :len(order)] = scores[r, h, order]
    return out, vals


def _check(q, k, w, K, mode):
    idx, val, sc = _score_topk(q, k, w, K, mode)
    S1, S2 = q.shape[1], k.shape[1]
    ref_idx, ref_val = _expected(sc, S1, S2, K, mode)
    for r in range(idx.shape[0]):
        np.testing.assert_array_equal(idx[r], ref_idx[r], err_msg=f"row {r}")
    got = val.float().cpu().numpy()
    exp = torch.from_numpy(ref_val).to(val.dtype).float().numpy()
    valid = ref_idx >= 0
    np.testing.assert_array_equal(got[valid], exp[valid])
    assert np.all(np.isneginf(got[~valid]))


def _inputs(S1, S2, N1, D, seed, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn(1, S1, N1, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(1, S2, 1, D, generator=g, device="cuda").to(dtype)
    w = torch.randn(1, S1, N1, generator=g, device="cuda") / N1 ** 0.5
    return q, k, w


@pytest.mark.parametrize("mode", [0, 3])
def test_topk_exact_spread_scores(mode):
    q, k, w = _inputs(6, 4096, 64, 128, seed=1)
    _check(q, k, w, 2048, mode)


def test_topk_exact_with_ties():
    q, k, w = _inputs(4, 4096, 64, 128, seed=2)
    k[0, 1::2] = k[0, 0::2]           # keys 2j and 2j+1 identical: every score appears twice
    k[0, 3::7] = k[0, 5]              # and one score appears ~600 times
    _check(q, k, w, 2048, 0)


def test_topk_exact_outlier_and_clusters():
    q, k, w = _inputs(4, 4096, 64, 128, seed=3)
    w = w.abs()
    k[0, 100] = 50.0                  # one score far above the rest
    _check(q, k, w, 2048, 0)
    _check(q, k, w, 1000, 3)


def test_topk_exact_equal_and_negative_scores():
    q, k, w = _inputs(3, 4096, 64, 128, seed=4)
    _check(torch.zeros_like(q), k, w, 2048, 0)     # every score 0: index order
    _check(q, k, -w.abs(), 2048, 3)                # scores <= 0


def test_topk_exact_small_k_and_short_rows():
    q, k, w = _inputs(700, 700, 32, 128, seed=5)
    _check(q, k, w, 64, 0)
    _check(q, k, w, 512, 3)                        # causal rows shorter than K: -1 padding
