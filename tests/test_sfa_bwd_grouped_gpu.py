"""K3 row pairs: the shared keys of two adjacent query rows reduced once (GPU).

A 5-output backward call reorders each pair of adjacent rows' compacted key lists into three
runs (keys of row 0 only, keys of both, keys of row 1 only; the shared run in row 0's order
in both rows), and K3 sums the two rows' products for a shared key in TMEM before the one
scatter into the key's fp32 accumulator.  These cases drive every pair layout against the
oracle: identical lists in different orders, disjoint lists, partial overlap, an odd row
count, an inactive row beside an active one, ragged -1 tails and a key listed twice (which
keeps the pair unshared).  Some cases read the reordered lists and the run table back from
the workspace.
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import cuda, icuda, host, assert_close
from oracle import sfa

pytestmark = pytest.mark.gpu

NAMES = ("dq", "dk", "dv", "dqr", "dkr")


def _pattern(name, rng, B, S1, S2, cnt):
    si = np.full((B, S1, 1, cnt), -1, np.int32)
    for b in range(B):
        if name == "identical":      # one set, every row its own order: all keys shared
            base = rng.choice(S2, cnt, replace=False)
            for s in range(S1):
                si[b, s, 0] = rng.permutation(base)
        elif name == "disjoint":     # even rows and odd rows draw from separate halves
            for s in range(S1):
                half = np.arange(S2 // 2) + (S2 // 2) * (s & 1)
                si[b, s, 0] = rng.choice(half, cnt, replace=False)
        elif name in ("overlap", "odd"):   # independent draws from 2 x cnt keys: ~half shared
            for s in range(S1):
                si[b, s, 0] = rng.choice(2 * cnt, cnt, replace=False)
        elif name == "ragged":       # -1 tails of different lengths, partial overlap
            for s in range(S1):
                n = int(rng.integers(1, cnt + 1))
                si[b, s, 0, :n] = rng.choice(2 * cnt, n, replace=False)
        elif name == "duplicate":    # a key listed twice in row 0: that pair stays unshared
            for s in range(S1):
                si[b, s, 0] = rng.choice(2 * cnt, cnt, replace=False)
            si[b, 0, 0, 1] = si[b, 0, 0, 0]
    return si


CASES = [
    # name, B, S1, S2, N1, D, cnt, act_q
    ("identical", 1, 4, 700, 16, 512, 300, None),
    ("disjoint", 1, 4, 1400, 16, 512, 300, None),
    ("overlap", 2, 4, 700, 32, 256, 300, None),
    ("odd", 1, 5, 700, 16, 128, 300, None),
    ("ragged", 1, 6, 700, 16, 512, 300, None),
    ("duplicate", 1, 4, 700, 16, 512, 300, None),
    ("inactive", 1, 4, 700, 16, 512, 300, [3]),
    ("headline", 1, 4, 4096, 128, 512, 2048, None),
]


def _run(name, B, S1, S2, N1, D, cnt, act_q, workspace=None):
    from dsa_triton_ascend_b200 import check_device_errors
    from dsa_triton_ascend_b200.sparse_flash_attention_grad import _sfa_grad, INT64_MAX
    rng = np.random.default_rng(sum(map(ord, name)))
    c = I.sfa_case(B, S1, S2, N1, D, cnt, 1, 0, "bf16", seed=7)
    pat = "overlap" if name in ("inactive", "headline") else name
    c["si"] = _pattern(pat, rng, B, S1, S2, cnt)
    act_k = [S2] * B if act_q is not None else None
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              act_q=act_q, act_k=act_k, sparse_mode=0, dtype="bf16")
    res = _sfa_grad(
        cuda(c["q"]), cuda(c["k"]), cuda(c["k"]), icuda(c["si"]), cuda(c["dout"]), cuda(out),
        cuda(mx, "fp32"), cuda(sm, "fp32"), c["scale"], cuda(c["qr"]), cuda(c["kr"]),
        act_q, act_k, 1, "BSND", 0, INT64_MAX, INT64_MAX, False, defer_cast=False,
        workspace=workspace)
    check_device_errors()
    ref = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["dout"], out, mx, sm,
                      c["scale"], act_q=act_q, act_k=act_k, sparse_mode=0, dtype="bf16",
                      rounding="kernel")
    return c, [host(t) for t in res], ref


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_bwd_row_pairs_match_oracle(case):
    c, got, ref = _run(*case)
    for gi, ri, key in zip(got, ref, NAMES):
        assert_close(gi, ri, what=f"{case[0]} {key}")


def _align256(x):
    return (x + 255) // 256 * 256


@pytest.mark.parametrize("name", ["overlap", "identical", "duplicate", "inactive", "odd"])
def test_row_pair_runs_in_workspace(name):
    """The reordered lists hold each row's keys exactly once in a fixed order (own keys, then
    shared keys, in list order; the shared run in row 0's order in both rows); unshared pairs
    keep their lists and describe them as two runs."""
    from dsa_triton_ascend_b200._lib import lib
    case = {c[0]: c for c in CASES}[name]
    _, B, S1, S2, N1, D, cnt, act_q = case
    rows = B * S1
    ws_bytes = lib().dsa_sfa_bwd_workspace_size(rows, cnt, 1)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    c, got, ref = _run(*case, workspace=ws)
    for gi, ri, key in zip(got, ref, NAMES):
        assert_close(gi, ri, what=f"{name} {key}")
    w = ws.cpu().numpy()
    lists = w[: 4 * rows * cnt].view(np.int32).reshape(rows, cnt)
    npairs = (rows + 1) // 2
    runs_off = ws_bytes - _align256(npairs * 48)
    runs = w[runs_off: runs_off + npairs * 48].view(np.int32).reshape(npairs, 3, 4)
    si = c["si"].reshape(rows, cnt)
    active = np.ones(rows, bool)
    if act_q is not None:
        for b in range(B):
            active[b * S1 + act_q[b]: (b + 1) * S1] = False

    def keys_of(r):   # key-matrix rows the row selects (BSND: batch b's keys start at b*S2)
        if r >= rows or not active[r]:
            return np.zeros(0, np.int64)
        v = si[r][si[r] >= 0].astype(np.int64)
        return v + (r // S1) * S2

    for g in range(npairs):
        r0, r1 = 2 * g, 2 * g + 1
        k0, k1 = keys_of(r0), keys_of(r1)
        (m1, c1, a1, b1), (m3, c3, a3, b3), (m2, c2, a2, b2) = runs[g]
        assert (m1, m3, m2) == (1, 3, 2)
        grouped = len(k0) > 0 and len(k1) > 0 and len(set(k0)) == len(k0) and len(set(k1)) == len(k1)
        if not grouped:
            assert (c1, c3, c2) == (len(k0), 0, len(k1)) and (a1, b1, a2, b2) == (0, 0, 0, 0)
            continue
        shared = set(k0.tolist()) & set(k1.tolist())
        assert (c1, c3, c2) == (len(k0) - len(shared), len(shared), len(k1) - len(shared))
        assert (a3, b3, b2) == (c1, 0, c3)
        # row 0: its own keys, then the shared ones, each in row 0's order; row 1: the shared
        # keys in row 0's order, then its own keys in its own order
        own0 = [k for k in k0 if k not in shared]
        sh0 = [k for k in k0 if k in shared]
        own1 = [k for k in k1 if k not in shared]
        assert lists[r0, : c1 + c3].tolist() == own0 + sh0
        assert lists[r1, : c3 + c2].tolist() == sh0 + own1
