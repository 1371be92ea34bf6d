"""K3 row groups: the shared keys of adjacent query rows reduced once (GPU).

A 5-output backward call reorders the compacted key lists of adjacent rows into runs, one
per set of member rows (the rows that select the key), every member row listing a run's keys
in the same order, and K3 sums the member rows' products for a key in TMEM before the one
scatter into the key's fp32 accumulator.  Groups of four rows run K3 on CTA pairs (D = 256
or 512, at most 2048 keys a row; groups of two in the merged key == value mode); otherwise
pairs of rows on single CTAs (D = 128, or longer lists).  These cases drive both against the oracle: identical lists in different orders,
disjoint lists, partial overlap, row counts that leave a short last group, an inactive row,
ragged -1 tails, a key listed twice (which keeps its group unshared) and lists too long for
groups of four.  Some cases read the reordered lists and the run records back from the
workspace.
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
    ("six", 1, 6, 700, 16, 256, 300, None),
    ("long", 1, 4, 4400, 16, 512, 2100, None),
]


def _run(name, B, S1, S2, N1, D, cnt, act_q, workspace=None, merged=False):
    from dsa_triton_ascend_b200 import check_device_errors
    from dsa_triton_ascend_b200.sparse_flash_attention_grad import _sfa_grad, INT64_MAX
    rng = np.random.default_rng(sum(map(ord, name)))
    c = I.sfa_case(B, S1, S2, N1, D, cnt, 1, 0, "bf16", seed=7)
    pat = "overlap" if name in ("inactive", "headline", "six", "long") else name
    c["si"] = _pattern(pat, rng, B, S1, S2, cnt)
    act_k = [S2] * B if act_q is not None else None
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              act_q=act_q, act_k=act_k, sparse_mode=0, dtype="bf16")
    res = _sfa_grad(
        cuda(c["q"]), cuda(c["k"]), cuda(c["k"]), icuda(c["si"]), cuda(c["dout"]), cuda(out),
        cuda(mx, "fp32"), cuda(sm, "fp32"), c["scale"], cuda(c["qr"]), cuda(c["kr"]),
        act_q, act_k, 1, "BSND", 0, INT64_MAX, INT64_MAX, False, defer_cast=False,
        workspace=workspace, merged=merged)
    check_device_errors()
    ref = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["dout"], out, mx, sm,
                      c["scale"], act_q=act_q, act_k=act_k, sparse_mode=0, dtype="bf16",
                      rounding="kernel", round_out=not merged)
    if merged:   # dK + dV as one fp32 sum rounded once
        dq, dk, dv, dqr, dkr = ref
        ref = [sfa.round_to(dq, "bf16"), sfa.round_to(dk + dv, "bf16"), sfa.round_to(dqr, "bf16"),
               sfa.round_to(dkr, "bf16")]
    return c, [host(t) for t in res], ref


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_bwd_row_pairs_match_oracle(case):
    c, got, ref = _run(*case)
    for gi, ri, key in zip(got, ref, NAMES):
        assert_close(gi, ri, what=f"{case[0]} {key}")


MERGED = ["overlap", "identical", "duplicate", "inactive", "six", "headline"]


@pytest.mark.parametrize("name", MERGED)
def test_bwd_row_groups_merged_match_oracle(name):
    """key == value: the merged K3 on CTA pairs (groups of two rows) against the oracle's
    dq, dk + dv (one fp32 sum rounded once), dq_rope, dk_rope."""
    case = {c[0]: c for c in CASES}[name]
    c, got, ref = _run(*case, merged=True)
    for gi, ri, key in zip(got, ref, ("dq", "dk + dv", "dqr", "dkr")):
        assert_close(gi, ri, what=f"merged {name} {key}")


def _align256(x):
    return (x + 255) // 256 * 256


WALK4 = [1, 3, 5, 7, 9, 11, 13, 15, 2, 6, 10, 14, 4, 12, 8]


def _expected_runs(lists_in, G):
    """Reference reordering of G rows' key lists: one run per member mask (walking order:
    for four rows the masks holding row 0 first, then row 1, row 2, row 3; for two rows
    1, 3, 2), a run's keys in the order of its lowest member row's list.  Returns the
    rewritten lists and the runs [(mask, length, first slot per row)], or None when a list
    holds a key twice (the group stays unshared)."""
    if any(len(set(l)) != len(l) for l in lists_in):
        return None
    member = {}
    for g, l in enumerate(lists_in):
        for k in l:
            member[k] = member.get(k, 0) | (1 << g)
    walk = WALK4 if G == 4 else [1, 3, 2]
    out = [[] for _ in range(G)]
    runs = []
    for m in walk:
        low = (m & -m).bit_length() - 1
        if low >= G:
            continue
        keys = [k for k in lists_in[low] if member[k] == m]
        if not keys:
            continue
        runs.append((m, len(keys), [len(out[g]) if (m >> g) & 1 else None for g in range(G)]))
        for g in range(G):
            if (m >> g) & 1:
                out[g] += keys
    return out, runs


@pytest.mark.parametrize("name,merged", [(n, False) for n in ["overlap", "identical", "duplicate",
                                                                "inactive", "odd", "six", "long"]]
                         + [("overlap", True), ("inactive", True)])
def test_row_group_runs_in_workspace(name, merged):
    """The reordered lists and the run records equal a plain restatement of the reordering
    (records of four rows for D = 256 / 512 with at most 2048 keys a row, of two rows in the
    merged mode, pair runs otherwise); groups with a key listed twice keep their lists, one
    run per row."""
    from dsa_triton_ascend_b200._lib import lib
    case = {c[0]: c for c in CASES}[name]
    _, B, S1, S2, N1, D, cnt, act_q = case
    rows = B * S1
    ws_bytes = lib().dsa_sfa_bwd_workspace_size(rows, cnt, 1)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    c, got, ref = _run(*case, workspace=ws, merged=merged)
    for gi, ri in zip(got, ref):
        assert_close(gi, ri, what=f"{name}")
    w = ws.cpu().numpy()
    lists = w[: 4 * rows * cnt].view(np.int32).reshape(rows, cnt)
    pair_k3 = D in (256, 512) and cnt <= 2048   # records (CTA-pair K3) or pair runs
    G = (2 if merged else 4) if pair_k3 else 2
    ngroups = (rows + G - 1) // G
    region = _align256((rows + 1) // 2 * 512)
    orig_map = _align256(2 * rows * cnt)   # the teacher's position map follows the records
    tab = w[ws_bytes - orig_map - region: ws_bytes - orig_map].view(np.int32)
    si = c["si"].reshape(rows, cnt)
    active = np.ones(rows, bool)
    if act_q is not None:
        for b in range(B):
            active[b * S1 + act_q[b]: (b + 1) * S1] = False

    def keys_of(r):   # the row's compacted list (BSND: batch b's keys start at b*S2)
        if r >= rows or not active[r]:
            return []
        v = si[r][si[r] >= 0].astype(np.int64)
        return (v + (r // S1) * S2).tolist()

    tiles = lambda n: (n + 127) // 128
    for grp in range(ngroups):
        r0 = G * grp
        ins = [keys_of(r0 + g) for g in range(G)]
        exp = _expected_runs(ins, G)
        if exp is None:   # unshared: lists as compacted, one run per row with keys
            outs = ins
            runs = [(1 << g, len(ins[g]), [0 if h == g else None for h in range(G)])
                    for g in range(G) if ins[g]]
        else:
            outs, runs = exp
        for g in range(G):
            if r0 + g < rows:
                assert lists[r0 + g, : len(outs[g])].tolist() == outs[g], (grp, g)
        if pair_k3:
            rec = tab[grp * 128: (grp + 1) * 128].reshape(32, 4)
            t, last = 0, [-1] * 4
            for i, (m, n, offs) in enumerate(runs):
                ra, rb = rec[2 + 2 * i], rec[3 + 2 * i]
                assert (ra[0], ra[1]) == (m, n), (grp, i)
                got_offs = [ra[2], ra[3], rb[0], rb[1]]
                for g in range(len(offs)):
                    if offs[g] is not None:
                        assert got_offs[g] == offs[g], (grp, i, g)
                t += tiles(n)
                for g in range(4):
                    if (m >> g) & 1:
                        last[g] = t - 1
            assert rec[0].tolist() == [t, last[0], last[1], last[2]], grp
            assert rec[1][:2].tolist() == [last[3], len(runs)], grp
        else:
            rec = tab[grp * 12: (grp + 1) * 12].reshape(3, 4)
            byk = {m: (n, offs) for m, n, offs in runs}
            for j, m in enumerate([1, 3, 2]):
                assert rec[j][0] == m
                n, offs = byk.get(m, (0, [None, None]))
                assert rec[j][1] == n, (grp, m)
                if n:
                    for g in range(2):
                        if offs[g] is not None:
                            assert rec[j][2 + g] == offs[g], (grp, m, g)
