"""SFA backward on the B200 vs the reference goldens and the numpy oracle (GPU)."""
import numpy as np
import pytest

import inputs as I
from gen_golden import SFA_BWD_CASES
from golden_io import load, from_bits16
from gpu_util import cuda, icuda, host, assert_close
from oracle import sfa

pytestmark = pytest.mark.gpu

NAMES = ("dq", "dk", "dv", "dqr", "dkr")


def _bwd(c, out, mx, sm, dt, mode, blk=1, act_q=None, act_k=None):
    from dsa_triton_ascend_b200 import sparse_flash_attention_grad_triton, check_device_errors
    res = sparse_flash_attention_grad_triton(
        cuda(c["q"], dt), cuda(c["k"], dt), cuda(c["k"], dt), icuda(c["si"]),
        cuda(c["dout"], dt), cuda(out, dt), cuda(mx, "fp32"), cuda(sm, "fp32"), c["scale"],
        query_rope=cuda(c["qr"], dt), key_rope=cuda(c["kr"], dt),
        actual_seq_lengths_query=act_q, actual_seq_lengths_kv=act_k, sparse_block_size=blk,
        sparse_mode=mode)
    check_device_errors()
    return [host(t) for t in res]


@pytest.mark.parametrize("case", SFA_BWD_CASES, ids=[c[0] for c in SFA_BWD_CASES])
def test_bwd_matches_golden(case):
    name, B, S1, S2, N1, D, cnt, blk, mode, dt, seed = case
    c = I.sfa_case(B, S1, S2, N1, D, cnt, blk, mode, dt, seed)
    g = load(name)
    out = from_bits16(g["out"], dt)
    got = _bwd(c, out, g["softmax_max"], g["softmax_sum"], dt, mode, blk)
    tok = sfa.expand_block_indices(c["si"], blk)
    ref = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["dout"], out, g["softmax_max"],
                      g["softmax_sum"], c["scale"], sparse_mode=mode, dtype=dt, rounding="kernel")
    for gi, ri, key in zip(got, ref, NAMES):
        assert_close(gi, ri, what=f"{name} {key} vs kernel-rounding oracle")
        # the golden keeps P/dS in fp32: same values up to their bf16 rounding, so the
        # reference test's own band (test_sfa_grad_triton.py:85-93) applies
        assert_close(gi, from_bits16(g[key], dt), rtol=6e-2, atol=5e-2, what=f"{name} {key} vs golden")


def _fwd_stats(c, dt, mode, act_q=None, act_k=None):
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              act_q=act_q, act_k=act_k, sparse_mode=mode, dtype=dt)
    return out, mx, sm


@pytest.mark.parametrize("N1,D,dt", [(128, 512, "bf16"), (64, 256, "fp16"), (16, 128, "bf16"),
                                     (1, 512, "bf16")])
def test_bwd_oracle_heads_dims(N1, D, dt):
    c = I.sfa_case(2, 4, 300, N1, D, 96, 1, 3, dt, seed=200 + N1)
    out, mx, sm = _fwd_stats(c, dt, 3)
    got = _bwd(c, out, mx, sm, dt, 3)
    ref = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["dout"], out, mx, sm,
                      c["scale"], sparse_mode=3, dtype=dt, rounding="kernel")
    for gi, ri, key in zip(got, ref, NAMES):
        assert_close(gi, ri, what=key)


def test_bwd_lengths_scattered_many_tiles():
    """act lengths, empty rows, scattered/duplicate ids, > 2 tiles of keys, mode 0."""
    rng = np.random.default_rng(3)
    act_q, act_k = [6, 3], [700, 500]
    c = I.sfa_case(2, 6, 700, 32, 512, 320, 1, 0, "bf16", seed=31, act_q=act_q, act_k=act_k)
    si = rng.integers(-1, 700, size=c["si"].shape).astype(np.int32)
    si[0, 0, 0, :4] = [5, 5, 5, -1]
    c["si"] = si
    out, mx, sm = _fwd_stats(c, "bf16", 0, act_q, act_k)
    got = _bwd(c, out, mx, sm, "bf16", 0, act_q=act_q, act_k=act_k)
    ref = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], si, c["dout"], out, mx, sm, c["scale"],
                      act_q=act_q, act_k=act_k, sparse_mode=0, rounding="kernel")
    for gi, ri, key in zip(got, ref, NAMES):
        assert_close(gi, ri, what=key)
    assert np.all(got[0][1, 3:] == 0)


def test_bwd_tnd_matches_bsnd():
    from dsa_triton_ascend_b200 import sparse_flash_attention_grad_triton, check_device_errors
    lq, lk = [3, 5], [90, 200]
    c = I.sfa_case(2, 5, 200, 16, 512, 64, 1, 3, "bf16", seed=41, act_q=lq, act_k=lk)
    out, mx, sm = _fwd_stats(c, "bf16", 3, lq, lk)
    cat = lambda x, l: np.concatenate([x[b, :l[b]] for b in range(2)])
    res = sparse_flash_attention_grad_triton(
        cuda(cat(c["q"], lq)), cuda(cat(c["k"], lk)), cuda(cat(c["k"], lk)), icuda(cat(c["si"], lq)),
        cuda(cat(c["dout"], lq)), cuda(cat(out, lq)),
        cuda(np.concatenate([mx[b, 0, :lq[b]] for b in range(2)])[None], "fp32"),
        cuda(np.concatenate([sm[b, 0, :lq[b]] for b in range(2)])[None], "fp32"), c["scale"],
        query_rope=cuda(cat(c["qr"], lq)), key_rope=cuda(cat(c["kr"], lk)),
        actual_seq_lengths_query=list(np.cumsum(lq)), actual_seq_lengths_kv=list(np.cumsum(lk)),
        layout="TND", sparse_mode=3)
    check_device_errors()
    ref = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["dout"], out, mx, sm,
                      c["scale"], act_q=lq, act_k=lk, sparse_mode=3, rounding="kernel")
    for gi, ri, key in zip(res, ref, NAMES):
        lens = lq if key in ("dq", "dqr") else lk
        assert_close(host(gi), cat(ri, lens), what="tnd " + key)


def _bwd_merged(c, out, mx, sm, dt, mode, blk=1):
    from dsa_triton_ascend_b200 import sparse_flash_attention_grad_merged, check_device_errors
    res = sparse_flash_attention_grad_merged(
        cuda(c["q"], dt), cuda(c["k"], dt), icuda(c["si"]), cuda(c["dout"], dt), cuda(out, dt),
        cuda(mx, "fp32"), cuda(sm, "fp32"), c["scale"], query_rope=cuda(c["qr"], dt),
        key_rope=cuda(c["kr"], dt), sparse_block_size=blk, sparse_mode=mode)
    check_device_errors()
    return [host(t) for t in res]


@pytest.mark.parametrize("N1,D,dt,blk", [(128, 512, "bf16", 1), (64, 256, "fp16", 1),
                                         (16, 128, "bf16", 4), (1, 512, "bf16", 1)])
def test_bwd_merged_key_gradient(N1, D, dt, blk):
    """key == value: the merged kernels return dK + dV (one fp32 accumulator) equal to the
    oracle's dk + dv, and the query gradients equal the 5-output call's."""
    c = I.sfa_case(2, 4, 300, N1, D, 96 // blk, blk, 3, dt, seed=300 + N1)
    tok = sfa.expand_block_indices(c["si"], blk)
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["scale"], sparse_mode=3,
                              dtype=dt)
    dq, dkv, dqr, dkr = _bwd_merged(c, out, mx, sm, dt, 3, blk)
    rdq, rdk, rdv, rdqr, rdkr = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["dout"], out,
                                            mx, sm, c["scale"], sparse_mode=3, dtype=dt,
                                            rounding="kernel")
    assert_close(dq, rdq, what="dq")
    assert_close(dqr, rdqr, what="dqr")
    assert_close(dkr, rdkr, what="dkr")
    # the merged gradient is the fp32 sum rounded once (not the sum of two rounded terms)
    _, fdk, fdv, _, _ = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["dout"], out, mx, sm,
                                    c["scale"], sparse_mode=3, dtype=dt, rounding="kernel",
                                    round_out=False)
    assert_close(dkv, sfa.round_to(fdk + fdv, dt), what="dk + dv")
    # the 5-output call reorders the key lists of row pairs (K3's shared-key runs), so its
    # dQ sums the same key terms in another order
    five = _bwd(c, out, mx, sm, dt, 3, blk)
    assert_close(dq, five[0], what="dq vs 5-output call")
    assert_close(dqr, five[3], what="dqr vs 5-output call")


def test_bwd_merged_partial_accumulators_match_separate():
    """The fp32 accumulators of the merged partial call equal dk_acc + dv_acc of the
    separate one (same products, summed in another order), and one buffer holds both."""
    import torch
    from dsa_triton_ascend_b200 import sparse_flash_attention_grad_partial, check_device_errors
    c = I.sfa_case(1, 6, 512, 128, 512, 256, 1, 3, "bf16", seed=41)
    out, mx, sm = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              sparse_mode=3, dtype="bf16")
    args = (cuda(c["q"]), cuda(c["k"]), cuda(c["k"]), icuda(c["si"]), cuda(c["dout"]), cuda(out),
            cuda(mx, "fp32"), cuda(sm, "fp32"), c["scale"])
    kw = dict(query_rope=cuda(c["qr"]), key_rope=cuda(c["kr"]))
    (dk, dkr, dv), fin = sparse_flash_attention_grad_partial(*args, **kw)
    (dkv, dkr2), fin2 = sparse_flash_attention_grad_partial(*args, merge_key_grads=True, **kw)
    torch.cuda.synchronize()
    check_device_errors()
    assert fin2.key_grad_buffer.numel() == dkv.numel() + dkr2.numel()
    ref = (dk + dv).cpu().numpy()
    np.testing.assert_allclose(dkv.cpu().numpy(), ref, rtol=1e-4, atol=1e-5 * np.abs(ref).max())
    np.testing.assert_allclose(dkr2.cpu().numpy(), dkr.cpu().numpy(), rtol=1e-4,
                               atol=1e-5 * np.abs(dkr.cpu().numpy()).max())
    dq, dkv_b, dqr, dkr_b = fin2()
    assert dkv_b.shape == c["k"].shape and dkr_b.shape == c["kr"].shape
