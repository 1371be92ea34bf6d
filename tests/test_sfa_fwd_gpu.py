"""SFA forward on the B200 vs the reference goldens and the numpy oracle (GPU)."""
import numpy as np
import pytest
import torch

import inputs as I
from gen_golden import SFA_FWD_CASES, CONFIG1_ROWS
from golden_io import load, from_bits16
from gpu_util import cuda, icuda, host, assert_close, STAT_RTOL
from oracle import sfa

pytestmark = pytest.mark.gpu


def _run(c, dt, mode, blk=1, act_q=None, act_k=None, lse=True):
    from dsa_triton_ascend_b200 import sparse_flash_attention_triton, check_device_errors
    out, mx, sm = sparse_flash_attention_triton(
        cuda(c["q"], dt), cuda(c["k"], dt), cuda(c["k"], dt), icuda(c["si"]), c["scale"],
        actual_seq_lengths_query=act_q, actual_seq_lengths_kv=act_k,
        query_rope=cuda(c["qr"], dt), key_rope=cuda(c["kr"], dt), sparse_block_size=blk,
        sparse_mode=mode, return_softmax_lse=lse)
    check_device_errors()
    return host(out), host(mx), host(sm)


def _stats_close(got_m, ref_m, got_s, ref_s, what):
    assert_close(got_m, ref_m, rtol=STAT_RTOL, atol=1e-5, what=what + " softmax_max")
    assert_close(got_s, ref_s, rtol=STAT_RTOL, atol=1e-5, what=what + " softmax_sum")


@pytest.mark.parametrize("case", SFA_FWD_CASES, ids=[c[0] for c in SFA_FWD_CASES])
def test_fwd_matches_golden(case):
    name, B, S1, S2, N1, D, cnt, blk, mode, dt, seed = case
    c = I.sfa_case(B, S1, S2, N1, D, cnt, blk, mode, dt, seed)
    g = load(name)
    out, mx, sm = _run(c, dt, mode, blk)
    assert_close(out, from_bits16(g["out"], dt), what=name + " out")
    _stats_close(mx, g["softmax_max"], sm, g["softmax_sum"], name)


def test_fwd_config1_golden_and_oracle():
    c = I.config1()
    g = load("config1")
    out, mx, sm = _run(c, "bf16", 3)
    assert_close(out[:, CONFIG1_ROWS], from_bits16(g["out_rows"], "bf16"), what="config1 out")
    _stats_close(mx, g["softmax_max"], sm, g["softmax_sum"], "config1")
    ref, _, _ = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"], sparse_mode=3,
                            rounding="kernel")
    assert_close(out, ref, what="config1 out vs oracle")


@pytest.mark.parametrize("D,dt", [(512, "bf16"), (256, "fp16"), (128, "bf16")])
@pytest.mark.parametrize("N1", [1, 16, 64, 128])
def test_fwd_oracle_heads_dims(D, dt, N1):
    c = I.sfa_case(2, 5, 300, N1, D, 96, 1, 3, dt, seed=100 + N1 + D)
    out, mx, sm = _run(c, dt, 3)
    ref, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"], sparse_mode=3,
                              dtype=dt, rounding="kernel")
    assert_close(out, ref, what="out")
    _stats_close(mx, rm, sm, rs, "stats")


def test_fwd_actual_lengths_and_empty_rows():
    """act_q < S1 (inactive rows -> zeros), act_k < S2, mode 3 with act_q > act_k."""
    B, S1, S2, N1, D = 3, 12, 200, 16, 512
    act_q, act_k = [12, 7, 9], [200, 150, 5]
    c = I.sfa_case(B, S1, S2, N1, D, 64, 1, 3, "bf16", seed=7, act_q=act_q, act_k=act_k)
    out, mx, sm = _run(c, "bf16", 3, act_q=act_q, act_k=act_k)
    ref, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              act_q=act_q, act_k=act_k, sparse_mode=3, rounding="kernel")
    assert_close(out, ref, what="out")
    _stats_close(mx, rm, sm, rs, "stats")
    assert np.all(out[1, 7:] == 0) and np.all(mx[1, 0, 7:] == 0)


def test_fwd_unsorted_scattered_and_duplicate_indices():
    """Valid ids anywhere in the row (not front packed), -1 holes, duplicates, ids past
    the causal threshold: each entry is masked on its own (reference kernel rule)."""
    rng = np.random.default_rng(5)
    c = I.sfa_case(1, 6, 256, 32, 512, 80, 1, 3, "bf16", seed=9)
    si = rng.integers(-1, 256, size=c["si"].shape).astype(np.int32)
    si[0, 0, 0, :5] = [0, 0, 0, -1, 3]
    c["si"] = si
    out, mx, sm = _run(c, "bf16", 3)
    ref, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], si, c["scale"], sparse_mode=3,
                              rounding="kernel")
    assert_close(out, ref, what="out")
    _stats_close(mx, rm, sm, rs, "stats")


def test_fwd_mode0_blockwise_many_tiles():
    c = I.sfa_case(1, 4, 4096, 64, 512, 256, 8, 0, "bf16", seed=11)
    out, mx, sm = _run(c, "bf16", 0, blk=8)
    tok = sfa.expand_block_indices(c["si"], 8)
    ref, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], tok, c["scale"], sparse_mode=0,
                              rounding="kernel")
    assert_close(out, ref, what="out")
    _stats_close(mx, rm, sm, rs, "stats")


def test_fwd_tnd_layout():
    from dsa_triton_ascend_b200 import sparse_flash_attention_triton, check_device_errors
    lens_q, lens_k = [3, 5], [100, 180]
    c = I.sfa_case(2, 5, 180, 16, 512, 64, 1, 3, "bf16", seed=13, act_q=lens_q, act_k=lens_k)
    q_t = np.concatenate([c["q"][b, :lens_q[b]] for b in range(2)])
    qr_t = np.concatenate([c["qr"][b, :lens_q[b]] for b in range(2)])
    si_t = np.concatenate([c["si"][b, :lens_q[b]] for b in range(2)])
    k_t = np.concatenate([c["k"][b, :lens_k[b]] for b in range(2)])
    kr_t = np.concatenate([c["kr"][b, :lens_k[b]] for b in range(2)])
    out, mx, sm = sparse_flash_attention_triton(
        cuda(q_t), cuda(k_t), cuda(k_t), icuda(si_t), c["scale"],
        actual_seq_lengths_query=list(np.cumsum(lens_q)), actual_seq_lengths_kv=list(np.cumsum(lens_k)),
        query_rope=cuda(qr_t), key_rope=cuda(kr_t), layout_query="TND", layout_kv="TND",
        sparse_mode=3, return_softmax_lse=True)
    check_device_errors()
    ref, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"],
                              act_q=lens_q, act_k=lens_k, sparse_mode=3, rounding="kernel")
    ref_t = np.concatenate([ref[b, :lens_q[b]] for b in range(2)])
    assert out.shape == (8, 16, 512) and mx.shape == (1, 8, 16)
    assert_close(host(out), ref_t, what="tnd out")
    rm_t = np.concatenate([rm[b, 0, :lens_q[b]] for b in range(2)])[None]
    rs_t = np.concatenate([rs[b, 0, :lens_q[b]] for b in range(2)])[None]
    _stats_close(host(mx), rm_t, host(sm), rs_t, "tnd")


def test_fwd_split_rows_match_oracle():
    """Few query rows with many keys: each row's keys are split over several CTA pairs whose
    fp32 partials are merged by a second kernel. Batch 1 sees at most 100 keys (most of its
    splits are empty) and its last row is past actual_seq_lengths_query (all splits empty)."""
    act_q, act_k = [3, 2], [4096, 100]
    c = I.sfa_case(2, 3, 4096, 128, 512, 2048, 1, 3, "bf16", seed=31, act_q=act_q, act_k=act_k)
    out, mx, sm = _run(c, "bf16", 3, act_q=act_q, act_k=act_k)
    ref, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"], act_q=act_q,
                              act_k=act_k, sparse_mode=3, rounding="kernel")
    assert_close(out, ref, what="split out")
    _stats_close(mx, rm, sm, rs, "split")
    assert np.all(out[1, 2] == 0) and np.all(mx[1, 0, 2] == 0) and np.all(sm[1, 0, 2] == 0)


@pytest.mark.parametrize("S1,N1", [(80, 16), (4, 128)], ids=["one_pair_per_row", "split_rows"])
def test_fwd_running_max_rescale(S1, N1):
    """Later key tiles score far above the first ones (the rope part of keys past position
    600 scaled by 20, ids sorted ascending), so the running max grows by more than the
    lazy-rescale threshold and O and the row sum move onto a new exponent reference mid-row.
    80 rows run one CTA pair per row; 4 rows are split over several pairs whose partials are
    merged.

    The softmax is then so peaked that bf16 rounding of the unnormalised probabilities
    (relative error <= 2^-8 each, whatever exponent reference they are taken against)
    dominates the output error, so the output is checked against an exact float64 softmax
    with the bound that rounding allows: |O - O_exact| <= 2^-7 (sum_i p_i |v_i| / l +
    |O_exact|) + 1e-3 (P rounding, the bf16 output, a factor 2 of margin). The statistics
    are fp32 quantities and keep the oracle's tolerance."""
    c = I.sfa_case(1, S1, 2048, N1, 512, 1024, 1, 0, "bf16", seed=41)
    c["kr"][:, 600:] = I.cast(c["kr"][:, 600:] * 20.0, "bf16")
    out, mx, sm = _run(c, "bf16", 0)
    _, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"], sparse_mode=0,
                            rounding="kernel")
    _stats_close(mx, rm, sm, rs, "rescale")
    for s1 in range(S1):
        pos = c["si"][0, s1, 0]
        pos = pos[pos >= 0]
        kk = np.concatenate([c["k"][0, pos, 0], c["kr"][0, pos, 0]], 1).astype(np.float64)
        qf = np.concatenate([c["q"][0, s1], c["qr"][0, s1]], 1).astype(np.float64)
        sc = qf @ kk.T * c["scale"]
        p = np.exp(sc - sc.max(1, keepdims=True))
        l = p.sum(1, keepdims=True)
        v = kk[:, :512]
        exact, mag = (p @ v) / l, (p @ np.abs(v)) / l
        err = np.abs(out[0, s1].astype(np.float64) - exact)
        bound = 2.0 ** -7 * (mag + np.abs(exact)) + 1e-3
        assert np.all(err <= bound), f"row {s1}: worst excess {float((err - bound).max()):.3g}"


def test_fwd_paged_decode_split():
    """Decode-shaped PA_BSND call (one query token per sequence, 2048 keys each): split."""
    from dsa_triton_ascend_b200 import sparse_flash_attention_triton, check_device_errors
    rng = np.random.default_rng(23)
    B, N1, D, page, nblk, maxb = 3, 128, 512, 128, 80, 24
    kv_len = [3000, 2048, 2500]
    cache = I.randn(rng, (nblk, page, 1, D), "bf16")
    cache_r = I.randn(rng, (nblk, page, 1, 64), "bf16")
    bt = rng.permutation(nblk)[:B * maxb].reshape(B, maxb).astype(np.int32)
    q = I.randn(rng, (B, 1, N1, D), "bf16")
    qr = I.randn(rng, (B, 1, N1, 64), "bf16")
    si = np.stack([np.sort(rng.permutation(kv_len[b])[:2048]) for b in range(B)]).astype(np.int32)
    si = si.reshape(B, 1, 1, 2048)
    scale = 1 / np.sqrt(576)
    out, mx, sm = sparse_flash_attention_triton(
        cuda(q), cuda(cache), cuda(cache), icuda(si), scale, block_table=icuda(bt),
        actual_seq_lengths_kv=kv_len, query_rope=cuda(qr), key_rope=cuda(cache_r),
        layout_kv="PA_BSND", sparse_mode=0, return_softmax_lse=True, block_size=page)
    check_device_errors()
    k_dense = sfa.pa_to_bsnd(cache, bt, maxb * page)
    kr_dense = sfa.pa_to_bsnd(cache_r, bt, maxb * page)
    ref, rm, rs = sfa.sfa_fwd(q, k_dense, qr, kr_dense, si, scale, act_k=kv_len, sparse_mode=0,
                              rounding="kernel")
    assert_close(host(out), ref, what="pa split out")
    _stats_close(host(mx), rm, host(sm), rs, "pa split")


def test_fwd_paged_kv():
    """PA_BSND: cache blocks addressed through block_table inside the kernel."""
    from dsa_triton_ascend_b200 import sparse_flash_attention_triton, check_device_errors
    rng = np.random.default_rng(17)
    B, N1, D, page, nblk, maxb = 3, 128, 512, 128, 40, 8
    kv_len = [900, 1024, 300]
    cache = I.randn(rng, (nblk, page, 1, D), "bf16")
    cache_r = I.randn(rng, (nblk, page, 1, 64), "bf16")
    bt = rng.permutation(nblk)[:B * maxb].reshape(B, maxb).astype(np.int32)
    q = I.randn(rng, (B, 1, N1, D), "bf16")
    qr = I.randn(rng, (B, 1, N1, 64), "bf16")
    si = np.full((B, 1, 1, 256), -1, np.int32)
    for b in range(B):
        n = min(256, kv_len[b])
        si[b, 0, 0, :n] = np.sort(rng.permutation(kv_len[b])[:n])
    scale = 1 / np.sqrt(576)
    out, mx, sm = sparse_flash_attention_triton(
        cuda(q), cuda(cache), cuda(cache), icuda(si), scale, block_table=icuda(bt),
        actual_seq_lengths_kv=kv_len, query_rope=cuda(qr), key_rope=cuda(cache_r),
        layout_kv="PA_BSND", sparse_mode=0, return_softmax_lse=True, block_size=page)
    check_device_errors()
    k_dense = sfa.pa_to_bsnd(cache, bt, maxb * page)
    kr_dense = sfa.pa_to_bsnd(cache_r, bt, maxb * page)
    ref, rm, rs = sfa.sfa_fwd(q, k_dense, qr, kr_dense, si, scale, act_k=kv_len, sparse_mode=0,
                              rounding="kernel")
    assert_close(host(out), ref, what="pa out")
    _stats_close(host(mx), rm, host(sm), rs, "pa")
