"""Parity of the BASELINE geometries themselves against the numpy oracle (GPU).

The other GPU tests compare small shapes with the oracle; here the kernels run at the exact
sizes the benchmark measures, and the oracle recomputes what it can in seconds:

* config 4 (B=1, S1=S2=8192, N1=128, D=512+64, top-2048 causal ids, sparse_mode 3): the
  whole forward and backward run on the GPU; the oracle (rounding="kernel") recomputes
  out / softmax_max / softmax_sum and dQ / dQr of 16 query rows spread over the causal head
  (fewer than 2048 keys) and the full rows.  Query rows are independent in both directions,
  so a sampled row's results depend on that row only.
* the key gradients of the same geometry (N1=128, 2048 keys per row, more query rows than
  the GPU runs CTA pairs at once) in full: S1=96 rows at the end of S2=4096.
* config 3 at its real shape (PA_BSND, B=32, 16,384-block pool, kv_len 8k-64k, top-2048):
  every row, with the indexed keys de-paged on the host.
* config 5 (S1=S2=8192, N1=128, Nidx1=64, top-2048): dQueryIndex and dWeights of sampled
  rows against the fp32 oracle, with the softmax statistics of config 4's forward.
"""
import math

import numpy as np
import pytest
import torch

from gpu_util import OUT_ATOL, OUT_RTOL, STAT_RTOL, assert_close, host
from oracle import sfa, sli

pytestmark = pytest.mark.gpu

S = 8192
ROWS = [0, 1, 7, 100, 1023, 2046, 2047, 2048, 3000, 4095, 5000, 6143, 7000, 8000, 8190, 8191]


@pytest.fixture(scope="module")
def cfg4():
    from dsa_triton_ascend_b200.synthetic import sfa_prefill
    return sfa_prefill(S1=S, S2=S, device="cuda", seed=17)


def _np(t):
    return t.detach().float().cpu().numpy()


def test_config4_forward_and_query_grads_sampled_rows(cfg4):
    import dsa_triton_ascend_b200 as dsa
    w = cfg4
    out, mx, sm = dsa.sparse_flash_attention_triton(
        w["q"], w["k"], w["k"], w["si"], w["scale"], query_rope=w["qr"], key_rope=w["kr"],
        sparse_mode=3, return_softmax_lse=True)
    dq, dk, dv, dqr, dkr = dsa.sparse_flash_attention_grad_triton(
        w["q"], w["k"], w["k"], w["si"], w["dout"], out, mx, sm, w["scale"],
        query_rope=w["qr"], key_rope=w["kr"], sparse_mode=3)
    dsa.check_device_errors()
    rows = torch.tensor(ROWS, device="cuda")
    pick = lambda t: _np(t[:, rows])
    q, qr, do = pick(w["q"]), pick(w["qr"]), pick(w["dout"])
    si = w["si"][:, rows].cpu().numpy()
    k, kr = _np(w["k"]), _np(w["kr"])
    # the sampled rows' ids are causal and -1 padded, so sparse_mode 0 over the same lists
    # keeps exactly the keys sparse_mode 3 keeps at the rows' original positions
    n_valid = (si >= 0).sum(-1).ravel()
    assert n_valid.min() == 1 and n_valid.max() == 2048
    ro, rm, rs = sfa.sfa_fwd(q, k, qr, kr, si, w["scale"], sparse_mode=0, rounding="kernel")
    assert_close(pick(out), ro, what="config4 out")
    assert_close(_np(mx[:, :, rows]), rm, rtol=STAT_RTOL, atol=1e-5, what="config4 softmax_max")
    assert_close(_np(sm[:, :, rows]), rs, rtol=STAT_RTOL, atol=1e-5, what="config4 softmax_sum")
    # the backward consumes the GPU forward's outputs, as the reference's bprop does
    rdq, _, _, rdqr, _ = sfa.sfa_bwd(q, k, qr, kr, si, do, pick(out), _np(mx[:, :, rows]),
                                     _np(sm[:, :, rows]), w["scale"], sparse_mode=0,
                                     rounding="kernel")
    assert_close(pick(dq), rdq, what="config4 dq")
    assert_close(pick(dqr), rdqr, what="config4 dq_rope")
    for t, n in ((dk, "dk"), (dv, "dv"), (dkr, "dkr")):
        assert torch.isfinite(t.float()).all() and float(t.float().abs().mean()) > 0, n


def test_config4_geometry_key_gradients_in_full():
    """N1=128 with 2048 keys per row and 96 rows (one CTA pair per row, 32 key tiles per
    pair, as at config 4): every output and all key gradients against the oracle."""
    import dsa_triton_ascend_b200 as dsa
    from dsa_triton_ascend_b200.synthetic import sfa_prefill
    w = sfa_prefill(S1=96, S2=4096, device="cuda", seed=23)
    out, mx, sm = dsa.sparse_flash_attention_triton(
        w["q"], w["k"], w["k"], w["si"], w["scale"], query_rope=w["qr"], key_rope=w["kr"],
        sparse_mode=3, return_softmax_lse=True)
    grads = dsa.sparse_flash_attention_grad_triton(
        w["q"], w["k"], w["k"], w["si"], w["dout"], out, mx, sm, w["scale"],
        query_rope=w["qr"], key_rope=w["kr"], sparse_mode=3)
    dsa.check_device_errors()
    q, qr, k, kr, do = (_np(w[n]) for n in ("q", "qr", "k", "kr", "dout"))
    si = w["si"].cpu().numpy()
    assert int((si >= 0).sum(-1).min()) == 2048
    ro, rm, rs = sfa.sfa_fwd(q, k, qr, kr, si, w["scale"], sparse_mode=3, rounding="kernel")
    assert_close(_np(out), ro, what="out")
    assert_close(_np(mx), rm, rtol=STAT_RTOL, atol=1e-5, what="softmax_max")
    assert_close(_np(sm), rs, rtol=STAT_RTOL, atol=1e-5, what="softmax_sum")
    ref = sfa.sfa_bwd(q, k, qr, kr, si, do, _np(out), _np(mx), _np(sm), w["scale"],
                      sparse_mode=3, rounding="kernel")
    for g, r, n in zip(grads, ref, ("dq", "dk", "dv", "dq_rope", "dk_rope")):
        assert_close(_np(g), r, what=n)
    # key == value: the merged kernels' dK + dV at the same geometry
    mdq, mdkv, mdqr, mdkr = dsa.sparse_flash_attention_grad_merged(
        w["q"], w["k"], w["si"], w["dout"], out, mx, sm, w["scale"], query_rope=w["qr"],
        key_rope=w["kr"], sparse_mode=3)
    dsa.check_device_errors()
    _, fdk, fdv, _, _ = sfa.sfa_bwd(q, k, qr, kr, si, do, _np(out), _np(mx), _np(sm), w["scale"],
                                    sparse_mode=3, rounding="kernel", round_out=False)
    assert_close(_np(mdkv), sfa.round_to(fdk + fdv, "bf16"), what="dk + dv")
    assert_close(_np(mdkr), ref[4], what="dk_rope (merged call)")
    # the 5-output call reorders row pairs' key lists (K3's shared-key runs): dQ sums the same
    # key terms in another order
    assert_close(_np(mdq), _np(grads[0]), what="dq (merged call vs 5-output call)")


def test_config3_decode_real_shape_all_rows():
    import dsa_triton_ascend_b200 as dsa
    from dsa_triton_ascend_b200.synthetic import sfa_decode
    w = sfa_decode(seed=29)
    out, mx, sm = dsa.sparse_flash_attention_triton(
        w["q"], w["cache"], w["cache"], w["si"], w["scale"], block_table=w["block_table"],
        actual_seq_lengths_kv=w["lens"], query_rope=w["qr"], key_rope=w["cache_r"],
        layout_kv="PA_BSND", sparse_mode=0, return_softmax_lse=True, block_size=w["page"])
    dsa.check_device_errors()
    B, page = w["q"].shape[0], w["page"]
    tok = w["si"].reshape(B, -1).long()                                  # [B, 2048] token ids
    assert int(tok.min()) >= 0 and bool((tok < torch.tensor(w["lens"], device="cuda")[:, None]).all())
    pool_row = w["block_table"].long().gather(1, tok // page) * page + tok % page
    kg = w["cache"].reshape(-1, w["cache"].shape[-1])[pool_row]          # [B, 2048, 512]
    krg = w["cache_r"].reshape(-1, 64)[pool_row]
    K = tok.shape[1]
    ids = np.broadcast_to(np.arange(K, dtype=np.int32), (B, 1, 1, K)).copy()
    ro, rm, rs = sfa.sfa_fwd(_np(w["q"]), _np(kg)[:, :, None], _np(w["qr"]), _np(krg)[:, :, None],
                             ids, w["scale"], sparse_mode=0, rounding="kernel")
    assert_close(_np(out), ro, what="config3 out")
    assert_close(_np(mx), rm, rtol=STAT_RTOL, atol=1e-5, what="config3 softmax_max")
    assert_close(_np(sm), rs, rtol=STAT_RTOL, atol=1e-5, what="config3 softmax_sum")


def test_config5_sli_sampled_rows():
    import dsa_triton_ascend_b200 as dsa
    from dsa_triton_ascend_b200.synthetic import sli_prefill
    w = sli_prefill(seed=31)
    _, mx, sm = dsa.sparse_flash_attention_triton(
        w["q"], w["k"], w["k"], w["si"], w["scale"], query_rope=w["qr"], key_rope=w["kr"],
        sparse_mode=3, return_softmax_lse=True)
    dqi, dki, dw, loss = dsa.sparse_lightning_indexer_grad_kl_loss_triton(
        w["q"], w["k"], w["qi"], w["ki"], w["w"], w["si"], mx, sm, query_rope=w["qr"],
        key_rope=w["kr"], scale_value=w["scale"])
    dsa.check_device_errors()
    assert torch.isfinite(loss).all() and float(loss) > 0
    k, kr, ki = _np(w["k"]), _np(w["kr"]), _np(w["ki"])
    for s1 in (0, 5, 1500, 2047, 4096, 8191):
        one = lambda t: _np(t[:, s1:s1 + 1])
        # a one-row query at position s1: act_k = s1 + 1 gives the row's window
        # min(topK, act_k - act_q + 0 + 1) = min(topK, s1 + 1)
        ref = sli.sli_grad(one(w["q"]), k, one(w["qr"]), kr, one(w["qi"]), ki, one(w["w"]),
                           w["si"][:, s1:s1 + 1].cpu().numpy(), _np(mx[:, :, s1:s1 + 1]),
                           _np(sm[:, :, s1:s1 + 1]), w["scale"], act_q=[1], act_k=[s1 + 1])
        assert_close(one(dqi), ref["dQueryIndex"], what=f"config5 row {s1} dQueryIndex")
        assert_close(one(dw), ref["dWeights"], what=f"config5 row {s1} dWeights")
