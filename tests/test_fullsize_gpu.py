"""Config-4 geometry at full size (B=1, S1=S2=8192, N1=128, D=512+64, top-2048 causal ids)
through size-independent properties (GPU). The oracle cannot run this size in seconds, so:

* query rows are independent: a contiguous causal row range [r0, r1) passed as its own query
  (actual length S1 - r0) gives bit-identical outputs, statistics and dQ / dQr rows;
* key gradients are linear in the rows: the fp32 key-gradient accumulators of row shards
  added into one set equal the full call's (up to fp32 summation order, as with the
  reference's atomics).
"""
import pytest
import torch

from gpu_util import OUT_ATOL, OUT_RTOL

pytestmark = pytest.mark.gpu

S = 8192


@pytest.fixture(scope="module")
def cfg4():
    from dsa_triton_ascend_b200.synthetic import sfa_prefill
    return sfa_prefill(S1=S, S2=S, device="cuda", seed=5)


def _rows(w, r0, r1):
    cut = lambda t: t[:, r0:r1].contiguous()
    return cut(w["q"]), cut(w["qr"]), cut(w["si"]), cut(w["dout"])


def _fwd(w, r0, r1):
    import dsa_triton_ascend_b200 as dsa
    q, qr, si, _ = _rows(w, r0, r1)
    return dsa.sparse_flash_attention_triton(
        q, w["k"], w["k"], si, w["scale"], actual_seq_lengths_query=[S - r0], query_rope=qr,
        key_rope=w["kr"], sparse_mode=3, return_softmax_lse=True)


def test_fullsize_forward_rows_are_independent(cfg4):
    import dsa_triton_ascend_b200 as dsa
    out, mx, sm = _fwd(cfg4, 0, S)
    dsa.check_device_errors()
    assert torch.isfinite(out.float()).all() and float(out.float().abs().mean()) > 0
    for r0, r1 in [(0, 1000), (1000, 5000), (5000, S)]:
        o, m, s = _fwd(cfg4, r0, r1)
        dsa.check_device_errors()
        assert torch.equal(o, out[:, r0:r1]), (r0, r1)
        assert torch.equal(m, mx[:, :, r0:r1]), (r0, r1)
        assert torch.equal(s, sm[:, :, r0:r1]), (r0, r1)


def test_fullsize_backward_rows_and_key_gradient_linearity(cfg4):
    import dsa_triton_ascend_b200 as dsa
    w = cfg4
    out, mx, sm = _fwd(w, 0, S)
    full = dsa.sparse_flash_attention_grad_triton(
        w["q"], w["k"], w["k"], w["si"], w["dout"], out, mx, sm, w["scale"],
        query_rope=w["qr"], key_rope=w["kr"], sparse_mode=3)
    dsa.check_device_errors()
    accs, finish, dq_parts = None, None, []
    for r0, r1 in [(0, 3000), (3000, S)]:
        q, qr, si, do = _rows(w, r0, r1)
        cut = lambda t: t[:, :, r0:r1].contiguous()
        accs, finish = dsa.sparse_flash_attention_grad_partial(
            q, w["k"], w["k"], si, do, out[:, r0:r1].contiguous(), cut(mx), cut(sm), w["scale"],
            query_rope=qr, key_rope=w["kr"], actual_seq_lengths_query=[S - r0], sparse_mode=3,
            accumulators=accs)
        dq_parts.append((r0, r1) + tuple(t.clone() for t in finish.query_grads))
    dq, dk, dv, dqr, dkr = finish()
    dsa.check_device_errors()
    for r0, r1, dq_s, dqr_s in dq_parts:
        assert torch.equal(dq_s, full[0][:, r0:r1]), (r0, r1)
        assert torch.equal(dqr_s, full[3][:, r0:r1]), (r0, r1)
    for got, ref, name in ((dk, full[1], "dk"), (dv, full[2], "dv"), (dkr, full[4], "dkr")):
        assert float(ref.float().abs().mean()) > 0, name
        torch.testing.assert_close(got.float(), ref.float(), rtol=OUT_RTOL, atol=OUT_ATOL,
                                   msg=lambda m, n=name: f"{n}: {m}")


# ---- lightning indexer, config 2 (B=2, S1=S2=4096, N1=64, D=128, top-2048, mode 3) ----

@pytest.fixture(scope="module")
def cfg2():
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    B, S2, N1, D = 2, 4096, 64, 128
    q = torch.randn(B, S2, N1, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, S2, 1, D, generator=g, device="cuda").bfloat16()
    w = torch.randn(B, S2, N1, generator=g, device="cuda") / 8
    return q, k, w


def _li(q, k, w, r0, r1, S1):
    import dsa_triton_ascend_b200 as dsa
    B = q.shape[0]
    return dsa.lightning_indexer_triton(
        q[:, r0:r1].contiguous(), k, w[:, r0:r1].contiguous(),
        actual_seq_lengths_query=[S1 - r0] * B, sparse_count=2048, sparse_mode=3,
        return_value=True)


def test_fullsize_indexer_rows_and_sampled_scores(cfg2):
    """Row shards are bit-identical to the full call; on 24 sampled rows the top-k agrees
    with fp32 scores computed by torch (ties within 1e-5 of the k-th score excepted)."""
    import numpy as np
    import dsa_triton_ascend_b200 as dsa
    from test_li_gpu import check_topk
    q, k, w = cfg2
    B, S1, N1, D = q.shape
    idx, val = _li(q, k, w, 0, S1, S1)
    dsa.check_device_errors()
    for r0, r1 in [(0, 1500), (1500, S1)]:
        i2, v2 = _li(q, k, w, r0, r1, S1)
        assert torch.equal(i2, idx[:, r0:r1]) and torch.equal(v2, val[:, r0:r1]), (r0, r1)
    rows = np.linspace(0, S1 - 1, 12).astype(int)
    for b in range(B):
        qs = q[b, rows].float()                                   # [R, N1, D]
        sc = torch.einsum("rgd,sd->rgs", qs, k[b, :, 0].float()).relu()
        sc = (sc * w[b, rows].float()[:, :, None]).sum(1)         # [R, S2]
        vis = torch.arange(S1, device="cuda")[None, :] <= torch.as_tensor(rows, device="cuda")[:, None]
        sc = torch.where(vis, sc, torch.full_like(sc, -float("inf")))
        check_topk(idx[b, rows].cpu().numpy(), val[b, rows].float().cpu().numpy(),
                   sc.double().cpu().numpy(), 2048, what=f"cfg2 b{b}")


# ---- SLI KL-loss gradient, config 5 (S1=S2=8192, N1=128, Nidx1=64, top-2048) ----

def test_fullsize_sli_rows_and_linearity(cfg4):
    """dQueryIndex and dWeights rows of row shards equal the full call's bit for bit; the loss
    and dKeyIndex of the shards add up to the full call's."""
    import dsa_triton_ascend_b200 as dsa
    w4 = cfg4
    g = torch.Generator(device="cuda")
    g.manual_seed(8)
    qi = torch.randn(1, S, 64, 128, generator=g, device="cuda").bfloat16()
    ki = torch.randn(1, S, 1, 128, generator=g, device="cuda").bfloat16()
    wt = torch.randn(1, S, 64, generator=g, device="cuda") / 8
    _, mx, sm = _fwd(w4, 0, S)

    def sli(r0, r1):
        cut = lambda t: t[:, r0:r1].contiguous()
        return dsa.sparse_lightning_indexer_grad_kl_loss_triton(
            cut(w4["q"]), w4["k"], cut(qi), ki, cut(wt), cut(w4["si"]),
            mx[:, :, r0:r1].contiguous(), sm[:, :, r0:r1].contiguous(), query_rope=cut(w4["qr"]),
            key_rope=w4["kr"], actual_seq_qlen=[S - r0], scale_value=w4["scale"])

    dqi, dki, dw, loss = sli(0, S)
    dsa.check_device_errors()
    assert torch.isfinite(loss).all() and float(loss) > 0
    parts = [(r0, r1) + tuple(t.clone() for t in sli(r0, r1)) for r0, r1 in [(0, 3000), (3000, S)]]
    dsa.check_device_errors()
    for r0, r1, dqi_s, _, dw_s, _ in parts:
        assert torch.equal(dqi_s, dqi[:, r0:r1]), (r0, r1)
        assert torch.equal(dw_s, dw[:, r0:r1]), (r0, r1)
    torch.testing.assert_close(sum(p[5] for p in parts), loss, rtol=1e-4, atol=1e-6)
    # each call returns dKeyIndex rounded to bf16 (half an ulp: 2^-8 of the value), so the sum
    # of the shards' results may differ from the full call's by 2^-8 (|A| + |B| + |A + B|)
    a, b = (p[3].float() for p in parts)
    bound = 2.0 ** -7 * (a.abs() + b.abs()) + OUT_ATOL
    err = ((a + b) - dki.float()).abs()
    assert bool((err <= bound).all()), f"dKeyIndex: worst excess {float((err - bound).max()):.3g}"
