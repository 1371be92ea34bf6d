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
