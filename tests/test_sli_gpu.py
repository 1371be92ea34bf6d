"""Sparse lightning-indexer KL-loss gradient on the B200 vs goldens and the oracle (GPU)."""
import numpy as np
import pytest
import torch

import inputs as I
from gen_golden import SLI_CASES
from golden_io import load
from gpu_util import cuda, icuda, host, assert_close
from oracle import sli

pytestmark = pytest.mark.gpu


def _run(c, mx, sm, dt, act_q=None, act_k=None, w_dtype=None):
    from dsa_triton_ascend_b200 import (sparse_lightning_indexer_grad_kl_loss_triton,
                                        check_device_errors)
    w = cuda(c["w"], w_dtype or dt)
    res = sparse_lightning_indexer_grad_kl_loss_triton(
        cuda(c["q"], dt), cuda(c["k"], dt), cuda(c["qi"], dt), cuda(c["ki"], dt), w,
        icuda(c["si"]), cuda(mx, "fp32"), cuda(sm, "fp32"), query_rope=cuda(c["qr"], dt),
        key_rope=cuda(c["kr"], dt), actual_seq_qlen=act_q, actual_seq_klen=act_k,
        scale_value=c["scale"])
    check_device_errors()
    return [host(t) for t in res]


def _check(got, ref, what, loss_rtol=1e-4):
    dqi, dki, dw, loss = got
    assert_close(dqi, ref["dQueryIndex"], what=what + " dQueryIndex")
    assert_close(dki, ref["dKeyIndex"], what=what + " dKeyIndex")
    assert_close(dw, ref["dWeights"], what=what + " dWeights")
    np.testing.assert_allclose(loss, ref["loss"], rtol=loss_rtol, atol=1e-6, err_msg=what + " loss")


@pytest.mark.parametrize("case", SLI_CASES, ids=[c[0] for c in SLI_CASES])
def test_sli_matches_golden(case):
    name, B, S1, S2, N1, D, Nidx1, Di, topK, pat, seed = case
    c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, topK, pat, "fp16", seed)
    g = load(name)
    got = _run(c, g["softmax_max"], g["softmax_sum"], "fp16")
    ref = sli.sli_grad(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"], c["w"], c["si"],
                       g["softmax_max"], g["softmax_sum"], c["scale"])
    _check(got, ref, name)
    # against the golden itself (it rounds inputs and dots to fp16 and skips out-of-range
    # scatter targets) at the reference test's own band (test_sli_grad_kl_loss_triton.py:9-10)
    for gi, key in zip(got, ("dQueryIndex", "dKeyIndex", "dW", "loss")):
        np.testing.assert_allclose(gi, g[key], rtol=1e-2, atol=1e-2, err_msg=name + " golden " + key)


@pytest.mark.parametrize("N1,Ni,topk,S1,S2", [(128, 64, 256, 24, 512), (32, 8, 64, 8, 300),
                                               (64, 16, 300, 6, 640)])
def test_sli_oracle_bf16(N1, Ni, topk, S1, S2):
    c = I.sli_case(1, S1, S2, N1, 512, Ni, 128, topk, "causal_random", "bf16", seed=N1 + Ni)
    mx, sm = sli.softmax_stats_full(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
    got = _run(c, mx, sm, "bf16", w_dtype="fp32")
    ref = sli.sli_grad(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"], c["w"], c["si"], mx, sm,
                       c["scale"])
    _check(got, ref, f"bf16 N1={N1}")


def test_sli_actual_lengths():
    c = I.sli_case(2, 6, 256, 32, 512, 16, 128, 128, "causal_random", "bf16", seed=77)
    aq, ak = [6, 4], [256, 200]
    mx, sm = sli.softmax_stats_full(c["q"], c["k"], c["qr"], c["kr"], c["scale"], act_q=aq, act_k=ak)
    got = _run(c, mx, sm, "bf16", act_q=aq, act_k=ak, w_dtype="fp32")
    ref = sli.sli_grad(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"], c["w"], c["si"], mx, sm,
                       c["scale"], act_q=aq, act_k=ak)
    _check(got, ref, "lens")
    assert np.all(got[0][1, 4:] == 0) and np.all(got[2][1, 4:] == 0)


def test_sli_partial_row_shards_sum_to_full_call():
    """Query-row shards through the partial entry point (fp32 dKeyIndex and loss left
    unreduced, as a multi-GPU caller gets them): their sum, cast once, equals the full call."""
    import dsa_triton_ascend_b200 as dsa
    B, S1, S2 = 1, 40, 512
    c = I.sli_case(B, S1, S2, 64, 512, 16, 128, 96, "causal_random", "bf16", seed=61)
    mx, sm = sli.softmax_stats_full(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
    t = {n: cuda(c[n], "bf16") for n in ("q", "k", "qr", "kr", "qi", "ki")}
    w = cuda(c["w"], "fp32")
    si, mxg, smg = icuda(c["si"]), cuda(mx, "fp32"), cuda(sm, "fp32")
    full = dsa.sparse_lightning_indexer_grad_kl_loss_triton(
        t["q"], t["k"], t["qi"], t["ki"], w, si, mxg, smg, query_rope=t["qr"], key_rope=t["kr"],
        scale_value=c["scale"])
    total, fin = None, []
    for r0, r1 in [(0, 17), (17, S1)]:
        cut = lambda x: x[:, r0:r1].contiguous()
        (acc, loss), finish = dsa.sparse_lightning_indexer_grad_kl_loss_partial(
            cut(t["q"]), t["k"], cut(t["qi"]), t["ki"], cut(w), cut(si),
            mxg[:, :, r0:r1].contiguous(), smg[:, :, r0:r1].contiguous(), query_rope=cut(t["qr"]),
            key_rope=t["kr"], actual_seq_qlen=[S1 - r0], scale_value=c["scale"])
        buf = finish.key_grad_buffer
        total = buf.clone() if total is None else total + buf
        fin.append((r0, r1, finish))
    # the summed buffer (dKeyIndex | loss) goes back into one shard's buffer, as an
    # all-reduce would leave it, and that shard's finish() casts it
    r0, r1, finish = fin[-1]
    finish.key_grad_buffer.copy_(total)
    dqi, dki, dw, loss = finish()
    dsa.check_device_errors()
    torch.testing.assert_close(loss, full[3], rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(dki.float(), full[1].float(), rtol=2e-2, atol=2e-3)
    assert torch.equal(dqi, full[0][:, r0:r1]) and torch.equal(dw, full[2][:, r0:r1])
