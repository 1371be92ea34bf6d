"""Streamed forward + backward of host tensors vs the direct operator calls (GPU).

sfa_fwd_bwd_from_host splits the query rows into chunks, runs them on a kernel stream
between two copy streams and adds the key gradients of all chunks into one fp32 set; its
results must match one direct call of the forward and backward on the whole query.
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import OUT_ATOL, OUT_RTOL

pytestmark = pytest.mark.gpu


def _direct(c, mode, dt):
    import dsa_triton_ascend_b200 as dsa
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).cuda().to(dt)
         for k in ("q", "qr", "k", "kr", "dout")}
    si = torch.from_numpy(np.ascontiguousarray(c["si"], np.int32)).cuda()
    o, m, s_ = dsa.sparse_flash_attention_triton(
        t["q"], t["k"], t["k"], si, c["scale"], query_rope=t["qr"], key_rope=t["kr"],
        sparse_mode=mode, return_softmax_lse=True)
    dq, dk, dv, dqr, dkr = dsa.sparse_flash_attention_grad_triton(
        t["q"], t["k"], t["k"], si, t["dout"], o, m, s_, c["scale"], query_rope=t["qr"],
        key_rope=t["kr"], sparse_mode=mode)
    return [x.float().cpu() for x in (o, dq, dk, dv, dqr, dkr)]


@pytest.mark.parametrize("mode,chunks", [(3, 3), (0, 4)])
def test_streamed_matches_direct(mode, chunks):
    import dsa_triton_ascend_b200 as dsa
    dt = torch.bfloat16
    c = I.sfa_case(2, 96, 512, 16, 512, 128, 1, mode, "bf16", seed=21 + mode)
    host = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(dt).pin_memory()
            for k in ("q", "qr", "k", "kr", "dout")}
    hsi = torch.from_numpy(np.ascontiguousarray(c["si"], np.int32)).pin_memory()
    res = dsa.sfa_fwd_bwd_from_host(host["q"], host["k"], hsi, host["dout"], c["scale"],
                                    host["qr"], host["kr"], sparse_mode=mode, chunks=chunks)
    torch.cuda.synchronize()
    dsa.check_device_errors()
    ref = _direct(c, mode, dt)
    for got, want, name in zip(res, ref, ("out", "dq", "dk", "dv", "dq_rope", "dk_rope")):
        torch.testing.assert_close(got.float(), want, rtol=OUT_RTOL, atol=OUT_ATOL, msg=name)


def test_streamed_shard_of_a_causal_query():
    """Rows [r0, S1) passed alone with actual_seq_length_query = S1 - r0 give the rows of
    the whole query (the multi-GPU shard case)."""
    import dsa_triton_ascend_b200 as dsa
    dt = torch.bfloat16
    c = I.sfa_case(1, 128, 512, 16, 512, 128, 1, 3, "bf16", seed=33)
    r0 = 40
    host = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(dt) for k in ("q", "qr", "dout")}
    host = {k: v[:, r0:].contiguous().pin_memory() for k, v in host.items()}
    hk = torch.from_numpy(np.ascontiguousarray(c["k"])).to(dt).pin_memory()
    hkr = torch.from_numpy(np.ascontiguousarray(c["kr"])).to(dt).pin_memory()
    hsi = torch.from_numpy(np.ascontiguousarray(c["si"][:, r0:], np.int32)).pin_memory()
    out, dq, *_ = dsa.sfa_fwd_bwd_from_host(host["q"], hk, hsi, host["dout"], c["scale"],
                                            host["qr"], hkr, sparse_mode=3, chunks=2,
                                            actual_seq_length_query=128 - r0)
    torch.cuda.synchronize()
    ref = _direct(c, 3, dt)
    torch.testing.assert_close(out.float(), ref[0][:, r0:], rtol=OUT_RTOL, atol=OUT_ATOL)
    torch.testing.assert_close(dq.float(), ref[1][:, r0:], rtol=OUT_RTOL, atol=OUT_ATOL)
