"""dsa_sfa_fwd_noalloc (the forward that allocates nothing) vs dsa_sfa_fwd, through the C-ABI (GPU).

The file name sorts last so that pytest runs it after every other test file; it must pass
both then and alone in a fresh process, where its first call is the one that looks up the
device's scratch array.
"""
import ctypes

import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import OUT_ATOL, OUT_RTOL, STAT_RTOL, cuda

pytestmark = pytest.mark.gpu


def _case_params(c, B, S1, S2, N1, D, topk, mode, noalloc_ws=False):
    """Build DsaSfaFwdParams for a dense BSND case; returns (params, keep-alive dict)."""
    from dsa_triton_ascend_b200 import _lib
    dev = torch.device("cuda", torch.cuda.current_device())
    t = {
        "q": cuda(c["q"], "bf16"), "qr": cuda(c["qr"], "bf16"),
        "k": cuda(c["k"], "bf16"), "kr": cuda(c["kr"], "bf16"),
        "si": torch.from_numpy(np.ascontiguousarray(c["si"], np.int32)).to(dev),
        "act_q": torch.full((B,), S1, dtype=torch.int32, device=dev),
        "act_k": torch.full((B,), S2, dtype=torch.int32, device=dev),
        "q_base": torch.arange(B, dtype=torch.int32, device=dev) * S1,
        "k_base": torch.arange(B, dtype=torch.int32, device=dev) * S2,
    }
    t["out"] = torch.empty_like(t["q"])
    t["smax"] = torch.zeros((B * S1, N1), dtype=torch.float32, device=dev)
    t["ssum"] = torch.zeros_like(t["smax"])
    num_rows = B * S1
    p = _lib.SfaFwdParams()
    p.q, p.q_rope, p.key, p.key_rope = (_lib.ptr(t[n]) for n in ("q", "qr", "k", "kr"))
    p.sparse_indices, p.act_q, p.act_k = _lib.ptr(t["si"]), _lib.ptr(t["act_q"]), _lib.ptr(t["act_k"])
    p.q_row_base, p.k_row_base, p.block_table = _lib.ptr(t["q_base"]), _lib.ptr(t["k_base"]), 0
    p.out, p.softmax_max, p.softmax_sum = _lib.ptr(t["out"]), _lib.ptr(t["smax"]), _lib.ptr(t["ssum"])
    p.error_flag = _lib.ptr(_lib.error_flag(dev))
    if noalloc_ws:
        p.workspace, p.workspace_bytes = 0, 0          # ignored by the no-alloc entry point
    else:
        # the workspace with room for key-split partials, so few-row calls split here too
        ws_bytes = _lib.lib().dsa_sfa_fwd_fast_workspace_size(num_rows, N1, D, topk, 1)
        t["ws"] = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        p.workspace, p.workspace_bytes = _lib.ptr(t["ws"]), ws_bytes
    p.num_rows, p.batch, p.n1, p.d, p.topk = num_rows, B, N1, D, topk
    p.sparse_block_size = 1
    p.kv_rows, p.page_size, p.max_blocks, p.s2_cap = B * S2, 0, 0, S2
    p.scale = float(c["scale"])
    p.sparse_mode = mode
    p.dtype = _lib.DSA_DTYPE_BF16
    return p, t


# (B, S1, S2, N1, D, topk, sparse_mode, seed): each case has fewer query rows than the one
# before it, so it runs over the previous call's leftover scratch contents.  The last one is
# decode-shaped (2 query rows of 2048 keys): both entry points split its keys over several
# CTA pairs and put the fp32 partials in their workspace (the fixed array for the no-alloc
# entry point).
CASES = [(2, 48, 640, 16, 512, 512, 3, 11), (1, 20, 300, 64, 512, 96, 0, 12),
         (1, 2, 4096, 128, 512, 2048, 0, 14)]


def test_noalloc_matches_workspace_entry_point_calls_in_a_row():
    from dsa_triton_ascend_b200 import _lib, check_device_errors
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    cases, noalloc, ref = [], [], []
    for B, S1, S2, N1, D, K, mode, seed in CASES:
        c = I.sfa_case(B, S1, S2, N1, D, K, 1, mode, "bf16", seed=seed)
        cases.append(c)
        noalloc.append(_case_params(c, B, S1, S2, N1, D, K, mode, noalloc_ws=True))
        ref.append(_case_params(c, B, S1, S2, N1, D, K, mode))
    # decode-shaped case: its partials fit in the fixed array beside the compaction, so the
    # no-alloc call takes the same split path as the reference call
    nr, n1, d, k = 2, 128, 512, 2048
    assert L.dsa_sfa_fwd_fast_workspace_size(nr, n1, d, k, 1) > L.dsa_sfa_fwd_workspace_size(nr, k, 1)
    assert L.dsa_sfa_fwd_fast_workspace_size(nr, n1, d, k, 1) <= _lib.SFA_FWD_NOALLOC_SCRATCH_BYTES
    # no-alloc calls back to back on one stream, then the workspace entry point
    for p, _ in noalloc:
        assert L.dsa_sfa_fwd_noalloc(ctypes.byref(p), ctypes.c_void_p(stream)) == _lib.DSA_OK
    for p, _ in ref:
        assert L.dsa_sfa_fwd(ctypes.byref(p), ctypes.c_void_p(stream)) == _lib.DSA_OK
    torch.cuda.synchronize()
    check_device_errors()
    for (_, a), (_, b) in zip(noalloc, ref):
        torch.testing.assert_close(a["out"].float(), b["out"].float(), rtol=OUT_RTOL, atol=OUT_ATOL)
        torch.testing.assert_close(a["smax"], b["smax"], rtol=STAT_RTOL, atol=1e-5)
        torch.testing.assert_close(a["ssum"], b["ssum"], rtol=STAT_RTOL, atol=1e-5)
        assert float(a["ssum"].abs().sum()) > 0


def test_noalloc_rejects_oversized_requests():
    from dsa_triton_ascend_b200 import _lib
    L = _lib.lib()
    B, S1, S2, N1, D, K = 1, 8, 256, 16, 512, 64
    c = I.sfa_case(B, S1, S2, N1, D, K, 1, 0, "bf16", seed=13)
    p, _ = _case_params(c, B, S1, S2, N1, D, K, 0, noalloc_ws=True)
    # claim more query rows than the fixed scratch array can hold; nothing is launched
    p.num_rows = _lib.SFA_FWD_NOALLOC_SCRATCH_BYTES // (4 * K) + 1
    assert L.dsa_sfa_fwd_workspace_size(p.num_rows, K, 1) > _lib.SFA_FWD_NOALLOC_SCRATCH_BYTES
    assert L.dsa_sfa_fwd_noalloc(ctypes.byref(p), None) == _lib.DSA_ERR_TOO_LARGE
