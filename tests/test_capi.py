"""The C-ABI library loads and exports every entry point include/dsa_b200.h declares (CPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsa_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t)\s+(dsa_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from dsa_triton_ascend_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from dsa_triton_ascend_b200 import build
        build.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_entry_points():
    names = declared_functions()
    for expected in ("dsa_version", "dsa_sfa_fwd", "dsa_sfa_bwd", "dsa_sfa_bwd_cast",
                     "dsa_li_score_topk", "dsa_sli_grad"):
        assert expected in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in dsa_b200.h but not exported"


def test_version_and_workspace_queries(lib):
    lib.dsa_version.restype = ctypes.c_int
    assert lib.dsa_version() >= 1
    for fn in ("dsa_sfa_fwd_workspace_size", "dsa_sfa_bwd_workspace_size", "dsa_sli_workspace_size"):
        f = getattr(lib, fn)
        f.restype = ctypes.c_int64
        f.argtypes = [ctypes.c_int64] * 3
        assert f(8, 16, 1) > 0
        assert f(-1, 16, 1) == -1
    f = lib.dsa_li_workspace_size
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_int64] * 3
    assert f(8, 1, 128) == 4 * 8 * 128


def test_null_params_rejected_without_gpu_work(lib):
    """Argument validation happens on the host before any CUDA call."""
    for fn in ("dsa_sfa_fwd", "dsa_sfa_bwd", "dsa_sfa_bwd_cast", "dsa_li_score_topk", "dsa_sli_grad"):
        f = getattr(lib, fn)
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        assert f(None, None) == 1   # DSA_ERR_INVALID_ARG


def test_bwd_rejects_misaligned_workspace_without_gpu_work(lib):
    """The backward's scratch takes 32-byte stores: a workspace not 256-byte aligned is an
    argument error, reported before any CUDA call (the pointers below are never touched)."""
    from dsa_triton_ascend_b200._lib import SfaBwdParams
    p = SfaBwdParams()
    fake = 1 << 20
    for name, _ in SfaBwdParams._fields_:
        if name in ("block_table", "dk", "dkr", "dv", "error_flag", "workspace"):
            continue
        if name in ("q", "q_rope", "key", "key_rope", "d_out", "out", "softmax_max", "softmax_sum",
                    "sparse_indices", "act_q", "act_k", "q_row_base", "k_row_base", "dq", "dqr",
                    "dk_acc", "dkr_acc", "dv_acc"):
            setattr(p, name, fake)
    p.num_rows, p.batch, p.n1, p.d, p.topk, p.sparse_block_size, p.kv_rows = 4, 1, 16, 512, 64, 1, 64
    f = lib.dsa_sfa_bwd_workspace_size
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_int64] * 3
    p.workspace_bytes = f(4, 64, 1)
    p.workspace = fake + 16            # 16-byte aligned, not 256
    g = lib.dsa_sfa_bwd
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    assert g(ctypes.addressof(p), None) == 1   # DSA_ERR_INVALID_ARG


def test_fast_forward_workspace_only_grows_for_split_calls(lib):
    """dsa_sfa_fwd_fast_workspace_size adds room for key-split partials only for calls with
    fewer rows than the 74 CTA pairs a B200 runs at once and enough tiles to split."""
    base = lib.dsa_sfa_fwd_workspace_size
    base.restype, base.argtypes = ctypes.c_int64, [ctypes.c_int64] * 3
    fast = lib.dsa_sfa_fwd_fast_workspace_size
    fast.restype, fast.argtypes = ctypes.c_int64, [ctypes.c_int64] * 5
    # decode: 32 rows, top-2048 -> 2 splits of 16 tiles
    assert fast(32, 128, 512, 2048, 1) >= base(32, 2048, 1) + 32 * 2 * 128 * (512 + 4) * 4
    # one row: as many splits as 4-tile pieces allow (32 tiles -> 8)
    assert fast(1, 128, 512, 2048, 1) >= base(1, 2048, 1) + 8 * 128 * (512 + 4) * 4
    # prefill (many rows) and short rows (fewer than 8 tiles): no split, the minimum
    assert fast(8192, 128, 512, 2048, 1) == base(8192, 2048, 1)
    assert fast(16, 128, 512, 256, 1) == base(16, 256, 1)
    assert fast(-1, 128, 512, 2048, 1) == -1 and fast(4, 0, 512, 2048, 1) == -1
