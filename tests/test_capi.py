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
