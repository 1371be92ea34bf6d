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
