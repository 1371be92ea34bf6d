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


def test_dense_indexer_and_fp8_li_reject_bad_arguments_without_gpu_work(lib):
    """The dense indexer loss entry points and the FP8 / paged indexer validate their
    arguments on the host (the fake pointers below are never touched)."""
    from dsa_triton_ascend_b200._lib import DenseIndexerParams, LiParams
    for fn in ("dsa_dense_indexer_softmax_lse", "dsa_dense_indexer_grad_kl_loss"):
        f = getattr(lib, fn)
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        assert f(None, None) == 1
    ws = lib.dsa_dense_indexer_workspace_size
    ws.restype = ctypes.c_int64
    ws.argtypes = [ctypes.c_int64] * 4
    assert ws(1, 4, 100, 128) == (4 * 100 * 4 + 255) // 256 * 256 + 100 * 128 * 4
    assert ws(-1, 4, 100, 128) == -1
    fake = 1 << 20
    d = DenseIndexerParams()
    for name in ("query_index", "key_index", "weights", "act_q", "act_k", "index_max", "index_sum"):
        setattr(d, name, fake)
    d.batch, d.s1, d.s2, d.n_index, d.d_index = 1, 4, 64, 256, 128   # n_index > 128
    f = lib.dsa_dense_indexer_softmax_lse
    f.argtypes = [ctypes.POINTER(DenseIndexerParams), ctypes.c_void_p]
    assert f(ctypes.byref(d), None) == 1
    p = LiParams()
    for name in ("query", "key", "weights", "act_q", "act_k", "q_row_base", "k_row_base",
                 "out_indices", "workspace"):
        setattr(p, name, fake)
    p.q_rows, p.batch, p.n1, p.n2, p.d, p.kv_rows = 4, 1, 64, 1, 128, 256
    p.sparse_count, p.s2_row, p.s2_cap, p.q_len_max, p.q_len_dense = 64, 256, 256, 4, 4
    p.workspace_bytes = 1 << 20
    p.dtype = 3                       # DSA_DTYPE_FP8_E4M3 without key_scale
    g = lib.dsa_li_score_topk
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.POINTER(LiParams), ctypes.c_void_p]
    assert g(ctypes.byref(p), None) == 1
    p.dtype, p.key_scale = 0, 0
    p.s2_row = p.s2_cap = (1 << 17) + 1   # score rows are capped at 131,072 keys
    p.workspace_bytes = 1 << 40           # (so that the cap, not the workspace, is what fails)
    assert g(ctypes.byref(p), None) == 1
    p.workspace_bytes = 1 << 20
    p.s2_row = p.s2_cap = 256
    p.block_table, p.page_size, p.max_blocks = fake, 96, 4   # page neither 128k nor 128/k
    assert g(ctypes.byref(p), None) == 1
