"""ctypes binding of libdsa_b200.so (the sm_100a kernels).

The library is loaded from this package directory.  There is no fallback: if the
library is missing or cannot be loaded, every operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdsa_b200.so")

DSA_OK = 0
DSA_ERR_INVALID_ARG = 1
DSA_ERR_CUDA = 2
DSA_ERR_TMA_DESCRIPTOR = 3
DSA_ERR_TOO_LARGE = 4
SFA_FWD_NOALLOC_SCRATCH_BYTES = 16 << 20   # DSA_SFA_FWD_NOALLOC_SCRATCH_BYTES
DSA_DTYPE_BF16 = 0
DSA_DTYPE_FP16 = 1
DSA_DTYPE_FP32 = 2
DSA_DTYPE_FP8_E4M3 = 3

_ERR_TEXT = {
    DSA_ERR_INVALID_ARG: "invalid argument",
    DSA_ERR_CUDA: "CUDA launch error",
    DSA_ERR_TMA_DESCRIPTOR: "TMA descriptor rejected (misaligned or oversized tensor)",
    DSA_ERR_TOO_LARGE: "request exceeds the library's fixed scratch array",
}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64


class SfaFwdParams(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("q_rope", _p), ("key", _p), ("key_rope", _p),
        ("sparse_indices", _p), ("act_q", _p), ("act_k", _p), ("q_row_base", _p),
        ("k_row_base", _p), ("block_table", _p), ("out", _p), ("softmax_max", _p),
        ("softmax_sum", _p), ("error_flag", _p), ("workspace", _p), ("workspace_bytes", _i64),
        ("num_rows", _i64), ("batch", _i64), ("n1", _i64), ("d", _i64), ("topk", _i64),
        ("sparse_block_size", _i64), ("kv_rows", _i64), ("page_size", _i64),
        ("max_blocks", _i64), ("s2_cap", _i64),
        ("scale", ctypes.c_float), ("sparse_mode", ctypes.c_int32), ("dtype", ctypes.c_int32),
    ]


class SfaBwdParams(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("q_rope", _p), ("key", _p), ("key_rope", _p), ("d_out", _p), ("out", _p),
        ("softmax_max", _p), ("softmax_sum", _p), ("sparse_indices", _p), ("act_q", _p),
        ("act_k", _p), ("q_row_base", _p), ("k_row_base", _p), ("block_table", _p),
        ("dq", _p), ("dqr", _p), ("dk", _p), ("dkr", _p), ("dv", _p),
        ("dk_acc", _p), ("dkr_acc", _p), ("dv_acc", _p), ("error_flag", _p),
        ("workspace", _p), ("workspace_bytes", _i64),
        ("num_rows", _i64), ("batch", _i64), ("n1", _i64), ("d", _i64), ("topk", _i64),
        ("sparse_block_size", _i64), ("kv_rows", _i64), ("page_size", _i64),
        ("max_blocks", _i64), ("s2_cap", _i64),
        ("scale", ctypes.c_float), ("sparse_mode", ctypes.c_int32), ("dtype", ctypes.c_int32),
        ("defer_cast", ctypes.c_int32), ("accumulate", ctypes.c_int32),
        ("teacher", _p),
    ]


class LiParams(ctypes.Structure):
    _fields_ = [
        ("query", _p), ("key", _p), ("weights", _p), ("act_q", _p), ("act_k", _p),
        ("q_row_base", _p), ("k_row_base", _p), ("out_indices", _p), ("out_values", _p),
        ("error_flag", _p), ("workspace", _p), ("workspace_bytes", _i64),
        ("q_rows", _i64), ("batch", _i64), ("n1", _i64), ("n2", _i64), ("d", _i64),
        ("kv_rows", _i64), ("sparse_count", _i64), ("s2_row", _i64), ("s2_cap", _i64),
        ("q_len_max", _i64), ("q_len_dense", _i64),
        ("sparse_mode", ctypes.c_int32), ("dtype", ctypes.c_int32), ("weights_dtype", ctypes.c_int32),
        ("block_table", _p), ("page_size", _i64), ("max_blocks", _i64), ("key_scale", _p),
    ]


class SliParams(ctypes.Structure):
    _fields_ = [
        ("query", _p), ("key", _p), ("query_rope", _p), ("key_rope", _p), ("query_index", _p),
        ("key_index", _p), ("weights", _p), ("sparse_indices", _p), ("softmax_max", _p),
        ("softmax_sum", _p), ("act_q", _p), ("act_k", _p), ("d_query_index", _p),
        ("d_key_index", _p), ("d_weights", _p), ("dki_acc", _p), ("loss", _p),
        ("error_flag", _p), ("workspace", _p), ("workspace_bytes", _i64),
        ("batch", _i64), ("s1", _i64), ("s2", _i64), ("n1", _i64), ("d", _i64),
        ("n_index", _i64), ("d_index", _i64), ("topk", _i64),
        ("scale", ctypes.c_float), ("dtype", ctypes.c_int32), ("weights_dtype", ctypes.c_int32),
        ("teacher", _p),
    ]


class DenseIndexerParams(ctypes.Structure):
    _fields_ = [
        ("query", _p), ("key", _p), ("query_rope", _p), ("key_rope", _p), ("query_index", _p),
        ("key_index", _p), ("weights", _p), ("softmax_max", _p), ("softmax_sum", _p),
        ("index_max", _p), ("index_sum", _p), ("act_q", _p), ("act_k", _p),
        ("d_query_index", _p), ("d_key_index", _p), ("d_weights", _p), ("loss", _p),
        ("workspace", _p), ("workspace_bytes", _i64),
        ("batch", _i64), ("s1", _i64), ("s2", _i64), ("n1", _i64), ("n2", _i64), ("d", _i64),
        ("d_rope", _i64), ("n_index", _i64), ("d_index", _i64),
        ("scale", ctypes.c_float), ("dtype", ctypes.c_int32), ("weights_dtype", ctypes.c_int32),
    ]


_lock = threading.Lock()
_lib = None
_err_bufs: dict = {}


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raises if it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m dsa_triton_ascend_b200.build`"
                        " (there is no CPU fallback)")
                l = ctypes.CDLL(LIB_PATH)
                l.dsa_version.restype = ctypes.c_int
                l.dsa_sfa_fwd.argtypes = [ctypes.POINTER(SfaFwdParams), _p]
                l.dsa_sfa_fwd.restype = ctypes.c_int
                l.dsa_sfa_fwd_workspace_size.argtypes = [_i64, _i64, _i64]
                l.dsa_sfa_fwd_workspace_size.restype = _i64
                l.dsa_sfa_fwd_fast_workspace_size.argtypes = [_i64] * 5
                l.dsa_sfa_fwd_fast_workspace_size.restype = _i64
                l.dsa_sfa_fwd_noalloc.argtypes = [ctypes.POINTER(SfaFwdParams), _p]
                l.dsa_sfa_fwd_noalloc.restype = ctypes.c_int
                l.dsa_sfa_bwd.argtypes = [ctypes.POINTER(SfaBwdParams), _p]
                l.dsa_sfa_bwd.restype = ctypes.c_int
                l.dsa_sfa_bwd_cast.argtypes = [ctypes.POINTER(SfaBwdParams), _p]
                l.dsa_sfa_bwd_cast.restype = ctypes.c_int
                l.dsa_sfa_bwd_workspace_size.argtypes = [_i64, _i64, _i64]
                l.dsa_sfa_bwd_workspace_size.restype = _i64
                l.dsa_li_score_topk.argtypes = [ctypes.POINTER(LiParams), _p]
                l.dsa_li_score_topk.restype = ctypes.c_int
                l.dsa_li_workspace_size.argtypes = [_i64, _i64, _i64]
                l.dsa_li_workspace_size.restype = _i64
                l.dsa_sli_grad.argtypes = [ctypes.POINTER(SliParams), _p]
                l.dsa_sli_grad.restype = ctypes.c_int
                l.dsa_sli_cast.argtypes = [ctypes.POINTER(SliParams), _p]
                l.dsa_sli_cast.restype = ctypes.c_int
                l.dsa_sli_workspace_size.argtypes = [_i64, _i64, _i64]
                l.dsa_sli_workspace_size.restype = _i64
                for fn in (l.dsa_dense_indexer_softmax_lse, l.dsa_dense_indexer_grad_kl_loss):
                    fn.argtypes = [ctypes.POINTER(DenseIndexerParams), _p]
                    fn.restype = ctypes.c_int
                l.dsa_dense_indexer_workspace_size.argtypes = [_i64] * 4
                l.dsa_dense_indexer_workspace_size.restype = _i64
                _lib = l
    return _lib


def check(rc: int, what: str) -> None:
    if rc != DSA_OK:
        raise RuntimeError(f"{what}: {_ERR_TEXT.get(rc, 'error')} (code {rc})")


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 the kernels OR their error bits into."""
    key = torch.device(device).index
    buf = _err_bufs.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=device)
        _err_bufs[key] = buf
    return buf


def check_device_errors(device=None) -> None:
    """Synchronise and raise if any kernel reported a device-side error."""
    dev = torch.device("cuda" if device is None else device)
    buf = error_flag(dev)
    torch.cuda.synchronize(dev)
    v = int(buf.item())
    if v:
        buf.zero_()
        raise RuntimeError(f"dsa kernel reported device error bits 0x{v:x} "
                           "(bit1: bounded wait timed out, bit3: misaligned shared memory)")


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
