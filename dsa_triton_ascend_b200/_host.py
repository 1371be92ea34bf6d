"""Host-side argument handling shared by the operators (no GPU compute here).

Mirrors the reference helpers ``_default_actual_seq_lens`` / ``_tnd_cumsum_to_per_batch``
(sparse_flash_attention_triton.py:338-347) but keeps everything on the device: TND
inputs are addressed through per-batch row offsets instead of being copied into a
padded BSND buffer.
"""
from __future__ import annotations

import torch

INT64_MAX = 9223372036854775807

# Small constant index tensors (row bases, default lengths) are cached per device: a
# decode step would otherwise spend more host time launching their fill kernels than
# the GPU spends on attention.  They are internal and never written after creation.
_const_cache: dict = {}


def _cached(key, make):
    t = _const_cache.get(key)
    if t is None:
        if len(_const_cache) > 256:
            _const_cache.clear()
        t = make()
        _const_cache[key] = t
    return t


def _i32_from_host(vals, device) -> torch.Tensor:
    """Host integers -> int32 device tensor without synchronising host and device.

    ``torch.tensor(list, device=cuda)`` copies from pageable memory and waits for the
    stream; a decode step would then pay a full host/device round trip per call. Values
    are cached per device (the tensors are never written), and a miss is copied from
    pinned memory asynchronously on the current stream."""
    key = ("i32", tuple(vals), str(device))
    t = _const_cache.get(key)
    if t is None:
        h = torch.tensor(list(vals), dtype=torch.int32).pin_memory()
        t = _cached(key, lambda: h.to(device, non_blocking=True))
    return t


def lens_tensor(lens, batch: int, default: int, device) -> torch.Tensor:
    """None -> [default]*batch; list/tuple/int -> int32 tensor; tensor -> int32 on device."""
    if lens is None or isinstance(lens, int):
        v = int(default) if lens is None else int(lens)
        return _cached(("full", batch, v, str(device)),
                       lambda: torch.full((batch,), v, dtype=torch.int32, device=device))
    if isinstance(lens, (list, tuple)):
        if len(lens) != batch:
            raise ValueError(f"expected {batch} sequence lengths, got {len(lens)}")
        return _i32_from_host([int(x) for x in lens], device)
    t = torch.as_tensor(lens)
    if t.numel() != batch:
        raise ValueError(f"expected {batch} sequence lengths, got {t.numel()}")
    return t.reshape(batch).to(device=device, dtype=torch.int32)


def cumulative(lens, device) -> torch.Tensor:
    """TND cumulative lengths (list/tuple/tensor) -> int32 tensor on device."""
    if lens is None:
        raise ValueError("TND layout requires cumulative actual sequence lengths")
    if isinstance(lens, (list, tuple)):
        return _i32_from_host([int(x) for x in lens], device)
    return torch.as_tensor(lens).reshape(-1).to(device=device, dtype=torch.int32)


def tnd_offsets(cum: torch.Tensor):
    """cumulative ends [B] -> (row_base [B], lens [B]); ``_tnd_cumsum_to_per_batch``."""
    base = torch.zeros_like(cum)
    if cum.numel() > 1:
        base[1:] = cum[:-1]
    return base, cum - base


def row_bases(batch: int, stride: int, device) -> torch.Tensor:
    return _cached(("bases", batch, int(stride), str(device)),
                   lambda: torch.arange(batch, dtype=torch.int32, device=device) * int(stride))


def dtype_code(t: torch.Tensor) -> int:
    from ._lib import DSA_DTYPE_BF16, DSA_DTYPE_FP16
    if t.dtype == torch.bfloat16:
        return DSA_DTYPE_BF16
    if t.dtype == torch.float16:
        return DSA_DTYPE_FP16
    raise ValueError(f"unsupported dtype {t.dtype}: expected bfloat16 or float16")


def require_cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors (no CPU fallback)")


def is_pow2_block(bs: int) -> bool:
    return 1 <= bs <= 128 and (bs & (bs - 1)) == 0
