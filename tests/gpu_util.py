"""Helpers for the GPU parity tests (torch <-> numpy, tolerance checks)."""
import numpy as np
import torch

TORCH_DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}

# Tolerances of the build contract (outputs/gradients: bf16 rtol 2e-2, atol 2e-3;
# softmax statistics and losses: 1e-4 relative).
OUT_RTOL, OUT_ATOL = 2e-2, 2e-3
STAT_RTOL = 1e-4


def cuda(x, dtype="bf16"):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", TORCH_DT[dtype])


def icuda(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.int32)).to("cuda")


def host(t):
    return t.detach().float().cpu().numpy()


def assert_close(got, ref, rtol=OUT_RTOL, atol=OUT_ATOL, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} vs {ref.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    bad = np.abs(got - ref) > atol + rtol * np.abs(ref)
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {bad.sum()}/{bad.size} outside rtol={rtol} atol={atol}; first at {tuple(i)}: "
            f"got {got[tuple(i)]} ref {ref[tuple(i)]}; max abs err {np.abs(got - ref).max():.3g}")
