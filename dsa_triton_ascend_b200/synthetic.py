"""Seeded synthetic workloads of the benchmark configurations (generated on device).

No dataset is involved: BASELINE configurations are defined by shapes and value
distributions only (bf16 N(0,1) activations, causal distinct top-k key ids).
"""
from __future__ import annotations

import math

import torch


def causal_topk_ids(S1: int, S2: int, topk: int, gen: torch.Generator, device,
                    chunk: int = 1024) -> torch.Tensor:
    """[S1, topk] int32: for query s1 (aligned to the end of S2), min(topk, visible)
    distinct key ids drawn uniformly from its causal range, sorted, -1 padded."""
    out = torch.full((S1, topk), -1, dtype=torch.int32, device=device)
    offset = S2 - S1
    cols = torch.arange(S2, device=device)
    for r0 in range(0, S1, chunk):
        r1 = min(S1, r0 + chunk)
        rows = torch.arange(r0, r1, device=device)
        vis = (offset + rows + 1).clamp(max=S2)                         # visible keys
        u = torch.rand((r1 - r0, S2), generator=gen, device=device)
        u = torch.where(cols[None, :] < vis[:, None], u, torch.full_like(u, -1.0))
        k = min(topk, S2)
        val, idx = torch.topk(u, k, dim=1)
        idx = torch.where(val >= 0, idx, torch.full_like(idx, S2 + 1))
        idx, _ = torch.sort(idx, dim=1)
        idx = torch.where(idx > S2, torch.full_like(idx, -1), idx)
        out[r0:r1, :k] = idx.to(torch.int32)
    return out


def sfa_prefill(S1=8192, S2=8192, N1=128, D=512, topk=2048, B=1, seed=0, device="cuda",
                dtype=torch.bfloat16):
    """SFA forward+backward prefill inputs (BSND)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    r = lambda *shape: torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)
    q = r(B, S1, N1, D)
    qr = r(B, S1, N1, 64)
    k = r(B, S2, 1, D)
    kr = r(B, S2, 1, 64)
    dout = r(B, S1, N1, D)
    si = torch.stack([causal_topk_ids(S1, S2, topk, g, device) for _ in range(B)])
    return dict(q=q, qr=qr, k=k, kr=kr, dout=dout, si=si.reshape(B, S1, 1, topk),
                scale=1.0 / math.sqrt(D + 64))


def valid_pairs_per_row(si: torch.Tensor) -> torch.Tensor:
    """Number of valid (non -1) key ids per query row of a front-packed index tensor."""
    return (si.reshape(-1, si.shape[-1]) >= 0).sum(dim=1)
