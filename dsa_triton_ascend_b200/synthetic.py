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


def sfa_decode(B=32, N1=128, D=512, page=128, pool_blocks=16384, max_blocks=512, topk=2048,
               len_lo=8192, len_hi=65536, seed=0, device="cuda", dtype=torch.bfloat16):
    """paged-KV decode (PA_BSND, S1 = 1).

    Per-batch KV lengths uniform in [len_lo, len_hi]; block_table [B, max_blocks] is a random
    permutation of the pool's blocks; each query row gets `topk` distinct token ids sampled
    uniformly from [0, kv_len), sorted."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    r = lambda *shape: torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)
    lens = torch.randint(len_lo, len_hi + 1, (B,), generator=g, device=device)
    cache = r(pool_blocks, page, 1, D)
    cache_r = r(pool_blocks, page, 1, 64)
    bt = torch.randperm(pool_blocks, generator=g, device=device)[: B * max_blocks]
    bt = bt.reshape(B, max_blocks).int()
    q, qr = r(B, 1, N1, D), r(B, 1, N1, 64)
    span = max_blocks * page
    u = torch.rand(B, span, generator=g, device=device)
    u = torch.where(torch.arange(span, device=device)[None] < lens[:, None], u, -1.0)
    si = torch.sort(torch.topk(u, topk, dim=1).indices, dim=1).values.int().reshape(B, 1, 1, topk)
    return dict(q=q, qr=qr, cache=cache, cache_r=cache_r, block_table=bt, lens=lens.tolist(),
                si=si, page=page, scale=1.0 / math.sqrt(D + 64))


def sli_prefill(S=8192, N1=128, D=512, n_index=64, d_index=128, topk=2048, seed=0,
                device="cuda", dtype=torch.bfloat16):
    """BASELINE config 5 inputs except the softmax statistics (which come from running
    config 4's forward on the same query / key): BSND, B=1, S1=S2=S."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    r = lambda *shape: torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)
    q, qr, k, kr = r(1, S, N1, D), r(1, S, N1, 64), r(1, S, 1, D), r(1, S, 1, 64)
    qi, ki = r(1, S, n_index, d_index), r(1, S, 1, d_index)
    w = torch.randn(1, S, n_index, generator=g, device=device) / 8
    si = causal_topk_ids(S, S, topk, g, device).reshape(1, S, 1, topk)
    return dict(q=q, qr=qr, k=k, kr=kr, qi=qi, ki=ki, w=w, si=si, scale=1.0 / math.sqrt(D + 64))
