"""Seeded numpy input generators shared by the golden-fixture script and the tests.

Frozen: the committed fixtures under ``tests/golden/`` were produced from exactly these
generators (numpy ``default_rng`` streams are platform independent), so changing any
function here requires regenerating the fixtures with ``gen_golden.py``.

Values are fp32 arrays that are exactly representable in the requested dtype.
"""
from __future__ import annotations

import numpy as np


def _round_bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    return ((u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).view(np.float32)


def cast(x, dtype):
    if dtype == "bf16":
        return _round_bf16(np.asarray(x, np.float32))
    if dtype == "fp16":
        return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, np.float32)


def randn(rng, shape, dtype, scale=1.0):
    return cast(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale), dtype)


def sparse_block_ids(rng, B, S1, S2, count, block, sparse_mode, act_q=None, act_k=None):
    """Front-packed sorted distinct block ids inside each row's window, -1 padded.

    Same contract as the reference generator ``test_sfa_triton.py:63-85``.
    """
    act_q = [S1] * B if act_q is None else list(act_q)
    act_k = [S2] * B if act_k is None else list(act_k)
    si = np.full((B, S1, 1, count), -1, np.int32)
    for b in range(B):
        for s1 in range(S1):
            if s1 >= act_q[b]:
                continue
            thr = act_k[b] if sparse_mode == 0 else act_k[b] - act_q[b] + s1 + 1
            if thr <= 0:
                continue
            nblk = -(-thr // block)
            n = min(count, nblk)
            si[b, s1, 0, :n] = np.sort(rng.permutation(nblk)[:n])
    return si


def sfa_case(B, S1, S2, N1, D, count, block=1, sparse_mode=3, dtype="bf16", seed=0,
             act_q=None, act_k=None):
    rng = np.random.default_rng(seed)
    q = randn(rng, (B, S1, N1, D), dtype)
    k = randn(rng, (B, S2, 1, D), dtype)
    qr = randn(rng, (B, S1, N1, 64), dtype)
    kr = randn(rng, (B, S2, 1, 64), dtype)
    si = sparse_block_ids(rng, B, S1, S2, count, block, sparse_mode, act_q, act_k)
    dout = randn(rng, (B, S1, N1, D), dtype)
    return dict(q=q, k=k, qr=qr, kr=kr, si=si, dout=dout,
                scale=float(1.0 / np.sqrt(D + 64)))


def config1(seed=0):
    """B=1, S1=128 at the last positions of S2=2048, N1=16, K=512."""
    return sfa_case(1, 128, 2048, 16, 512, 512, 1, 3, "bf16", seed)


def sli_indices(rng, B, S1, S2, topK, pattern):
    """Index patterns of ``test_sli_grad_kl_loss_triton.py:40-70`` (zero-filled tails)."""
    if pattern == "random":
        return rng.integers(0, S2, (B, S1, 1, topK)).astype(np.int32)
    si = np.zeros((B, S1, 1, topK), np.int32)
    if pattern == "causal_random":
        for b in range(B):
            for s1 in range(S1):
                vis = min(max(S2 - S1 + s1 + 1, 1), S2)
                n = min(topK, vis)
                si[b, s1, 0, :n] = rng.choice(vis, size=n, replace=False)
    elif pattern == "continuous":
        si[:] = (np.arange(topK) % S2).astype(np.int32)
    elif pattern == "repeated":
        row = np.zeros(topK, np.int32)
        row[1::2] = min(S2 - 1, 7)
        si[:] = row
    elif pattern == "causal_continuous":
        for s1 in range(S1):
            vis = min(max(S2 - S1 + s1 + 1, 1), S2)
            n = min(topK, vis)
            si[:, s1, 0, :n] = np.arange(n)
    else:
        raise ValueError(pattern)
    return si


def sli_case(B, S1, S2, N1, D, Nidx1, Di, topK, pattern="causal_random", dtype="bf16", seed=0):
    rng = np.random.default_rng(seed)
    q = randn(rng, (B, S1, N1, D), dtype)
    k = randn(rng, (B, S2, 1, D), dtype)
    qr = randn(rng, (B, S1, N1, 64), dtype)
    kr = randn(rng, (B, S2, 1, 64), dtype)
    qi = randn(rng, (B, S1, Nidx1, Di), dtype)
    ki = randn(rng, (B, S2, 1, Di), dtype)
    w = cast(np.abs(rng.standard_normal((B, S1, Nidx1), dtype=np.float32)), dtype)
    si = sli_indices(rng, B, S1, S2, topK, pattern)
    return dict(q=q, k=k, qr=qr, kr=kr, qi=qi, ki=ki, w=w, si=si,
                scale=float(1.0 / np.sqrt(D)))


def li_case(B, S1, S2, N1, N2, D, dtype="bf16", seed=0, wscale=None):
    rng = np.random.default_rng(seed)
    q = randn(rng, (B, S1, N1, D), dtype)
    k = randn(rng, (B, S2, N2, D), dtype)
    ws = (1.0 / np.sqrt(N1)) if wscale is None else wscale
    w = (rng.standard_normal((B, S1, N1), dtype=np.float32) * np.float32(ws)).astype(np.float32)
    return dict(q=q, k=k, w=w)
