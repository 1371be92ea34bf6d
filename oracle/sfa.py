"""Numpy restatement of sparse flash attention forward/backward (test oracle only).

Reference files (paths inside the reference project):

* forward kernel  ``sparse_flash_attention_triton.py:189-332`` (mask rules :264-268,
  empty rows keep zeros :326-332), host API :483-641
* forward golden  ``sparse_flash_attention_numpy.py:63-160``
* backward kernel ``sparse_flash_attention_grad_triton.py:158-308``, host :382-541
* backward golden ``sparse_flash_attention_grad_numpy.py:34-143``

Index semantics follow the *kernel*: every entry of a row's index list is tested on
its own (``tok != -1 and tok < threshold and tok < act_k``).  The goldens instead
stop at the first -1 and scan only the first ``ceil(threshold / block)`` entries; the
two agree whenever valid ids are packed at the front of the row, which is the
contract the reference tests generate (``test_sfa_triton.py:63-85``).  Negative ids
other than -1 are treated as invalid here (the reference would read out of bounds).
"""
from __future__ import annotations

import numpy as np

INT64_MAX = 9223372036854775807


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 -> fp32 (finite inputs), as the goldens round probs/outputs."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    return ((u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    return np.asarray(x, dtype=np.float32)


def expand_block_indices(si: np.ndarray, block: int) -> np.ndarray:
    """Block ids [..., K] -> token ids [..., K*block]; -1 stays -1.

    Restates ``sparse_flash_attention_triton.py:406-421``.
    """
    if block == 1:
        return si.astype(np.int32)
    base = si.astype(np.int64)[..., None]
    offs = np.arange(block, dtype=np.int64)
    tok = np.where(base == -1, -1, base * block + offs)
    return tok.reshape(*si.shape[:-1], si.shape[-1] * block).astype(np.int32)


def tnd_to_bsnd(t: np.ndarray, lens) -> np.ndarray:
    """[T, ...] -> [B, max_len, ...] zero padded; ``sparse_flash_attention_triton.py:350-363``."""
    lens = [int(x) for x in lens]
    out = np.zeros((len(lens), max(lens) if lens else 0) + t.shape[1:], dtype=t.dtype)
    start = 0
    for b, n in enumerate(lens):
        out[b, :n] = t[start:start + n]
        start += n
    return out


def bsnd_to_tnd(t: np.ndarray, lens) -> np.ndarray:
    """Inverse of :func:`tnd_to_bsnd`; ``sparse_flash_attention_triton.py:366-379``."""
    return np.concatenate([t[b, :int(n)] for b, n in enumerate(lens)], axis=0)


def cumsum_to_lens(cum) -> list:
    """TND cumulative lengths -> per-batch lengths; ``sparse_flash_attention_triton.py:345-347``."""
    cum = [int(x) for x in cum]
    return [c - p for c, p in zip(cum, [0] + cum[:-1])]


def pa_to_bsnd(cache: np.ndarray, block_table: np.ndarray, max_s2: int) -> np.ndarray:
    """Paged cache [nblk, bs, N, Dx] -> dense [B, max_s2, N, Dx].

    Restates ``sparse_flash_attention_triton.py:382-403``: block id -1 leaves zeros.
    """
    nblk, bs, n, dx = cache.shape
    B = block_table.shape[0]
    out = np.zeros((B, max_s2, n, dx), dtype=cache.dtype)
    for b in range(B):
        for i in range(block_table.shape[1]):
            bid = int(block_table[b, i])
            if bid == -1:
                continue
            dst = i * bs
            if dst >= max_s2:
                break
            end = min(dst + bs, max_s2)
            out[b, dst:end] = cache[bid, :end - dst]
    return out


def _row_window(s1: int, aq: int, ak: int, sparse_mode: int):
    """(active, threshold) of a query row; ``sparse_flash_attention_triton.py:242-252``."""
    threshold = ak if sparse_mode == 0 else ak - aq + s1 + 1
    return (s1 < aq) and (threshold > 0), threshold


def valid_positions(tok_row: np.ndarray, s1: int, aq: int, ak: int, sparse_mode: int, s2: int):
    """Kernel mask ``sparse_flash_attention_triton.py:264-266`` -> kept token ids (in order)."""
    active, thr = _row_window(s1, aq, ak, sparse_mode)
    if not active:
        return np.zeros(0, dtype=np.int64)
    t = tok_row.astype(np.int64)
    keep = (t >= 0) & (t < thr) & (t < ak) & (t < s2)
    return t[keep]


def sfa_fwd(q, k, qr, kr, tok_idx, scale, act_q=None, act_k=None, sparse_mode=3,
            dtype="bf16", rounding="golden"):
    """SFA forward on BSND numpy inputs (fp32 accumulate).

    q [B,S1,N1,D], k [B,S2,1,D] (value = k[..., :D]), qr [B,S1,N1,64], kr [B,S2,1,64],
    tok_idx [B,S1,1,K] token ids (block ids already expanded).  Returns
    (out [B,S1,N1,D] rounded to ``dtype``, softmax_max [B,1,S1,N1], softmax_sum
    [B,1,S1,N1]); inactive/empty rows stay zero (``sparse_flash_attention_triton.py:326-332``).
    ``rounding`` picks where probabilities are rounded to ``dtype`` before P@V:
    "golden" rounds the normalised probabilities (``sparse_flash_attention_numpy.py:108-114,
    149``); "kernel" rounds the unnormalised exp(s - max) and divides the fp32 product by
    the row sum afterwards, as the reference kernel does (``sparse_flash_attention_triton.py:
    309-324``).  Both are within rounding noise of each other.
    """
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32)
    qr = np.asarray(qr, np.float32); kr = np.asarray(kr, np.float32)
    B, S1, N1, D = q.shape
    S2 = k.shape[1]
    act_q = [S1] * B if act_q is None else [int(x) for x in act_q]
    act_k = [S2] * B if act_k is None else [int(x) for x in act_k]
    out = np.zeros((B, S1, N1, D), np.float32)
    smax = np.zeros((B, 1, S1, N1), np.float32)
    ssum = np.zeros((B, 1, S1, N1), np.float32)
    for b in range(B):
        kb = np.concatenate([k[b, :, 0, :], kr[b, :, 0, :]], axis=-1)
        for s1 in range(S1):
            pos = valid_positions(tok_idx[b, s1, 0], s1, act_q[b], act_k[b], sparse_mode, S2)
            if pos.size == 0:
                continue
            kk = kb[pos]
            qf = np.concatenate([q[b, s1], qr[b, s1]], axis=-1)        # [N1, D+64]
            sc = (qf @ kk.T) * np.float32(scale)                          # [N1, P]
            m = sc.max(axis=1)
            e = np.exp(sc - m[:, None])
            l = e.sum(axis=1)
            if rounding == "kernel":
                out[b, s1] = (round_to(e, dtype) @ kk[:, :D]) / l[:, None]
            else:
                out[b, s1] = round_to(e / l[:, None], dtype) @ kk[:, :D]
            smax[b, 0, s1] = m
            ssum[b, 0, s1] = l
    return round_to(out, dtype), smax, ssum


def sfa_bwd(q, k, qr, kr, tok_idx, d_out, out, smax, ssum, scale, act_q=None, act_k=None,
            sparse_mode=3, dtype="bf16", rounding="golden", round_out=True):
    """SFA backward on BSND numpy inputs; restates ``sparse_flash_attention_grad_triton.py:189-308``.

    P = exp(s - max) / sum (sum <= 0 -> 1, :232-234), delta = rowsum(dO*O) (:237),
    dS = P (dO.v - delta) scale (:262-268); dQ = dS K, dQr = dS Kr; dK += dS^T q,
    dKr += dS^T qr, dV += P^T dO scatter-added over rows (:270-300).  Returns
    (dq, dk, dv, dqr, dkr) rounded to ``dtype``.  ``rounding="kernel"`` additionally rounds P
    and dS to ``dtype`` before the three products, as the reference kernel does
    (``dS.to(k_full.dtype)``, ``P_t.to(do_sub.dtype)``, :271-298); the golden keeps them fp32.
    ``round_out=False`` returns the five gradients in fp32 (for sums such as dk + dv, which a
    merged caller rounds once).
    """
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32)
    qr = np.asarray(qr, np.float32); kr = np.asarray(kr, np.float32)
    do = np.asarray(d_out, np.float32); o = np.asarray(out, np.float32)
    B, S1, N1, D = q.shape
    S2 = k.shape[1]
    Dr = qr.shape[-1]
    act_q = [S1] * B if act_q is None else [int(x) for x in act_q]
    act_k = [S2] * B if act_k is None else [int(x) for x in act_k]
    dq = np.zeros_like(q); dqr = np.zeros_like(qr)
    dk = np.zeros((B, S2, 1, D), np.float32)
    dkr = np.zeros((B, S2, 1, Dr), np.float32)
    dv = np.zeros((B, S2, 1, D), np.float32)
    for b in range(B):
        kn = k[b, :, 0, :]; krb = kr[b, :, 0, :]
        for s1 in range(S1):
            pos = valid_positions(tok_idx[b, s1, 0], s1, act_q[b], act_k[b], sparse_mode, S2)
            if pos.size == 0:
                continue
            kk = kn[pos]; kkr = krb[pos]
            sc = (q[b, s1] @ kk.T + qr[b, s1] @ kkr.T) * np.float32(scale)   # [N1, P]
            mx = smax[b, 0, s1].astype(np.float32)
            sm = ssum[b, 0, s1].astype(np.float32)
            sm = np.where(sm > 0, sm, np.float32(1.0))
            P = np.exp(sc - mx[:, None]) / sm[:, None]
            dpv = do[b, s1] @ kk.T
            delta = (do[b, s1] * o[b, s1]).sum(axis=1)
            dS = P * (dpv - delta[:, None]) * np.float32(scale)
            if rounding == "kernel":
                P = round_to(P, dtype)
                dS = round_to(dS, dtype)
            dq[b, s1] = dS @ kk
            dqr[b, s1] = dS @ kkr
            np.add.at(dk[b, :, 0, :], pos, dS.T @ q[b, s1])
            np.add.at(dkr[b, :, 0, :], pos, dS.T @ qr[b, s1])
            np.add.at(dv[b, :, 0, :], pos, P.T @ do[b, s1])
    r = (lambda x: round_to(x, dtype)) if round_out else (lambda x: x)
    return r(dq), r(dk), r(dv), r(dqr), r(dkr)
