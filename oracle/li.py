"""Numpy restatement of the lightning indexer score + top-k (test oracle only).

Reference: ``lightning_indexer_triton.py`` -- score kernel :171-280, top-k :339-357,
host API :462-550.  The reference ships no golden for this operator
(``test_li_triton.py`` compares against closed CANN kernels only).  The score arithmetic is
pinned through the reference's SLI golden instead: its stage 1
(``sli_grad_kl_loss_numpy.py:64-76``) computes the same I = sum_g w_g ReLU(qi_g . ki) for
every key of an index row, so with index rows that list every visible key
(``causal_continuous``) its ``I_scores`` are this function's scores;
``tests/test_oracle_golden.py`` checks that with ``emulate_fp16=True`` (the golden rounds
inputs, weights and each dot product to fp16).  The top-k order itself stays unpinned: the
reference calls MindSpore's closed, unstable ``mint.topk``.

score[b,s1,n2,s2] = sum_{g in group n2} ReLU(q[b,s1,g] . k[b,s2,n2]) * w[b,s1,g]   (fp32,
no scale; :264-269).  Invisible positions are -inf (:219-227, :271-276):
mode 3 -> visible iff s2 < min(act_k, clamp(act_k - act_q + s1 + 1, 0, S2));
mode 0 -> visible iff s2 < act_k; rows with s1 >= act_q are all -inf.
Top-k keeps k = min(sparse_count, S2) entries ordered by (score desc, index asc) -- the
ascending-index tie break the build's contract requires; the reference's default
``mint.topk`` leaves tie order unspecified (:349-351).  -inf entries get index -1 (:354-355).
"""
from __future__ import annotations

import numpy as np


def visible_limit(s1: int, aq: int, ak: int, S2: int, sparse_mode: int) -> int:
    """Number of visible keys of a query row (0 if the row is inactive)."""
    if s1 >= aq:
        return 0
    if sparse_mode == 3:
        causal = min(max(ak - aq + s1 + 1, 0), S2)
        return max(0, min(ak, causal))
    return max(0, min(ak, S2))


def li_score(q, k, w, act_q=None, act_k=None, sparse_mode=3, emulate_fp16=False):
    """q [B,S1,N1,D], k [B,S2,N2,D], w [B,S1,N1] -> scores [B,S1,N2,S2] fp32 (-inf = invisible).

    ``emulate_fp16``: round q, k, w and every dot product to fp16 first, as the reference's
    SLI golden does in its stage 1 (``sli_grad_kl_loss_numpy.py:22-29, :72``)."""
    h = lambda x: np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32); w = np.asarray(w, np.float32)
    if emulate_fp16:
        q, k, w = h(q), h(k), h(w)
    B, S1, N1, D = q.shape
    _, S2, N2, _ = k.shape
    G = N1 // N2
    act_q = [S1] * B if act_q is None else [int(x) for x in act_q]
    act_k = [S2] * B if act_k is None else [int(x) for x in act_k]
    out = np.full((B, S1, N2, S2), -np.inf, np.float32)
    for b in range(B):
        for n2 in range(N2):
            kb = k[b, :, n2, :]                                   # [S2, D]
            qg = q[b, :, n2 * G:(n2 + 1) * G, :]                  # [S1, G, D]
            wg = w[b, :, n2 * G:(n2 + 1) * G]                     # [S1, G]
            dots = np.einsum("sgd,td->sgt", qg, kb)               # [S1, G, S2]
            if emulate_fp16:
                dots = h(dots)
            sc = (np.maximum(dots, 0.0) * wg[:, :, None]).sum(axis=1)
            for s1 in range(S1):
                lim = visible_limit(s1, act_q[b], act_k[b], S2, sparse_mode)
                out[b, s1, n2, :lim] = sc[s1, :lim]
    return out


def li_topk(scores, sparse_count):
    """scores [..., S2] -> (indices int32 [..., k], values fp32 [..., k]), k = min(count, S2).

    Order: score descending, then index ascending; -inf -> index -1.
    """
    S2 = scores.shape[-1]
    kk = min(int(sparse_count), S2)
    flat = scores.reshape(-1, S2)
    idx = np.empty((flat.shape[0], kk), np.int32)
    val = np.empty((flat.shape[0], kk), np.float32)
    ar = np.arange(S2)
    for r in range(flat.shape[0]):
        order = np.lexsort((ar, -flat[r].astype(np.float64)))[:kk]
        idx[r] = order
        val[r] = flat[r, order]
    idx[np.isneginf(val)] = -1
    shp = scores.shape[:-1] + (kk,)
    return idx.reshape(shp), val.reshape(shp)
