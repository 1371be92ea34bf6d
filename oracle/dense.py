"""Numpy restatement of the dense lightning-indexer KL loss (test infrastructure only).

Follows ``dense_loss_backward_triton.py`` of the reference: the index softmax statistics
(``_dense_indexer_stats_kernel``, :129-179), the loss (``_dense_loss_kernel``, :263-320),
dQueryIndex / dWeights (``_dense_main_grad_kernel``, :182-260) and the dKeyIndex scatter
(``_dense_dkey_index_kernel``, :323-397).  All visible keys of a query row take part (no
top-k): key s2 is visible to row s1 when s1 < act_q and s2 < min(max(act_k - act_q + s1 + 1,
0), S2).  The reference checks its statistics against a numpy baseline of the same formula
(``test_dense_loss_backward_triton.py:100-135``) and its gradients only against a CANN
kernel that does not exist here, so the gradients of this oracle are unpinned; they are
cross-checked against the sparse oracle ``oracle/sli.py`` (pinned to the reference's numpy
golden) on index sets that list every visible key.
"""
from __future__ import annotations

import numpy as np

EPS = 1e-8


def _visible(s1, aq, ak, S2):
    if s1 >= aq:
        return 0
    return min(max(ak - aq + s1 + 1, 0), S2)


def _lens(lens, B, default):
    return [int(default)] * B if lens is None else [int(x) for x in lens]


def index_scores(qi_row, ki_b, w_row, vis):
    """I[k] = sum_g w_g ReLU(qi_g . ki_k) for k < vis; also returns the dots [Ni, vis]."""
    dots = qi_row.astype(np.float64) @ ki_b[:vis].astype(np.float64).T
    return (w_row.astype(np.float64)[:, None] * np.maximum(dots, 0.0)).sum(0), dots


def dense_lse(qi, ki, w, act_q=None, act_k=None):
    """Index softmax statistics: (max [B,1,S1], sum of exp(I - max) [B,1,S1]); rows without
    visible keys give (-inf, 0) (:166-179)."""
    B, S1, Ni, Di = qi.shape
    S2 = ki.shape[1]
    aq, ak = _lens(act_q, B, S1), _lens(act_k, B, S2)
    mx = np.full((B, 1, S1), -np.inf, np.float32)
    sm = np.zeros((B, 1, S1), np.float32)
    for b in range(B):
        for s1 in range(S1):
            vis = _visible(s1, aq[b], ak[b], S2)
            if vis <= 0:
                continue
            I, _ = index_scores(qi[b, s1], ki[b, :, 0], w[b, s1], vis)
            m = I.max()
            mx[b, 0, s1] = m
            sm[b, 0, s1] = np.exp(I - m).sum()
    return mx, sm


def dense_grad(q, k, qr, kr, qi, ki, w, smax, ssum, imax, isum, scale, act_q=None, act_k=None):
    """(dQueryIndex, dKeyIndex, dWeights, loss) in float64.

    q [B,S1,N1,D], k [B,S2,N2,D], qr/kr [..,64] or None, qi [B,S1,Ni,Di], ki [B,S2,1,Di],
    w [B,S1,Ni], smax/ssum [B,N2,S1,N1/N2] (attention statistics), imax/isum [B,1,S1]."""
    B, S1, N1, D = q.shape
    S2, N2 = k.shape[1], k.shape[2]
    G = N1 // N2
    Ni, Di = qi.shape[2], qi.shape[3]
    aq, ak = _lens(act_q, B, S1), _lens(act_k, B, S2)
    dqi = np.zeros((B, S1, Ni, Di))
    dki = np.zeros((B, S2, 1, Di))
    dw = np.zeros((B, S1, Ni))
    loss = 0.0
    for b in range(B):
        for s1 in range(S1):
            vis = _visible(s1, aq[b], ak[b], S2)
            im, isu = float(imax[b, 0, s1]), float(isum[b, 0, s1])
            if vis <= 0 or not isu > 0.0:
                continue
            I, dots = index_scores(qi[b, s1], ki[b, :, 0], w[b, s1], vis)
            student = np.exp(I - im) / max(isu, EPS)
            p = np.zeros(vis)
            for h in range(N1):
                n2, g = h // G, h % G
                s = k[b, :vis, n2].astype(np.float64) @ q[b, s1, h].astype(np.float64)
                if qr is not None:
                    s = s + kr[b, :vis, n2].astype(np.float64) @ qr[b, s1, h].astype(np.float64)
                p += np.exp(s * scale - smax[b, n2, s1, g]) / (ssum[b, n2, s1, g] + EPS)
            p /= N1
            pc, qc = np.maximum(p, EPS), np.maximum(student, EPS)
            loss += float((pc * (np.log(pc) - np.log(qc))).sum())
            di = student - p
            relu = np.maximum(dots, 0.0)
            dw[b, s1] = relu @ di
            coeff = (dots > 0) * di[None, :] * w[b, s1].astype(np.float64)[:, None]   # [Ni, vis]
            dqi[b, s1] = coeff @ ki[b, :vis, 0].astype(np.float64)
            dki[b, :vis, 0] += coeff.T @ qi[b, s1].astype(np.float64)
    return dqi, dki, dw, loss


def attention_stats(q, k, qr, kr, scale, act_q=None, act_k=None):
    """Softmax max / sum of the full attention over the same visible keys, [B, N2, S1, G]
    (the statistics the teacher distribution takes, here from scores in float64)."""
    B, S1, N1, D = q.shape
    S2, N2 = k.shape[1], k.shape[2]
    G = N1 // N2
    aq, ak = _lens(act_q, B, S1), _lens(act_k, B, S2)
    mx = np.full((B, N2, S1, G), -np.inf, np.float32)
    sm = np.zeros((B, N2, S1, G), np.float32)
    for b in range(B):
        for s1 in range(S1):
            vis = _visible(s1, aq[b], ak[b], S2)
            if vis <= 0:
                continue
            for h in range(N1):
                n2, g = h // G, h % G
                s = k[b, :vis, n2].astype(np.float64) @ q[b, s1, h].astype(np.float64)
                if qr is not None:
                    s = s + kr[b, :vis, n2].astype(np.float64) @ qr[b, s1, h].astype(np.float64)
                s = s * scale
                mx[b, n2, s1, g] = s.max()
                sm[b, n2, s1, g] = np.exp(s - s.max()).sum()
    return mx, sm
