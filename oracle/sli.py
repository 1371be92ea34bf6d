"""Numpy restatement of the sparse lightning-indexer KL-loss gradient (test oracle only).

Reference kernel ``sparse_lightning_indexer_grad_kl_loss_triton.py:74-327`` (host
:355-464, :520-556) and golden ``sli_grad_kl_loss_numpy.py:16-152``.

Per query row (b, s1) with s1 < act_q:

* window n = min(topK, max(act_k - act_q + s1 + 1, 0)) entries of the index row
  (:107), ids clamped to [0, S2-1] (:63, :300) -- -1 is *not* special;
* I[k] = sum_g w_g ReLU(qi_g . ki[idx_k])                       (stage 1, :119-136)
* p[k] = (1/N1) sum_h exp(scale (q_h . k + qr_h . kr)[idx_k] - max_h) / (sum_h + 1e-8)
                                                                (stage 2, :145-177)
* sI = exp(I - max I) / (sum exp(I - max I) + 1e-8);  dI = sI - p (stages 3-4, :180-209)
* loss += sum_k max(p,1e-8) (log max(p,1e-8) - log max(sI,1e-8)), summed over rows (:210-216)
* dW_g = sum_k dI ReLU_g;  dQI_g = sum_k dI w_g 1[ReLU_g > 0] ki[idx_k]   (stage 5, :219-263)
* dKI[idx_k] += sum_g dI_k w_g 1[ReLU_gk > 0] qi_g             (scatter, :266-317)

Rows with s1 >= act_q produce zeros (the kernel returns early, :102-103).

``emulate_fp16=True`` reproduces the golden's CANN emulation (inputs rounded to fp16,
stage-1/2 dot products rounded to fp16, :22-29, :72, :89) and its scatter rule that skips
out-of-range ids (:143-144); the default fp32 mode follows the kernel, which is the
behaviour the CUDA kernels implement.
"""
from __future__ import annotations

import numpy as np


def sli_grad(q, k, qr, kr, qi, ki, w, si, sm_max, sm_sum, scale, act_q=None, act_k=None,
             emulate_fp16=False):
    """Returns dict with dQueryIndex [B,S1,Nidx1,Di], dKeyIndex [B,S2,1,Di], dWeights
    [B,S1,Nidx1], loss [1] (all fp32) plus intermediates."""
    f = (lambda x: np.asarray(x, np.float32).astype(np.float16).astype(np.float32)) \
        if emulate_fp16 else (lambda x: np.asarray(x, np.float32))
    q, k, qr, kr, qi, ki, w = map(f, (q, k, qr, kr, qi, ki, w))
    si = np.asarray(si).astype(np.int64)
    sm_max = np.asarray(sm_max, np.float32); sm_sum = np.asarray(sm_sum, np.float32)
    rnd = (lambda x: x.astype(np.float16).astype(np.float32)) if emulate_fp16 else (lambda x: x)
    B, S1, N1, D = q.shape
    S2 = k.shape[1]
    Nidx1, Di = qi.shape[2], qi.shape[3]
    topK = si.shape[3]
    act_q = [S1] * B if act_q is None else [int(x) for x in act_q]
    act_k = [S2] * B if act_k is None else [int(x) for x in act_k]
    eps = np.float32(1e-8)

    dqi = np.zeros((B, S1, Nidx1, Di), np.float32)
    dki = np.zeros((B, S2, 1, Di), np.float32)
    dw = np.zeros((B, S1, Nidx1), np.float32)
    loss = np.float64(0.0)
    for b in range(B):
        for s1 in range(S1):
            if s1 >= act_q[b]:
                continue
            n = min(topK, max(act_k[b] - act_q[b] + s1 + 1, 0))
            if n == 0:
                continue
            raw = si[b, s1, 0, :n]
            idx = np.clip(raw, 0, S2 - 1)
            kig = ki[b, idx, 0, :]                                  # [n, Di]
            dots = rnd(qi[b, s1] @ kig.T)                           # [Nidx1, n]
            relu = np.maximum(dots, 0.0)
            I = (w[b, s1][:, None] * relu).sum(axis=0)             # [n]
            kg = k[b, idx, 0, :]; krg = kr[b, idx, 0, :]
            sc = rnd((q[b, s1] @ kg.T + qr[b, s1] @ krg.T) * np.float32(scale))   # [N1, n]
            probs = np.exp(sc - sm_max[b, 0, s1][:, None]) / (sm_sum[b, 0, s1][:, None] + eps)
            p = probs.sum(axis=0) * np.float32(1.0 / N1)
            e = np.exp(I - I.max())
            sI = e / (e.sum() + eps)
            dI = sI - p
            pc = np.maximum(p, eps); sc_ = np.maximum(sI, eps)
            loss += float((pc * (np.log(pc) - np.log(sc_))).sum())
            dw[b, s1] = relu @ dI
            coef = (relu > 0).astype(np.float32) * w[b, s1][:, None] * dI[None, :]   # [Nidx1, n]
            dqi[b, s1] = coef @ kig
            contrib = coef.T @ qi[b, s1]                            # [n, Di]
            if emulate_fp16:
                keep = (raw >= 0) & (raw < S2)
                np.add.at(dki[b, :, 0, :], raw[keep], contrib[keep])
            else:
                np.add.at(dki[b, :, 0, :], idx, contrib)
    return {"dQueryIndex": dqi, "dKeyIndex": dki, "dWeights": dw,
            "loss": np.array([loss], np.float32)}


def softmax_stats_full(q, k, qr, kr, scale, act_q=None, act_k=None):
    """Dense causal softmax max/sum over all keys, [B,1,S1,N1] fp32 each.

    The forward statistics a dense flash attention would hand the indexer loss
    (``test_sli_grad_kl_loss_triton.py:80-116``, without its fp16 score rounding).
    """
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32)
    qr = np.asarray(qr, np.float32); kr = np.asarray(kr, np.float32)
    B, S1, N1, _ = q.shape
    S2 = k.shape[1]
    act_q = [S1] * B if act_q is None else [int(x) for x in act_q]
    act_k = [S2] * B if act_k is None else [int(x) for x in act_k]
    mx = np.full((B, 1, S1, N1), -np.inf, np.float32)
    sm = np.zeros((B, 1, S1, N1), np.float32)
    for b in range(B):
        for s1 in range(S1):
            if s1 >= act_q[b]:
                continue
            lim = min(max(act_k[b] - act_q[b] + s1 + 1, 0), S2)
            if lim <= 0:
                continue
            sc = (q[b, s1] @ k[b, :lim, 0].T + qr[b, s1] @ kr[b, :lim, 0].T) * np.float32(scale)
            m = sc.max(axis=1)
            mx[b, 0, s1] = m
            sm[b, 0, s1] = np.exp(sc - m[:, None]).sum(axis=1)
    return mx, sm
