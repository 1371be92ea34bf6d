"""Generate the golden fixtures under tests/golden/ from the reference's own numpy goldens.

Usage (needs a checkout of the reference project; it is not needed afterwards):

    python tests/golden/gen_golden.py --reference <path-to-dsa_triton_ascend>

It imports, unmodified, the reference files
  sparse_flash_attention_numpy.py       (SFA forward golden)
  sparse_flash_attention_grad_numpy.py  (SFA backward golden)
  sli_grad_kl_loss_numpy.py             (indexer KL-loss gradient golden)
runs them on the seeded inputs of ``inputs.py`` and stores their outputs (bf16/fp16
results as raw 16-bit patterns, fp32 statistics as fp32) in ``*.npz`` files.  The
inputs themselves are not stored: tests regenerate them from the same seeds.

``sli_grad_kl_loss_numpy.py`` imports mindspore at module level only to call
``set_context``; a stub module satisfies that import.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as I  # noqa: E402

# (name, B, S1, S2, N1, D, count, block, mode, dtype, seed)
SFA_FWD_CASES = [
    ("fwd_tok_m3_d512_bf16", 1, 4, 128, 8, 512, 64, 1, 3, "bf16", 1),
    ("fwd_tok_m0_d512_bf16", 1, 4, 128, 8, 512, 64, 1, 0, "bf16", 2),
    ("fwd_multibatch_d512_fp16", 2, 16, 256, 16, 512, 128, 1, 3, "fp16", 3),
    ("fwd_blk2_d256_bf16", 1, 8, 128, 8, 256, 32, 2, 3, "bf16", 4),
    ("fwd_blk4_d128_fp16", 1, 8, 256, 16, 128, 32, 4, 3, "fp16", 5),
    ("fwd_s1_1_d128_bf16", 1, 1, 128, 8, 128, 16, 1, 3, "bf16", 6),
    ("fwd_n1_128_d512_bf16", 1, 2, 256, 128, 512, 128, 1, 3, "bf16", 7),
    ("fwd_n1_1_d512_bf16", 1, 4, 128, 1, 512, 64, 1, 3, "bf16", 8),
]

SFA_BWD_CASES = [
    ("bwd_tok_m3_d512_bf16", 1, 4, 128, 8, 512, 64, 1, 3, "bf16", 11),
    ("bwd_tok_m0_d256_fp16", 1, 4, 128, 8, 256, 64, 1, 0, "fp16", 12),
    ("bwd_multibatch_d512_bf16", 2, 8, 128, 16, 512, 64, 1, 3, "bf16", 13),
    ("bwd_blk2_d128_bf16", 1, 8, 128, 8, 128, 16, 2, 3, "bf16", 14),
    ("bwd_n1_64_d512_bf16", 1, 2, 128, 64, 512, 64, 1, 3, "bf16", 15),
    ("bwd_blk4_d256_bf16", 1, 8, 256, 16, 256, 24, 4, 3, "bf16", 16),
]

# (name, B, S1, S2, N1, D, Nidx1, Di, topK, pattern, seed)
SLI_CASES = [
    ("sli_causal_random", 1, 4, 256, 16, 512, 8, 128, 64, "causal_random", 21),
    ("sli_continuous", 1, 4, 256, 16, 512, 8, 128, 64, "continuous", 22),
    ("sli_repeated", 1, 4, 256, 16, 512, 8, 128, 64, "repeated", 23),
    ("sli_n1_32_k128", 1, 3, 512, 32, 512, 16, 128, 128, "causal_random", 24),
]

# Lightning-indexer score pins: the SLI golden's stage-1 scores I_scores
# (sli_grad_kl_loss_numpy.py:64-76) with index rows that list every visible key
# ("causal_continuous", topK = S2), i.e. the indexer's score of every visible key.
# (name, B, S1, S2, N1, D, Nidx1, Di, seed); the SLI inputs are generated in fp16.
LI_SCORE_CASES = [
    ("li_scores_n8_d128", 1, 4, 128, 16, 512, 8, 128, 31),
    ("li_scores_n64_d128", 1, 3, 96, 16, 512, 64, 128, 32),
]

CONFIG1_ROWS = list(range(0, 128, 8))


def bits16(x, dtype):
    """fp32 values exactly representable in dtype -> their uint16 bit patterns."""
    x = np.asarray(x, np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).view(np.uint16)
    return (x.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def np_dtype(golden_mod, dtype):
    return golden_mod.BF16 if dtype == "bf16" else np.float16


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference project checkout")
    ap.add_argument("--only", nargs="*", default=None,
                    help="write only the fixtures with these names (default: all)")
    args = ap.parse_args()
    want = (lambda n: True) if not args.only else (lambda n: n in args.only)
    sys.path.insert(0, os.path.abspath(args.reference))
    stub = types.ModuleType("mindspore")
    stub.GRAPH_MODE, stub.PYNATIVE_MODE = 0, 1
    stub.set_context = lambda *a, **k: None
    sys.modules.setdefault("mindspore", stub)

    import sparse_flash_attention_numpy as fwd_g
    import sparse_flash_attention_grad_numpy as bwd_g
    import sli_grad_kl_loss_numpy as sli_g

    for name, B, S1, S2, N1, D, cnt, blk, mode, dt, seed in SFA_FWD_CASES:
        if not want(name):
            continue
        c = I.sfa_case(B, S1, S2, N1, D, cnt, blk, mode, dt, seed)
        out, mx, sm = fwd_g.sparse_flash_attention_golden_bsnd(
            c["q"], c["k"], c["k"], c["si"], c["qr"], c["kr"], c["scale"],
            [S1] * B, [S2] * B, sparse_block_size=blk, sparse_mode=mode,
            return_softmax_lse=True, dtype=np_dtype(fwd_g, dt))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), out=bits16(out, dt),
                            softmax_max=mx, softmax_sum=sm)
        print("wrote", name)

    if want("config1"):
        c = I.config1()
        out, mx, sm = fwd_g.sparse_flash_attention_golden_bsnd(
            c["q"], c["k"], c["k"], c["si"], c["qr"], c["kr"], c["scale"], [128], [2048],
            sparse_block_size=1, sparse_mode=3, return_softmax_lse=True, dtype=fwd_g.BF16)
        np.savez_compressed(os.path.join(HERE, "config1.npz"),
                            rows=np.array(CONFIG1_ROWS, np.int32),
                            out_rows=bits16(out[:, CONFIG1_ROWS], "bf16"),
                            softmax_max=mx, softmax_sum=sm)
        print("wrote config1")

    for name, B, S1, S2, N1, D, cnt, blk, mode, dt, seed in SFA_BWD_CASES:
        if not want(name):
            continue
        c = I.sfa_case(B, S1, S2, N1, D, cnt, blk, mode, dt, seed)
        out, mx, sm = fwd_g.sparse_flash_attention_golden_bsnd(
            c["q"], c["k"], c["k"], c["si"], c["qr"], c["kr"], c["scale"],
            [S1] * B, [S2] * B, sparse_block_size=blk, sparse_mode=mode,
            return_softmax_lse=True, dtype=np_dtype(fwd_g, dt))
        dq, dk, dv, dqr, dkr = bwd_g.sparse_flash_attention_grad_golden_bsnd(
            c["q"], c["k"], c["k"], c["si"], c["dout"], out, mx, sm, c["qr"], c["kr"],
            c["scale"], [S1] * B, [S2] * B, sparse_block_size=blk, sparse_mode=mode,
            dtype=np_dtype(fwd_g, dt))
        np.savez_compressed(os.path.join(HERE, name + ".npz"),
                            out=bits16(out, dt), softmax_max=mx, softmax_sum=sm,
                            dq=bits16(dq, dt), dk=bits16(dk, dt), dv=bits16(dv, dt),
                            dqr=bits16(dqr, dt), dkr=bits16(dkr, dt))
        print("wrote", name)

    for name, B, S1, S2, N1, D, Nidx1, Di, topK, pat, seed in SLI_CASES:
        if not want(name):
            continue
        c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, topK, pat, "fp16", seed)
        mx, sm = sli_g._compute_sm_stats(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
        r = sli_g.numpy_reference(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"],
                                  c["w"], c["si"], mx, sm, c["scale"])
        np.savez_compressed(os.path.join(HERE, name + ".npz"), softmax_max=mx, softmax_sum=sm,
                            dQueryIndex=r["dQueryIndex"], dKeyIndex=r["dKeyIndex"],
                            dW=r["dW"], loss=r["loss"])
        print("wrote", name)

    for name, B, S1, S2, N1, D, Nidx1, Di, seed in LI_SCORE_CASES:
        if not want(name):
            continue
        c = I.sli_case(B, S1, S2, N1, D, Nidx1, Di, S2, "causal_continuous", "fp16", seed)
        mx, sm = sli_g._compute_sm_stats(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
        r = sli_g.numpy_reference(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"],
                                  c["w"], c["si"], mx, sm, c["scale"])
        np.savez_compressed(os.path.join(HERE, name + ".npz"), I_scores=r["I_scores"])
        print("wrote", name)


if __name__ == "__main__":
    main()
