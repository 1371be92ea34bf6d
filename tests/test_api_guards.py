"""Host-side guards raise the reference's errors before touching a GPU (CPU only).

Conditions mirror sparse_flash_attention_triton.py:529-586,
sparse_flash_attention_grad_triton.py:428-478, lightning_indexer_triton.py:497-521 and
sparse_lightning_indexer_grad_kl_loss_triton.py:534-538.
"""
import pytest
import torch

import dsa_triton_ascend_b200 as dsa


def t(*shape, dtype=torch.bfloat16):
    return torch.zeros(*shape, dtype=dtype)


def sfa_args():
    return (t(1, 2, 8, 512), t(1, 16, 1, 512), t(1, 16, 1, 512), t(1, 2, 1, 4, dtype=torch.int32))


@pytest.mark.parametrize("kw,msg", [
    (dict(attention_mode=1), "attention_mode"),
    (dict(pre_tokens=5), "pre_tokens"),
    (dict(sparse_mode=1), "sparse_mode"),
    (dict(query_rope=None), "rope"),
    (dict(sparse_block_size=3), "sparse_block_size"),
    (dict(sparse_block_size=256), "sparse_block_size"),
])
def test_sfa_fwd_guards(kw, msg):
    args = dict(query_rope=t(1, 2, 8, 64), key_rope=t(1, 16, 1, 64))
    args.update(kw)
    with pytest.raises(ValueError, match=msg):
        dsa.sparse_flash_attention_triton(*sfa_args(), **args)


def test_sfa_fwd_requires_cuda():
    with pytest.raises(ValueError, match="CUDA"):
        dsa.sparse_flash_attention_triton(*sfa_args(), query_rope=t(1, 2, 8, 64),
                                          key_rope=t(1, 16, 1, 64))


@pytest.mark.parametrize("kw,msg", [
    (dict(deterministic=True), "deterministic"),
    (dict(sparse_mode=2), "sparse_mode"),
    (dict(next_tokens=0), "pre_tokens"),
    (dict(key_rope=None), "rope"),
])
def test_sfa_bwd_guards(kw, msg):
    q, k, v, si = sfa_args()
    args = dict(query_rope=t(1, 2, 8, 64), key_rope=t(1, 16, 1, 64))
    args.update(kw)
    with pytest.raises(ValueError, match=msg):
        dsa.sparse_flash_attention_grad_triton(q, k, v, si, q, q, t(1, 1, 2, 8, dtype=torch.float32),
                                               t(1, 1, 2, 8, dtype=torch.float32), **args)


def test_li_guards():
    q, k, w = t(1, 4, 8, 64), t(1, 16, 1, 64), t(1, 4, 8, dtype=torch.float32)
    with pytest.raises(ValueError, match="block_table"):
        dsa.lightning_indexer_triton(q, k, w, block_table=t(1, 1, dtype=torch.int32))
    with pytest.raises(ValueError, match="sparse_mode"):
        dsa.lightning_indexer_triton(q, k, w, sparse_mode=1)


def test_sli_guards():
    q, k = t(1, 2, 8, 512), t(1, 16, 1, 512)
    qi, ki, w = t(1, 2, 4, 128), t(1, 16, 1, 128), t(1, 2, 4)
    si, mx = t(1, 2, 1, 8, dtype=torch.int32), t(1, 1, 2, 8, dtype=torch.float32)
    f = dsa.sparse_lightning_indexer_grad_kl_loss_triton
    with pytest.raises(ValueError, match="BSND"):
        f(q, k, qi, ki, w, si, mx, mx, layout="TND")
    with pytest.raises(ValueError, match="sparse_mode"):
        f(q, k, qi, ki, w, si, mx, mx, sparse_mode=0)
    with pytest.raises(AssertionError, match="Nidx2"):
        f(q, k, qi, ki, w, t(1, 2, 2, 8, dtype=torch.int32), mx, mx)


def test_modules_forward_to_functions():
    m = dsa.SparseFlashAttentionTriton(sparse_mode=7)
    with pytest.raises(ValueError, match="sparse_mode"):
        m(*sfa_args(), query_rope=t(1, 2, 8, 64), key_rope=t(1, 16, 1, 64))
    assert dsa.LightningIndexerTriton().sparse_mode == 3
    assert dsa.SparseFlashAttentionGradTriton().sparse_mode == 3


def _dense_args(**over):
    B, S1, S2, N1, N2, D, Ni, Di = 1, 2, 64, 32, 32, 128, 32, 128
    a = dict(query=t(B, S1, N1, D, dtype=torch.float16), key=t(B, S2, N2, D, dtype=torch.float16),
             query_index=t(B, S1, Ni, Di, dtype=torch.float16),
             key_index=t(B, S2, 1, Di, dtype=torch.float16), weights=t(B, S1, Ni, dtype=torch.float16),
             softmax_max=t(B, N2, S1, N1 // N2, dtype=torch.float32),
             softmax_sum=t(B, N2, S1, N1 // N2, dtype=torch.float32))
    a.update(over)
    return a


@pytest.mark.parametrize("over,exc,msg", [
    (dict(layout="TND"), ValueError, "BSND"),
    (dict(sparse_mode=0), ValueError, "sparse_mode"),
    (dict(query_index=t(1, 2, 48, 128, dtype=torch.float16),
          weights=t(1, 2, 48, dtype=torch.float16)), ValueError, "Nidx1"),
    (dict(key=t(1, 64, 32, 128, dtype=torch.bfloat16)), TypeError, "share dtype"),
    (dict(softmax_max=t(1, 32, 2, 1, dtype=torch.float16)), TypeError, "float32"),
    (dict(softmax_sum=t(1, 1, 2, 32, dtype=torch.float32)), ValueError, "softmax_max"),
    (dict(query_rope=t(1, 2, 32, 64, dtype=torch.float16)), ValueError, "both"),
    (dict(softmax_max_index=t(1, 1, 2, dtype=torch.float32)), ValueError, "both"),
])
def test_dense_loss_guards(over, exc, msg):
    """dense_loss_backward_triton.py:649-749, :785-791"""
    a = _dense_args(**{k: v for k, v in over.items() if k not in ("layout", "sparse_mode")})
    kw = {k: v for k, v in over.items() if k in ("layout", "sparse_mode")}
    with pytest.raises(exc, match=msg):
        dsa.dense_loss_backward_triton(**a, **kw)


def test_dense_lse_guards():
    qi, ki, w = t(1, 2, 32, 128), t(1, 64, 1, 128), t(1, 2, 32)
    with pytest.raises(ValueError, match="key_index"):
        dsa.dense_lightning_indexer_softmax_lse_triton(qi, t(1, 64, 2, 128), w)
    with pytest.raises(ValueError, match="D_idx"):
        dsa.dense_lightning_indexer_softmax_lse_triton(t(1, 2, 32, 64), t(1, 64, 1, 64), w)
    with pytest.raises(ValueError, match="CUDA"):
        dsa.dense_lightning_indexer_softmax_lse_triton(qi, ki, w)


def test_paged_indexer_guards():
    """lightning_indexer_paged: no counterpart in the reference; its own argument checks."""
    q, w = t(1, 2, 8, 128), t(1, 2, 8, dtype=torch.float32)
    bt = t(1, 4, dtype=torch.int32)
    with pytest.raises(ValueError, match="key_cache"):
        dsa.lightning_indexer_paged(q, t(64, 1, 128), w, bt)
    with pytest.raises(ValueError, match="block_table"):
        dsa.lightning_indexer_paged(q, t(4, 64, 1, 128), w, t(1, 4, dtype=torch.int64))
    with pytest.raises(ValueError, match="page_size"):
        dsa.lightning_indexer_paged(q, t(4, 96, 1, 128), w, bt)
    with pytest.raises(ValueError, match="sparse_mode"):
        dsa.lightning_indexer_paged(q, t(4, 64, 1, 128), w, bt, sparse_mode=1)
    with pytest.raises(ValueError, match="CUDA"):
        dsa.lightning_indexer_paged(q, t(4, 64, 1, 128), w, bt)


def test_fp8_indexer_guards():
    f8 = torch.float8_e4m3fn
    q, k = t(1, 2, 8, 128, dtype=f8), t(1, 64, 1, 128, dtype=f8)
    ks, w = t(1, 64, 1, dtype=torch.float32), t(1, 2, 8, dtype=torch.float32)
    with pytest.raises(ValueError, match="float8_e4m3fn"):
        dsa.lightning_indexer_fp8(t(1, 2, 8, 128), k, ks, w)
    with pytest.raises(ValueError, match="key_scale"):
        dsa.lightning_indexer_fp8(q, k, t(1, 64, dtype=torch.float32), w)
    with pytest.raises(ValueError, match="CUDA"):
        dsa.lightning_indexer_fp8(q, k, ks, w)


def test_indexer_score_row_cap():
    """Score rows hold at most 131,072 keys (the top-k kernel packs its counts)."""
    q, w = t(1, 2, 8, 128), t(1, 2, 8, dtype=torch.float32)
    with pytest.raises(ValueError, match="score row"):
        dsa.lightning_indexer_paged(q, t(4, 128, 1, 128), w, t(1, 1025, dtype=torch.int32))
    f8 = torch.float8_e4m3fn
    with pytest.raises(ValueError, match="score row"):
        dsa.lightning_indexer_fp8(t(1, 2, 8, 128, dtype=f8), t(1, 131073, 1, 128, dtype=f8),
                                  t(1, 131073, 1, dtype=torch.float32), w)
