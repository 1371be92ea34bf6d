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
