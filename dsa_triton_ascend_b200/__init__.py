"""B200 (sm_100a) implementation of the DeepSeek Sparse Attention hot path.

Drop-in for the operators of 18851871668/dsa_triton_ascend, on CUDA torch tensors:

* :func:`sparse_flash_attention_triton` / :class:`SparseFlashAttentionTriton`
* :func:`sparse_flash_attention_grad_triton` / :class:`SparseFlashAttentionGradTriton`
"""
from ._lib import check_device_errors, lib as _load_library  # noqa: F401
from .sparse_flash_attention import (  # noqa: F401
    SparseFlashAttentionTriton,
    sparse_flash_attention_triton,
)
from .sparse_flash_attention_grad import (  # noqa: F401
    SparseFlashAttentionGradTriton,
    sparse_flash_attention_grad_partial,
    sparse_flash_attention_grad_triton,
)

__all__ = [
    "sparse_flash_attention_triton",
    "SparseFlashAttentionTriton",
    "sparse_flash_attention_grad_triton",
    "SparseFlashAttentionGradTriton",
    "check_device_errors",
]
