"""B200 (sm_100a) implementation of the DeepSeek Sparse Attention hot path.

Drop-in for the operators of 18851871668/dsa_triton_ascend, on CUDA torch tensors:

* :func:`sparse_flash_attention_triton` / :class:`SparseFlashAttentionTriton`
* :func:`sparse_flash_attention_grad_triton` / :class:`SparseFlashAttentionGradTriton`
* :func:`lightning_indexer_triton` / :class:`LightningIndexerTriton`
* :func:`sparse_lightning_indexer_grad_kl_loss_triton` /
  :class:`SparseLightningIndexerGradKLLossTriton`

plus :func:`sfa_fwd_bwd_from_host` (forward + backward of host-resident inputs, with the
copies overlapped with the kernels), :func:`lightning_indexer_paged` (the indexer over a
paged key cache, which the reference's indexer rejects), :func:`lightning_indexer_fp8` (the
FP8 indexer), the dense indexer KL loss of
:mod:`.dense_indexer_loss` (``dense_loss_backward_triton`` and its softmax-LSE helper) and
the autograd functions of :mod:`.autograd`.
"""
from ._lib import check_device_errors, lib as _load_library  # noqa: F401
from .sparse_flash_attention import (  # noqa: F401
    SparseFlashAttentionTriton,
    sparse_flash_attention_triton,
)
from .lightning_indexer import (  # noqa: F401
    LightningIndexerTriton,
    lightning_indexer_fp8,
    lightning_indexer_paged,
    lightning_indexer_triton,
)
from .sparse_lightning_indexer_grad_kl_loss import (  # noqa: F401
    SparseLightningIndexerGradKLLossTriton,
    sparse_lightning_indexer_grad_kl_loss_partial,
    sparse_lightning_indexer_grad_kl_loss_triton,
)
from .sparse_flash_attention_grad import (  # noqa: F401
    SparseFlashAttentionGradTriton,
    sparse_flash_attention_grad_merged,
    sparse_flash_attention_grad_partial,
    sparse_flash_attention_grad_triton,
)
from .dense_indexer_loss import (  # noqa: F401
    DenseLightningIndexerGradKLLossTriton,
    DenseLightningIndexerSoftmaxLseTriton,
    DenseLossBackwardTriton,
    dense_lightning_indexer_grad_kl_loss_triton,
    dense_lightning_indexer_softmax_lse_triton,
    dense_loss_backward_triton,
    npu_dense_lightning_indexer_grad_kl_loss_triton,
    npu_dense_lightning_indexer_softmax_lse_triton,
)
from .streaming import bind_host_to_device, host_outputs, sfa_fwd_bwd_from_host  # noqa: F401
from .autograd import (  # noqa: F401
    IndexerKLLossFunction,
    SparseAttentionWithIndexer,
    SparseFlashAttentionFunction,
)

__all__ = [
    "sparse_flash_attention_triton",
    "SparseFlashAttentionTriton",
    "sparse_flash_attention_grad_triton",
    "SparseFlashAttentionGradTriton",
    "lightning_indexer_triton",
    "LightningIndexerTriton",
    "sparse_lightning_indexer_grad_kl_loss_triton",
    "SparseLightningIndexerGradKLLossTriton",
    "check_device_errors",
]
