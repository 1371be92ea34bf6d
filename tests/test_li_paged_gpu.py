"""Lightning indexer over a paged key cache (``lightning_indexer_paged``) on the B200 (GPU).

The reference's indexer rejects ``block_table`` (lightning_indexer_triton.py:497-498), so
there is no reference output for this layout. The paged call must give exactly what the
dense operator gives for the same keys laid out contiguously: each score is one dot product
per (key, head) whatever tile the key lands in, so indices and values are compared bit for
bit, across page sizes that split a 128-key tile into several blocks or take several tiles
from one block. Rows longer than shared memory holds (decode-length caches) take the top-k
path that reads the score matrix from global memory; those are also checked against fp32
scores computed by torch under the build's top-k rule.
"""
import numpy as np
import pytest
import torch

from test_li_gpu import check_topk

pytestmark = pytest.mark.gpu


def _inputs(B, S1, S2, N1, D, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn(B, S1, N1, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, S2, 1, D, generator=g, device="cuda").bfloat16()
    w = torch.randn(B, S1, N1, generator=g, device="cuda") / 8
    return q, k, w


def _page(k, page, spare=3, seed=0):
    """Scatter dense keys [B, S2, 1, D] into a shuffled block pool; returns (pool, table)."""
    B, S2, N2, D = k.shape
    nb = S2 // page
    rng = np.random.default_rng(seed)
    perm = rng.permutation(B * nb + spare)
    table = torch.as_tensor(perm[:B * nb].reshape(B, nb).astype(np.int32), device="cuda")
    pool = torch.zeros(B * nb + spare, page, N2, D, dtype=k.dtype, device="cuda")
    pool[table.reshape(-1).long()] = k.reshape(B * nb, page, N2, D)
    return pool, table


@pytest.mark.parametrize("page", [16, 64, 128, 256])
@pytest.mark.parametrize("mode", [0, 3])
def test_li_paged_matches_dense(page, mode):
    import dsa_triton_ascend_b200 as dsa
    B, S1, S2, N1, D, K = 2, 5, 1024, 64, 128, 256
    q, k, w = _inputs(B, S1, S2, N1, D, seed=page + mode)
    lens_k = [700, 1024]
    pool, table = _page(k, page, seed=page)
    ref_i, ref_v = dsa.lightning_indexer_triton(q, k, w, actual_seq_lengths_key=lens_k,
                                                sparse_count=K, sparse_mode=mode, return_value=True)
    got_i, got_v = dsa.lightning_indexer_paged(q, pool, w, table, actual_seq_lengths_key=lens_k,
                                               sparse_count=K, sparse_mode=mode, return_value=True)
    dsa.check_device_errors()
    assert torch.equal(got_i, ref_i)
    assert torch.equal(got_v, ref_v)
    assert int((got_i >= 0).sum()) > 0


def test_li_paged_tnd_query():
    """TND queries (cumulative lengths) against a paged cache, vs the dense TND call."""
    import dsa_triton_ascend_b200 as dsa
    B, S2, N1, D, K = 2, 512, 32, 128, 128
    q, k, w = _inputs(B, 6, S2, N1, D, seed=11)
    lens_q = [4, 6]
    q_t = torch.cat([q[b, :lens_q[b]] for b in range(B)])
    w_t = torch.cat([w[b, :lens_q[b]] for b in range(B)])
    k_t = k.reshape(B * S2, 1, D)
    pool, table = _page(k, 64, seed=3)
    cum_q, cum_k = list(np.cumsum(lens_q)), [S2, 2 * S2]
    ref_i, ref_v = dsa.lightning_indexer_triton(q_t, k_t, w_t, actual_seq_lengths_query=cum_q,
                                                actual_seq_lengths_key=cum_k, layout_query="TND",
                                                layout_key="TND", sparse_count=K, return_value=True)
    got_i, got_v = dsa.lightning_indexer_paged(q_t, pool, w_t, table, actual_seq_lengths_query=cum_q,
                                               layout_query="TND", sparse_count=K, return_value=True)
    dsa.check_device_errors()
    assert got_i.shape == ref_i.shape == (10, 1, K)
    assert torch.equal(got_i, ref_i) and torch.equal(got_v, ref_v)


def test_li_paged_decode_long_rows():
    """Decode shape (one query token per sequence) over 56k-key caches: the score rows do not
    fit in shared memory, so the top-k reads them from global memory. Paged equals dense,
    and the selection agrees with fp32 scores computed by torch."""
    import dsa_triton_ascend_b200 as dsa
    B, N1, D, K, page, nb = 2, 64, 128, 2048, 128, 448
    S2 = page * nb
    q, k, w = _inputs(B, 1, S2, N1, D, seed=21)
    lens_k = [40000, S2 - 300]
    pool, table = _page(k, page, seed=5)
    ref_i, ref_v = dsa.lightning_indexer_triton(q, k, w, actual_seq_lengths_key=lens_k,
                                                sparse_count=K, sparse_mode=0, return_value=True)
    got_i, got_v = dsa.lightning_indexer_paged(q, pool, w, table, actual_seq_lengths_key=lens_k,
                                               sparse_count=K, sparse_mode=0, return_value=True)
    dsa.check_device_errors()
    assert torch.equal(got_i, ref_i) and torch.equal(got_v, ref_v)
    for b in range(B):
        sc = torch.einsum("gd,sd->gs", q[b, 0].float(), k[b, :, 0].float()).relu()
        sc = (sc * w[b, 0].float()[:, None]).sum(0)
        sc[lens_k[b]:] = -float("inf")
        check_topk(got_i[b, 0].cpu().numpy(), got_v[b, 0].float().cpu().numpy(),
                   sc.double().cpu().numpy()[None], K, what=f"decode b{b}")
