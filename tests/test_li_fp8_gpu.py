"""FP8 lightning indexer (``lightning_indexer_fp8``) on the B200 (GPU).

No counterpart in the reference (its indexer is bf16 / fp16); the scores are
key_scale * sum_g ReLU(q_g . k) * w_g on e4m3 query and key. Checked against fp32 scores
computed by torch from the dequantised fp8 values under the build's top-k rule (indices
exact except within 1e-5 of the k-th score), and the paged call against the dense one bit
for bit.
"""
import numpy as np
import pytest
import torch

from test_li_gpu import check_topk

pytestmark = pytest.mark.gpu
FP8 = torch.float8_e4m3fn


def _inputs(B, S1, S2, N1, D, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = (torch.randn(B, S1, N1, D, generator=g, device="cuda") * 2).to(FP8)
    k = (torch.randn(B, S2, 1, D, generator=g, device="cuda") * 2).to(FP8)
    ks = torch.rand(B, S2, 1, generator=g, device="cuda") * 1.5 + 0.25
    w = torch.randn(B, S1, N1, generator=g, device="cuda") / 8
    return q, k, ks, w


def _ref_scores(q, k, ks, w, mode):
    B, S1, N1, D = q.shape
    S2 = k.shape[1]
    sc = torch.einsum("bsgd,btd->bsgt", q.float(), k[:, :, 0].float()).relu()
    sc = (sc * w[..., None]).sum(2) * ks[:, None, :, 0]          # [B, S1, S2]
    if mode == 3:
        s1 = torch.arange(S1, device="cuda")[:, None]
        s2 = torch.arange(S2, device="cuda")[None, :]
        sc = torch.where(s2 < S2 - S1 + s1 + 1, sc, torch.full_like(sc, -float("inf")))
    return sc


@pytest.mark.parametrize("mode", [0, 3])
@pytest.mark.parametrize("N1,D", [(64, 128), (32, 256)])
def test_li_fp8_matches_fp32_scores(mode, N1, D):
    import dsa_triton_ascend_b200 as dsa
    B, S1, S2, K = 2, 40, 1024, 256
    q, k, ks, w = _inputs(B, S1, S2, N1, D, seed=N1 + mode)
    idx, val = dsa.lightning_indexer_fp8(q, k, ks, w, sparse_count=K, sparse_mode=mode,
                                         return_value=True)
    dsa.check_device_errors()
    assert idx.shape == (B, S1, 1, K) and val.dtype == torch.float32
    sc = _ref_scores(q, k, ks, w, mode)
    check_topk(idx.cpu().numpy(), val.cpu().numpy(), sc.double().cpu().numpy(), K, what=f"fp8 mode{mode}")


def test_li_fp8_paged_matches_dense():
    import dsa_triton_ascend_b200 as dsa
    B, S1, S2, N1, D, K, page = 2, 3, 2048, 64, 128, 512, 64
    q, k, ks, w = _inputs(B, S1, S2, N1, D, seed=9)
    nb = S2 // page
    perm = torch.as_tensor(np.random.default_rng(1).permutation(B * nb + 2), device="cuda")
    table = perm[:B * nb].reshape(B, nb).to(torch.int32)
    pool = torch.zeros(B * nb + 2, page, 1, D, device="cuda").to(FP8)
    pool_s = torch.zeros(B * nb + 2, page, 1, device="cuda")
    pool[table.reshape(-1).long()] = k.reshape(B * nb, page, 1, D)
    pool_s[table.reshape(-1).long()] = ks.reshape(B * nb, page, 1)
    lens = [1500, S2]
    ref = dsa.lightning_indexer_fp8(q, k, ks, w, actual_seq_lengths_key=lens, sparse_count=K,
                                    sparse_mode=0, return_value=True)
    got = dsa.lightning_indexer_fp8(q, pool, pool_s, w, actual_seq_lengths_key=lens,
                                    block_table=table, sparse_count=K, sparse_mode=0,
                                    return_value=True)
    dsa.check_device_errors()
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    assert int((got[0] >= 0).sum()) == B * S1 * K
