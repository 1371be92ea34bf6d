"""Multi-rank host logic on CPU ranks (gloo, world_size 2): row sharding with the causal
length trick and the fp32 key-gradient all-reduce reproduce the single-rank result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsa_triton_ascend_b200.sharding import shard_act_q, shard_rows


def test_shard_rows_balances_pairs():
    pairs = np.minimum(np.arange(1, 8193), 2048)
    for world in (1, 2, 4, 8):
        bounds = [shard_rows(pairs, world, r) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == len(pairs)
        assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))
        share = [pairs[a:b].sum() for a, b in bounds]
        assert max(share) - min(share) <= 2048
        # with a per-row cost the rank of the short causal rows takes fewer of them
        from dsa_triton_ascend_b200.sharding import SFA_ROW_COST
        cb = [shard_rows(pairs, world, r, row_cost=SFA_ROW_COST) for r in range(world)]
        assert cb[0][0] == 0 and cb[-1][1] == len(pairs)
        assert all(cb[i][1] == cb[i + 1][0] for i in range(world - 1))
        cost = [pairs[a:b].sum() + SFA_ROW_COST * (b - a) for a, b in cb]
        assert max(cost) - min(cost) <= 2 * (2048 + SFA_ROW_COST)   # a row at each end
        if world > 1:
            assert cb[0][1] - cb[0][0] < bounds[0][1] - bounds[0][0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import inputs as I
    from oracle import sfa
    c = I.sfa_case(*case)
    S1 = c["q"].shape[1]
    pairs = (c["si"][0, :, 0] >= 0).sum(axis=-1)
    r0, r1 = shard_rows(pairs, world, rank)
    aq = [shard_act_q(S1, r0)]
    sl = slice(r0, r1)
    out, mx, sm = sfa.sfa_fwd(c["q"][:, sl], c["k"], c["qr"][:, sl], c["kr"], c["si"][:, sl],
                              c["scale"], act_q=aq, sparse_mode=3)
    dq, dk, dv, dqr, dkr = sfa.sfa_bwd(c["q"][:, sl], c["k"], c["qr"][:, sl], c["kr"],
                                       c["si"][:, sl], c["dout"][:, sl], out, mx, sm, c["scale"],
                                       act_q=aq, sparse_mode=3, dtype="fp32")
    grads = [torch.from_numpy(np.ascontiguousarray(x)) for x in (dk, dv, dkr)]
    for g in grads:
        dist.all_reduce(g)
    parts = [torch.from_numpy(np.ascontiguousarray(x)) for x in (out, dq)]
    gathered = [[torch.zeros(0)] * world for _ in parts]
    for i, p in enumerate(parts):
        dist.all_gather_object(gathered[i], p)
    if rank == 0:
        out_q.put((torch.cat(gathered[0], dim=1).numpy(), torch.cat(gathered[1], dim=1).numpy(),
                   [g.numpy() for g in grads]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_stream_chunks_cover_rows_equally():
    """Host-streamed fwd+bwd: chunks of equal rows (the copies bound the step), 8 to 16."""
    from dsa_triton_ascend_b200.streaming import default_chunks
    assert default_chunks(8192) == 16 and default_chunks(1024) == 8 and default_chunks(64) == 8
    assert default_chunks(6144) == 12 and default_chunks(1 << 20) == 16
    for S1, n in [(8192, 32), (1000, 8), (5, 8)]:
        ones = np.ones(S1, dtype=np.int64)
        b = [shard_rows(ones, n, c) for c in range(n)]
        assert b[0][0] == 0 and b[-1][1] == S1
        assert all(b[c][1] == b[c + 1][0] for c in range(n - 1))
        sizes = [r1 - r0 for r0, r1 in b]
        assert max(sizes) - min(sizes) <= 1


def test_two_rank_fwd_bwd_matches_single_rank():
    case = (1, 12, 64, 4, 128, 16, 1, 3, "fp32", 5)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    out, dq, grads = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import inputs as I
    from oracle import sfa
    c = I.sfa_case(*case)
    ro, rm, rs = sfa.sfa_fwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["scale"], sparse_mode=3)
    rdq, rdk, rdv, _, rdkr = sfa.sfa_bwd(c["q"], c["k"], c["qr"], c["kr"], c["si"], c["dout"], ro,
                                         rm, rs, c["scale"], sparse_mode=3, dtype="fp32")
    np.testing.assert_allclose(out, ro, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dq, rdq, rtol=1e-5, atol=1e-6)
    for g, r in zip(grads, (rdk, rdv, rdkr)):
        np.testing.assert_allclose(g, r, rtol=1e-4, atol=1e-5)


def test_cpulist_parsing_and_binding_without_gpu():
    from dsa_triton_ascend_b200.streaming import _parse_cpulist, bind_host_to_device
    assert _parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert _parse_cpulist("") == set()
    if not torch.cuda.is_available():
        before = os.sched_getaffinity(0)
        assert bind_host_to_device() is False
        assert os.sched_getaffinity(0) == before


def _sli_worker(rank, world, port, case, out_q):
    """One rank: the indexer KL-loss gradient of its causal row shard (oracle), then the
    all-reduce of the fp32 dKeyIndex accumulator and the loss."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import inputs as I
    from oracle import sli
    c = I.sli_case(*case)
    S1 = c["q"].shape[1]
    topk = c["si"].shape[-1]
    S2 = c["k"].shape[1]
    pairs = np.minimum(topk, np.maximum(S2 - S1 + np.arange(S1) + 1, 0))
    r0, r1 = shard_rows(pairs, world, rank)
    sl = slice(r0, r1)
    mx, sm = sli.softmax_stats_full(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
    r = sli.sli_grad(c["q"][:, sl], c["k"], c["qr"][:, sl], c["kr"], c["qi"][:, sl], c["ki"],
                     c["w"][:, sl], c["si"][:, sl], mx[:, :, sl], sm[:, :, sl], c["scale"],
                     act_q=[shard_act_q(S1, r0)])
    buf = torch.from_numpy(np.concatenate([r["dKeyIndex"].ravel(), r["loss"].ravel()]).astype(np.float32))
    dist.all_reduce(buf)
    dqi = [torch.zeros(0)] * world
    dist.all_gather_object(dqi, torch.from_numpy(r["dQueryIndex"]))
    if rank == 0:
        out_q.put((buf.numpy(), torch.cat(dqi, dim=1).numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sli_matches_single_rank():
    """Config-5 style sharding of the indexer KL loss: S1 split into two causal row ranges,
    dKeyIndex and the loss summed by an all-reduce, dQueryIndex gathered."""
    case = (1, 10, 40, 8, 128, 4, 128, 16, "causal_random", "fp32", 9)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sli_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    buf, dqi = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import inputs as I
    from oracle import sli
    c = I.sli_case(*case)
    mx, sm = sli.softmax_stats_full(c["q"], c["k"], c["qr"], c["kr"], c["scale"])
    ref = sli.sli_grad(c["q"], c["k"], c["qr"], c["kr"], c["qi"], c["ki"], c["w"], c["si"], mx, sm,
                       c["scale"])
    nk = ref["dKeyIndex"].size
    np.testing.assert_allclose(buf[:nk].reshape(ref["dKeyIndex"].shape), ref["dKeyIndex"],
                               rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(buf[nk], ref["loss"][0], rtol=1e-5)
    np.testing.assert_allclose(dqi, ref["dQueryIndex"], rtol=1e-5, atol=1e-6)
