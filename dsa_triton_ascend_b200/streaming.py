"""Forward + backward of sparse flash attention for inputs that live in host memory.

A caller whose activations are kept in (pinned) host memory -- CPU offload of a long
prefill, or a data pipeline that hands over host tensors -- would otherwise copy every
input to the GPU, run the forward and backward, and copy every result back, one after the
other; at config-4 sizes the copies (about 4.7 GB) take longer than the kernels.
:func:`sfa_fwd_bwd_from_host` splits the query rows into chunks and runs three streams:
host-to-device copies of chunk i+1, the forward and backward kernels of chunk i, and
device-to-host copies of chunk i-1's results. The copies, not the kernels, bound the step
(every row moves its query, query_rope and dO in and its output, dq and dq_rope out: about
570 KB a row at N1 = 128, D = 512, against a few microseconds of kernel time), so chunks
hold equal numbers of rows. More chunks shorten the pipeline's fill and drain (the first
chunk's input copies and the last chunk's kernels and output copies, which nothing
overlaps) but each costs about half a millisecond of launches and allocations; about 512
rows a chunk, 8 to 16 chunks, measured best at config-4 sizes (65 ms a step against 68 ms
for 8 chunks balanced by valid pairs and 71 ms for 32 chunks, on 55 GB/s H2D and 51 GB/s
D2H PCIe links). The key
gradients of all chunks of a batch are added into one set of fp32 accumulators
(``accumulate`` in the C ABI) and cast once after the batch's last chunk.

A contiguous row range [r0, r1) of one batch of a causal (sparse_mode 3) BSND query is
itself a BSND query of r1 - r0 rows with actual query length S1 - r0 (the kernels' window
act_k - act_q + s1 + 1 is unchanged); in sparse_mode 0 the window does not depend on the
row, so the chunk's own length is passed.
"""
from __future__ import annotations

import numpy as np
import torch

from .sharding import shard_rows
from .sparse_flash_attention import sparse_flash_attention_triton
from .sparse_flash_attention_grad import sparse_flash_attention_grad_partial


def _parse_cpulist(text: str):
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-")
            cpus.update(range(int(lo), int(hi) + 1))
        else:
            cpus.add(int(part))
    return cpus


def bind_host_to_device(device=None) -> bool:
    """Run this process on the CPUs next to ``device``'s PCIe root (Linux sysfs).

    Pinned host buffers are placed on the NUMA node of the thread that first touches them,
    and every host<->device copy crosses from that node to the GPU; a rank whose buffers sit
    on the far socket pays the inter-socket link on every byte. Call this before allocating
    the pinned buffers of :func:`sfa_fwd_bwd_from_host` (one process per GPU). Returns False
    (and changes nothing) where the topology is not visible."""
    import os
    try:
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        prop = torch.cuda.get_device_properties(dev)
        bus = "%04x:%02x:%02x.0" % (prop.pci_domain_id, prop.pci_bus_id, prop.pci_device_id)
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
            cpus = _parse_cpulist(f.read()) & set(os.sched_getaffinity(0))
        if not cpus:
            return False
        os.sched_setaffinity(0, cpus)
        return True
    except (OSError, ValueError, AttributeError, RuntimeError, AssertionError):
        return False


def default_chunks(S1: int) -> int:
    """Chunks of about 512 rows, at least 8 and at most 16."""
    return max(8, min(16, S1 // 512))


def host_outputs(query, key, query_rope, key_rope):
    """Pinned host buffers for the results of :func:`sfa_fwd_bwd_from_host`."""
    pin = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    return (pin(query), pin(query), pin(key), pin(key), pin(query_rope), pin(key_rope))


def sfa_fwd_bwd_from_host(query, key, sparse_indices, d_out, scale_value, query_rope, key_rope,
                          sparse_mode: int = 3, chunks=None, device=None, host_out=None,
                          actual_seq_length_query=None, reduce_key_grads=None):
    """Sparse flash attention forward and backward of BSND host tensors, streamed.

    query [B,S1,N1,D], query_rope [B,S1,N1,64], key [B,S2,1,D], key_rope [B,S2,1,64],
    sparse_indices [B,S1,1,K] int32 and d_out [B,S1,N1,D] are CPU tensors (pin them, or the
    copies cannot overlap the kernels); value = key (MLA-absorb), the key length is S2 and
    the query length ``actual_seq_length_query`` (default S1; S1_total - r0 for rows
    [r0, r0 + S1) of a longer causal query, as in a multi-GPU shard).  Returns host tensors
    ``(out, dq, dk, dv, dq_rope, dk_rope)``, the values of sparse_flash_attention_triton and
    sparse_flash_attention_grad_triton on the same inputs; pass ``host_out`` (from
    :func:`host_outputs`) to reuse pinned buffers; ``chunks`` sets the number of row chunks
    (default :func:`default_chunks`).  ``reduce_key_grads(accs)``, if given, is
    called with each batch's fp32 key-gradient accumulators before their cast (e.g. an
    all-reduce across the ranks that share the keys).
    Asynchronous like a non_blocking copy: the results are complete once the caller's
    current stream, which is made to wait for the last copy, has been synchronised.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if query.dim() != 4 or tuple(d_out.shape) != tuple(query.shape) or sparse_indices.dim() != 4:
        raise ValueError("BSND host tensors expected")
    if sparse_mode not in (0, 3):
        raise ValueError("sparse_mode must be 0 or 3")
    B, S1, N1, D = query.shape
    if host_out is None:
        host_out = host_outputs(query, key, query_rope, key_rope)
    h_out, h_dq, h_dk, h_dv, h_dqr, h_dkr = host_out

    compute = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    # Stream bookkeeping for the caching allocator: a block is reused only after every
    # stream that touched it has passed the use. Inputs are allocated on the copy stream
    # and read by the kernels; results are allocated on the kernel stream and read by the
    # device-to-host copies.
    def used_by(stream, *ts):
        for t in ts:
            t.record_stream(stream)
    h2d.wait_stream(compute)        # earlier work of the caller on these buffers
    with torch.cuda.stream(h2d):
        k_d = key.to(dev, non_blocking=True)
        kr_d = key_rope.to(dev, non_blocking=True)
    compute.wait_stream(h2d)
    used_by(compute, k_d, kr_d)
    act_q = S1 if actual_seq_length_query is None else int(actual_seq_length_query)
    chunks = default_chunks(S1) if chunks is None else int(chunks)
    if chunks < 1:
        raise ValueError("chunks must be >= 1")
    rows = np.ones(S1, dtype=np.int64)      # equal rows: the copies bound the step
    bounds = [shard_rows(rows, chunks, c) for c in range(chunks)]
    for b in range(B):
        kb, krb = k_d[b:b + 1], kr_d[b:b + 1]
        accs = None
        finish = None
        for r0, r1 in bounds:
            if r1 <= r0:
                continue
            with torch.cuda.stream(h2d):
                q_d = query[b:b + 1, r0:r1].to(dev, non_blocking=True)
                qr_d = query_rope[b:b + 1, r0:r1].to(dev, non_blocking=True)
                si_d = sparse_indices[b:b + 1, r0:r1].to(dev, non_blocking=True)
                do_d = d_out[b:b + 1, r0:r1].to(dev, non_blocking=True)
            compute.wait_stream(h2d)
            used_by(compute, q_d, qr_d, si_d, do_d)
            aq = [act_q - r0] if sparse_mode == 3 else [r1 - r0]
            o, m, s_ = sparse_flash_attention_triton(
                q_d, kb, kb, si_d, scale_value, actual_seq_lengths_query=aq, query_rope=qr_d,
                key_rope=krb, sparse_mode=sparse_mode, return_softmax_lse=True)
            accs, finish = sparse_flash_attention_grad_partial(
                q_d, kb, kb, si_d, do_d, o, m, s_, scale_value, query_rope=qr_d, key_rope=krb,
                actual_seq_lengths_query=aq, sparse_mode=sparse_mode, accumulators=accs)
            dq, dqr = finish.query_grads
            d2h.wait_stream(compute)
            with torch.cuda.stream(d2h):
                h_out[b:b + 1, r0:r1].copy_(o, non_blocking=True)
                h_dq[b:b + 1, r0:r1].copy_(dq, non_blocking=True)
                h_dqr[b:b + 1, r0:r1].copy_(dqr, non_blocking=True)
            used_by(d2h, o, dq, dqr)
        if finish is not None:
            if reduce_key_grads is not None:
                reduce_key_grads(accs)
            _, dk, dv, _, dkr = finish()
            d2h.wait_stream(compute)
            with torch.cuda.stream(d2h):
                h_dk[b:b + 1].copy_(dk, non_blocking=True)
                h_dv[b:b + 1].copy_(dv, non_blocking=True)
                h_dkr[b:b + 1].copy_(dkr, non_blocking=True)
            used_by(d2h, dk, dv, dkr)
    compute.wait_stream(d2h)
    return h_out, h_dq, h_dk, h_dv, h_dqr, h_dkr
