#!/usr/bin/env python
"""Benchmark of the DSA hot path on B200: SFA forward + backward at BASELINE config 4.

Workload (one step): BSND, B=1, S1=S2=8192, N1=128, D=512+64 rope, topK=2048 distinct
causal key ids per query (-1 padded for early queries), sparse_mode=3, bf16 N(0,1)
activations, scale 1/sqrt(576).  With N GPUs the 8192 query rows are split into N
contiguous ranges balanced by valid (query, key) pairs; KV is replicated.  Strong
scaling: the job is the same at every N.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's numpy CPU
path (restated in ``oracle/``) on a bounded sample of query rows instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SFA fwd/bwd TFLOP/s + tokens/s at N1=128,D=576,topK=2048; % roofline"
S1 = S2 = 8192
N1, D, DR, TOPK = 128, 512, 64, 2048
FWD_FLOP_PER_PAIR = N1 * (2 * (D + DR) + 2 * D)              # QK^T + P V
BWD_FLOP_PER_PAIR = N1 * (3 * 2 * (D + DR) + 2 * 2 * D)        # S, dQ, dK (576) + dP, dV (512)
GATHER_BYTES_PER_PAIR = (D + DR) * 2                           # one bf16 key row
# backward, roofline bytes by the north-star definition (gathered bytes at HBM): the key row
# gathered twice, for the scores (K1) and for dQ (K2)
BWD_BYTES_PER_PAIR = 2 * GATHER_BYTES_PER_PAIR
# backward: the fp32 dK / dKr / dV scatter-add into accumulators that stay in L2 (35.7 MB at
# config 4), per reduced key row (a key that several rows of a row group select is reduced
# once);
# reported beside the roofline, not in it
BWD_SCATTER_BYTES_PER_KEY_ROW = 4 * (2 * D + DR)


def reduced_key_rows(si_rows, group=4):
    """Key rows the backward's fp32 scatter reduces in one 5-output call over these query
    rows ([rows, topk] ids, -1 = none): the library groups `group` adjacent rows of the call
    (four at D = 512 with top-2048; two in the merged key == value mode) and reduces a key the
    group's rows share once, so a group
    costs the size of the union of its rows' keys (the synthetic ids of a row are distinct)."""
    import torch
    R, K = si_rows.shape
    pad = (-R) % group
    if pad:
        si_rows = torch.cat([si_rows, si_rows.new_full((pad, K), -1)])
    G = si_rows.shape[0] // group
    s = torch.sort(si_rows.reshape(G, group * K), dim=1).values
    valid = s >= 0
    dup = (s[:, 1:] == s[:, :-1]) & valid[:, 1:]
    return int(valid.sum()) - int(dup.sum())
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per valid pair, from one
# `ncu --set full` capture of the last 256 query rows of config 4 (524,288 pairs; command and
# figures in profiles/sfa_kernels_config4_rows256_full.md), scaled to a launch by its pairs.
# Backward: K1 + K2 + the four-row group pass + K3, plus the delta kernel's read of dO and O
# (2 x N1 x D x 2 B a row).  Builds of the captures: the forward, K1 and K2 of commit cb19fcd;
# the group pass and K3 of commit a714e58 (profiles/sfa_bwd_dkv_reductions.md).
PROFILE_PAIRS = 524288
BWD_DRAM_BYTES_PER_PAIR = (103.11 + 218.89 + 146.14 + 19.40 + 2.14 + 392.66 + 15.62) * 1e6 / PROFILE_PAIRS
BWD_DRAM_BYTES_PER_ROW = 2 * N1 * D * 2
FWD_DRAM_BYTES_PER_PAIR = (49.35 + 1.95) * 1e6 / PROFILE_PAIRS
# DRAM traffic of one call of each secondary workload at the size bench.py runs, from one ncu
# capture of the library's kernels (profiles/secondary_workloads_traffic.md)
WORKLOAD_DRAM_BYTES = {
    "li": (138.45 + 52.63 + 67.75 + 49.59) * 1e6,            # score + top-k (profiles/li_score_topk_config2.md)
    "decode": (0.33 + 84.43 + 0.10 + 16.92) * 1e6,           # prep + forward + combine
    "sli": (1284.81 + 58.37 + 260.75 + 109.38 + 4.20) * 1e6,  # teacher + index + cast
    "dense": (1361.01 + 128.45 + 412.56 + 124.68) * 1e6,      # teacher + index (profiles/dense_indexer_loss_config5.md)
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        sm, smax = [], None
        for s in self.samples:
            try:
                sm.append(float(s[0]))
                smax = float(s[1])
            except ValueError:
                continue
            for n, v in zip(names, s[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------------------
# CPU side: the reference algorithm (numpy restatement) on a bounded sample of rows
# ----------------------------------------------------------------------------------------
def cpu_sample_tflops(seconds_budget: float = 10.0, rows: int = 2):
    """Time the numpy forward + backward (the reference algorithm, restated in oracle/) on
    `rows` query rows of config 4 with all 2048 keys valid, scaled by FLOPs.
    Returns (TFLOP/s, description, threads)."""
    from oracle import sfa as osfa
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, rows, N1, D), dtype=np.float32)
    qr = rng.standard_normal((1, rows, N1, DR), dtype=np.float32)
    k = rng.standard_normal((1, S2, 1, D), dtype=np.float32)
    kr = rng.standard_normal((1, S2, 1, DR), dtype=np.float32)
    do = rng.standard_normal((1, rows, N1, D), dtype=np.float32)
    si = np.stack([np.sort(rng.permutation(S2)[:TOPK]) for _ in range(rows)]).astype(np.int32)
    si = si.reshape(1, rows, 1, TOPK)
    sc = 1 / math.sqrt(576)
    t0 = time.perf_counter()
    n_done = 0
    while True:
        out, mx, sm = osfa.sfa_fwd(q, k, qr, kr, si, sc, act_q=[S2], act_k=[S2], sparse_mode=0)
        osfa.sfa_bwd(q, k, qr, kr, si, do, out, mx, sm, sc, act_q=[S2], act_k=[S2], sparse_mode=0)
        n_done += 1
        if time.perf_counter() - t0 > seconds_budget or n_done >= 50:
            break
    dt = (time.perf_counter() - t0) / n_done
    flops = rows * TOPK * (FWD_FLOP_PER_PAIR + BWD_FLOP_PER_PAIR)
    threads = torch.get_num_threads()
    return (flops / dt / 1e12,
            f"numpy SFA forward+backward, {rows} query rows x {TOPK} keys x {N1} heads", threads)


def run_reference(args, rank, world):
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_sample_tflops(seconds_budget=0.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, desc, threads = cpu_sample_tflops(seconds_budget=0.0)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = float(np.median(vals))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": wall / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config 4 SFA forward + backward, sampled rows (CPU)", "S1": S1, "S2": S2,
                   "N1": N1, "D": D + DR, "topK": TOPK},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------
# GPU side
# ----------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="sfa", choices=["sfa", "li", "li_fp8", "decode", "sli", "dense", "dsa_step"],
                    help="sfa: config 4 forward+backward (the headline); li: config 2 indexer; "
                         "li_fp8: config 2 geometry through the FP8 indexer (e4m3 query / key, "
                         "per-key scales); decode: config 3 paged forward; sli: config 5 "
                         "indexer KL-loss grad; dense: the dense indexer KL loss (every "
                         "visible key) at config-5 geometry, one key head; dsa_step: one "
                         "training step of the indexer -> attention -> KL-loss layer")
    ap.add_argument("--rows", type=int, default=0,
                    help="profiling aid: time only the last ROWS query rows of config 4 "
                         "(each sees the full 2048 keys); 0 = the whole workload")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload != "sfa":
        return run_other(args, rank, world, local)

    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import dsa_triton_ascend_b200 as dsa
    from dsa_triton_ascend_b200.sharding import SFA_ROW_COST, shard_act_q, shard_rows
    from dsa_triton_ascend_b200.synthetic import sfa_prefill, valid_pairs_per_row

    w = sfa_prefill(device=dev)
    dout_full = w["dout"]
    pairs = valid_pairs_per_row(w["si"]).cpu().numpy()
    if args.rows:
        pairs[: S1 - args.rows] = 0
    r0, r1 = shard_rows(pairs, world, rank, row_cost=SFA_ROW_COST)
    if args.rows:
        r0 = max(r0, S1 - args.rows)
    my_pairs = int(pairs[r0:r1].sum())
    total_pairs = int(pairs.sum())
    q = w["q"][:, r0:r1].contiguous()
    qr = w["qr"][:, r0:r1].contiguous()
    si = w["si"][:, r0:r1].contiguous()
    red_rows = reduced_key_rows(si.reshape(-1, si.shape[-1]))
    red_rows_merged = reduced_key_rows(si.reshape(-1, si.shape[-1]), group=2)   # key == value
    k, kr, scale = w["k"], w["kr"], w["scale"]
    dout = dout_full[:, r0:r1].contiguous()
    aq = [shard_act_q(S1, r0)]   # see dsa_triton_ascend_b200/sharding.py

    def fwd():
        return dsa.sparse_flash_attention_triton(
            q, k, k, si, scale, actual_seq_lengths_query=aq, query_rope=qr, key_rope=kr,
            sparse_mode=3, return_softmax_lse=True)

    def bwd(out, mx, sm, ev_r=None):
        """Backward of this rank's rows; the fp32 key gradients are summed over ranks with
        one NCCL all-reduce of their contiguous buffer (dk | dkr | dv)."""
        accs, finish = dsa.sparse_flash_attention_grad_partial(
            q, k, k, si, dout, out, mx, sm, scale, query_rope=qr, key_rope=kr,
            actual_seq_lengths_query=aq, sparse_mode=3)
        if world > 1:
            if ev_r is not None:
                ev_r[0].record(stream)
            dist.all_reduce(finish.key_grad_buffer)
            if ev_r is not None:
                ev_r[1].record(stream)
        return finish()

    def step(ev_f=None, ev_b=None, ev_r=None):
        if ev_f is not None:
            ev_f[0].record(stream)
        out, mx, sm = fwd()
        if ev_f is not None:
            ev_f[1].record(stream)
            ev_b[0].record(stream)
        grads = bwd(out, mx, sm, ev_r)
        if ev_b is not None:
            ev_b[1].record(stream)
        return out, grads

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    dsa.check_device_errors(dev)

    sampler = ClockSampler(local)
    sampler.start()
    mk = lambda: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev_f = [mk() for _ in range(args.steps)]
    ev_b = [mk() for _ in range(args.steps)]
    ev_r = [mk() for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        step(ev_f[i], ev_b[i], ev_r[i])
    end.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    dsa.check_device_errors(dev)
    ms_total = start.elapsed_time(end)
    fwd_ms = float(np.mean([a.elapsed_time(b) for a, b in ev_f]))
    bwd_ms = float(np.mean([a.elapsed_time(b) for a, b in ev_b]))
    ar_ms = float(np.mean([a.elapsed_time(b) for a, b in ev_r])) if world > 1 else 0.0
    t = torch.tensor([ms_total], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    # per-rank breakdown (rank 0 reports it): step, forward, backward (including the
    # all-reduce) and all-reduce times, and the rank's share of the valid pairs
    mine = torch.tensor([ms_total / args.steps, fwd_ms, bwd_ms, ar_ms, float(my_pairs)],
                        device=dev, dtype=torch.float64)
    if world > 1:
        allr = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [x.tolist() for x in allr]
    else:
        per_rank = [mine.tolist()]

    flops_total = total_pairs * (FWD_FLOP_PER_PAIR + BWD_FLOP_PER_PAIR)
    value = flops_total / (ms_step * 1e-3) / 1e12
    tokens_per_s = S1 / (ms_step * 1e-3)

    # ---- the same step with the merged key gradient (key == value, as autograd uses it):
    # dK + dV in one fp32 accumulator, one all-reduce of [dkv | dkr]; an extra field, the
    # headline above is the 5-output operator ----
    def bwd_merged(out, mx, sm):
        _, finish = dsa.sparse_flash_attention_grad_partial(
            q, k, k, si, dout, out, mx, sm, scale, query_rope=qr, key_rope=kr,
            actual_seq_lengths_query=aq, sparse_mode=3, merge_key_grads=True)
        if world > 1:
            dist.all_reduce(finish.key_grad_buffer)
        return finish()

    m_steps = max(2, min(args.steps, 5))
    out_m, mx_m, sm_m = fwd()
    for _ in range(2):
        bwd_merged(out_m, mx_m, sm_m)
    ev_m = [mk() for _ in range(m_steps)]
    barrier()
    torch.cuda.synchronize(dev)
    for a_, b_ in ev_m:
        a_.record(stream)
        bwd_merged(out_m, mx_m, sm_m)
        b_.record(stream)
    torch.cuda.synchronize(dev)
    dsa.check_device_errors(dev)
    tm = torch.tensor([float(np.mean([a_.elapsed_time(b_) for a_, b_ in ev_m]))], device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    bwd_merged_ms = float(tm.item())
    del out_m, mx_m, sm_m

    # ---- end to end through the public API with host buffers (pinned) ----
    # Inputs in pinned host memory; the public streaming entry point copies them in, runs
    # the forward and backward in row chunks and copies every result out, with the copies
    # of one chunk overlapping the kernels of the next.
    cpus_all = os.sched_getaffinity(0)
    bound = dsa.bind_host_to_device(dev)   # pinned buffers on the GPU's NUMA node
    host_in = [x.cpu().pin_memory() for x in (q, qr, k, kr, si, dout)]
    h2d = sum(x.numel() * x.element_size() for x in host_in)
    hq, hqr, hk, hkr, hsi, hdo = host_in
    outs_h = dsa.host_outputs(hq, hk, hqr, hkr)
    red = (lambda accs: [dist.all_reduce(t) for t in accs]) if world > 1 else None

    def e2e_step():
        dsa.sfa_fwd_bwd_from_host(hq, hk, hsi, hdo, scale, hqr, hkr, sparse_mode=3,
                                  host_out=outs_h, actual_seq_length_query=aq[0],
                                  reduce_key_grads=red)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    d2h = sum(x.numel() * x.element_size() for x in outs_h)
    e_steps = max(2, min(args.steps, 4))
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item()) / e_steps
    e2e_value = flops_total / (e2e_ms * 1e-3) / 1e12
    os.sched_setaffinity(0, cpus_all)      # the CPU baseline below uses every host thread

    hbm_peak, tf_peak, peak_kind = load_peaks()
    # roofline of the dominant call on this rank's share (fwd or bwd, whichever is longer):
    # time bound = max(algorithmic FLOPs / tensor peak, gathered bytes / HBM peak), the
    # north-star definition; the backward's time excludes its all-reduce
    if bwd_ms >= fwd_ms:
        kname, kms = "dsa_sfa_bwd", bwd_ms - ar_ms
        kflops, kbytes = my_pairs * BWD_FLOP_PER_PAIR, my_pairs * BWD_BYTES_PER_PAIR
        ktraffic = my_pairs * BWD_DRAM_BYTES_PER_PAIR + (r1 - r0) * BWD_DRAM_BYTES_PER_ROW
    else:
        kname, kms = "dsa_sfa_fwd", fwd_ms
        kflops, kbytes = my_pairs * FWD_FLOP_PER_PAIR, my_pairs * GATHER_BYTES_PER_PAIR
        ktraffic = my_pairs * FWD_DRAM_BYTES_PER_PAIR
    t_bytes = kbytes / (hbm_peak * 1e9)
    t_flops = kflops / (tf_peak * 1e12)
    bound = "hbm" if t_bytes >= t_flops else "tensor"
    roof = {"bound": bound,
            "achieved": kbytes / (kms * 1e-3) / 1e9 if bound == "hbm" else kflops / (kms * 1e-3) / 1e12,
            "peak": hbm_peak if bound == "hbm" else tf_peak,
            "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
            "frac": max(t_bytes, t_flops) / (kms * 1e-3),
            "traffic": ktraffic,
            "traffic_source": "ncu dram bytes of the last 256 rows, scaled by pairs",
            "kernel": kname,
            "peak_source": peak_kind,
            "tensor_frac": t_flops / (kms * 1e-3),
            "achieved_tflops": kflops / (kms * 1e-3) / 1e12}
    fwd_roof_frac = max(my_pairs * GATHER_BYTES_PER_PAIR / (hbm_peak * 1e9),
                        my_pairs * FWD_FLOP_PER_PAIR / (tf_peak * 1e12)) / (fwd_ms * 1e-3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, desc, threads = cpu_sample_tflops()
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded bf16 N(0,1), causal distinct top-k ids)",
            "config": {"workload": "BASELINE config 4 SFA forward + backward (B=1, S1=S2=8192, N1=128, D=512+64, topK=2048, mode 3)",
                       "global_batch": 1, "seq_len": S1, "parallelism": f"query-row shards x{world}",
                       "l2": "inputs (q 1.2 GB, out 1 GB) exceed L2; the 9.4 MB KV is L2-resident by design"},
            "tokens_per_s": tokens_per_s,
            "fwd_ms": fwd_ms,
            "bwd_ms": bwd_ms,
            "fwd_tflops": total_pairs * FWD_FLOP_PER_PAIR / (fwd_ms * 1e-3) / 1e12 if world == 1 else None,
            "bwd_tflops": total_pairs * BWD_FLOP_PER_PAIR / (bwd_ms * 1e-3) / 1e12 if world == 1 else None,
            "fwd_roofline_frac": fwd_roof_frac,
            "bwd_scatter": {"bytes_per_key_row": BWD_SCATTER_BYTES_PER_KEY_ROW,
                            "key_rows_per_step": red_rows,
                            "pairs_per_step": my_pairs,
                            "bytes_per_step": red_rows * BWD_SCATTER_BYTES_PER_KEY_ROW,
                            "target": "fp32 key-gradient accumulators, L2-resident; a key the "
                                      "rows of a four-row group share is reduced once",
                            "gbs_over_bwd": red_rows * BWD_SCATTER_BYTES_PER_KEY_ROW / ((bwd_ms - ar_ms) * 1e-3) / 1e9},
            "merged_key_grad": {
                "bwd_ms": bwd_merged_ms,
                "step_ms": fwd_ms + bwd_merged_ms,
                "value": flops_total / ((fwd_ms + bwd_merged_ms) * 1e-3) / 1e12,
                "unit": "TFLOP/s",
                "scatter_bytes_per_key_row": 4 * (D + DR),
                "key_rows_per_step": red_rows_merged,
                "note": "key == value (MLA): dK + dV accumulated as one (the autograd path); "
                        "forward time from the headline run, backward timed separately"},
            "ranks": [{"rank": i, "step_ms": r[0], "fwd_ms": r[1], "bwd_ms": r[2],
                       "allreduce_ms": r[3], "pairs": int(r[4])} for i, r in enumerate(per_rank)],
            "step_ms_max_min": [max(r[0] for r in per_rank), min(r[0] for r in per_rank)],
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "host_numa_bound": bool(bound)},
            "gpu_launches": args.steps * (2 + 8),   # per step: prep + fwd; prep, delta, 3 bwd kernels, 3 casts
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _timed(fn, steps, warmup, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for a, b in ev:
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return float(np.mean([a.elapsed_time(b) for a, b in ev]))


def run_sli(args, rank, world, local):
    """BASELINE config 5 (indexer KL-loss gradient, S1=S2=8192, N1=128, Nidx1=64, top-2048)
    with S1 sharded over the ranks (strong scaling): each rank computes its causal row range,
    the fp32 dKeyIndex accumulators and the loss are summed with one NCCL all-reduce, then
    cast.  The softmax statistics come from config 4's forward on the same query / key."""
    import torch.distributed as dist
    from datetime import timedelta
    import dsa_triton_ascend_b200 as dsa
    from dsa_triton_ascend_b200.sharding import shard_act_q, shard_rows
    from dsa_triton_ascend_b200.synthetic import sli_prefill, valid_pairs_per_row
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.current_stream(dev)
    w = sli_prefill(device=dev, seed=0)
    S = w["q"].shape[1]
    pairs = valid_pairs_per_row(w["si"]).cpu().numpy()
    r0, r1 = shard_rows(pairs, world, rank)
    cut = lambda t: t[:, r0:r1].contiguous()
    q, qr, qi, wt, si = cut(w["q"]), cut(w["qr"]), cut(w["qi"]), cut(w["w"]), cut(w["si"])
    aq = [shard_act_q(S, r0)]
    _, mx, sm = dsa.sparse_flash_attention_triton(
        q, w["k"], w["k"], si, w["scale"], actual_seq_lengths_query=aq, query_rope=qr,
        key_rope=w["kr"], sparse_mode=3, return_softmax_lse=True)

    def step(ev=None):
        (_, _), finish = dsa.sparse_lightning_indexer_grad_kl_loss_partial(
            q, w["k"], qi, w["ki"], wt, si, mx, sm, query_rope=qr, key_rope=w["kr"],
            actual_seq_qlen=aq, scale_value=w["scale"])
        if world > 1:
            if ev is not None:
                ev[0].record(stream)
            dist.all_reduce(finish.key_grad_buffer)
            if ev is not None:
                ev[1].record(stream)
        return finish()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    dsa.check_device_errors(dev)
    mk = lambda: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev_r = [mk() for _ in range(args.steps)]
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = mk()
    start.record(stream)
    for i in range(args.steps):
        step(ev_r[i])
    end.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    dsa.check_device_errors(dev)
    ms_mine = start.elapsed_time(end) / args.steps
    ar_ms = float(np.mean([a.elapsed_time(b) for a, b in ev_r])) if world > 1 else 0.0
    mine = torch.tensor([ms_mine, ar_ms, float(pairs[r0:r1].sum())], device=dev, dtype=torch.float64)
    if world > 1:
        allr = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [x.tolist() for x in allr]
    else:
        per_rank = [mine.tolist()]
    ms = max(r[0] for r in per_rank)
    total_pairs = int(pairs.sum())
    flops = total_pairs * 2 * (64 * 128 * 3 + 128 * 576)
    nbytes = total_pairs * (GATHER_BYTES_PER_PAIR + 256)
    hbm_peak, tf_peak, peak_kind = load_peaks()
    t_b, t_f = nbytes / (hbm_peak * 1e9) / world, flops / (tf_peak * 1e12) / world
    bound = "hbm" if t_b >= t_f else "tensor"
    if rank == 0:
        line = {"metric": "SLI KL-grad TFLOP/s", "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic",
                "config": {"workload": "BASELINE config 5 (S1=S2=8192, N1=128, Nidx1=64, top-2048), S1 sharded",
                           "timing": "CUDA events around the steps, max over ranks",
                           "parallelism": f"query-row shards x{world}"},
                "roofline": {"bound": bound,
                             "achieved": (nbytes / world / (ms * 1e-3) / 1e9) if bound == "hbm"
                             else flops / world / (ms * 1e-3) / 1e12,
                             "peak": hbm_peak if bound == "hbm" else tf_peak,
                             "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
                             "frac": max(t_b, t_f) / (ms * 1e-3),
                             "traffic": WORKLOAD_DRAM_BYTES.get("sli") if world == 1 else None,
                             "peak_source": peak_kind},
                "ranks": [{"rank": i, "step_ms": r[0], "allreduce_ms": r[1], "pairs": int(r[2])}
                          for i, r in enumerate(per_rank)],
                "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_other(args, rank, world, local):
    """Secondary workloads (configs 2, 3, 5): one GPU, device-timed, one JSON line each.

    With N GPUs every rank runs its own replica of the workload (weak scaling)."""
    import math as _m
    import dsa_triton_ascend_b200 as dsa
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    rn = lambda *sh: torch.randn(*sh, generator=g, device=dev).to(torch.bfloat16)
    hbm_peak, tf_peak, peak_kind = load_peaks()
    if args.workload == "li":
        B, S, N1_, Dh, K = 2, 4096, 64, 128, 2048
        q, k = rn(B, S, N1_, Dh), rn(B, S, 1, Dh)
        w = torch.randn(B, S, N1_, generator=g, device=dev) / _m.sqrt(N1_)
        fn = lambda: dsa.lightning_indexer_triton(q, k, w, sparse_count=K, sparse_mode=3,
                                                  return_value=True)
        pairs = B * S * (S + 1) // 2
        flops, nbytes = pairs * N1_ * 2 * Dh, q.numel() * 2 + k.numel() * 2 + w.numel() * 4 + 2 * B * S * K * 4
        metric, unit, wl = "LI score+top-k TFLOP/s", "TFLOP/s", "BASELINE config 2 (B=2, S1=S2=4096, N1=64, D=128, top-2048, mode 3)"
    elif args.workload == "li_fp8":
        B, S, N1_, Dh, K = 2, 4096, 64, 128, 2048
        f8 = torch.float8_e4m3fn
        q = torch.randn(B, S, N1_, Dh, generator=g, device=dev).to(f8)
        k = torch.randn(B, S, 1, Dh, generator=g, device=dev).to(f8)
        ks = torch.rand(B, S, 1, generator=g, device=dev) + 0.5
        w = torch.randn(B, S, N1_, generator=g, device=dev) / _m.sqrt(N1_)
        fn = lambda: dsa.lightning_indexer_fp8(q, k, ks, w, sparse_count=K, sparse_mode=3,
                                               return_value=True)
        pairs = B * S * (S + 1) // 2
        flops = pairs * N1_ * 2 * Dh
        nbytes = q.numel() + k.numel() + ks.numel() * 4 + w.numel() * 4 + 2 * B * S * K * 4
        metric, unit, wl = ("LI FP8 score+top-k TFLOP/s", "TFLOP/s",
                            "config 2 geometry, FP8 indexer (B=2, S1=S2=4096, N1=64, D=128, top-2048, mode 3)")
    elif args.workload == "decode":
        from dsa_triton_ascend_b200.synthetic import sfa_decode
        wd = sfa_decode(device=dev, seed=0)
        fn = lambda: dsa.sparse_flash_attention_triton(
            wd["q"], wd["cache"], wd["cache"], wd["si"], wd["scale"], block_table=wd["block_table"],
            actual_seq_lengths_kv=wd["lens"], query_rope=wd["qr"], key_rope=wd["cache_r"],
            layout_kv="PA_BSND", sparse_mode=0, return_softmax_lse=True, block_size=wd["page"])
        pairs = wd["si"].numel()
        flops, nbytes = pairs * FWD_FLOP_PER_PAIR, pairs * GATHER_BYTES_PER_PAIR
        metric, unit, wl = "SFA decode TFLOP/s", "TFLOP/s", "BASELINE config 3 (PA_BSND, B=32, S1=1, N1=128, top-2048, 16384-block pool)"
    elif args.workload == "dsa_step":
        # one training step (forward + backward) of SparseAttentionWithIndexer at config
        # 4 / 5 geometry: lightning indexer top-2048, sparse attention, indexer KL loss
        from dsa_triton_ascend_b200.synthetic import sli_prefill
        w = sli_prefill(device=dev, seed=0)
        S = w["q"].shape[1]
        leaves = {n: w[n].clone().requires_grad_(True) for n in ("q", "k", "qr", "kr", "qi", "ki")}
        leaves["w"] = w["w"].clone().requires_grad_(True)
        g_out = torch.randn(w["q"].shape, generator=g, device=dev).to(torch.bfloat16)
        layers = {f: dsa.SparseAttentionWithIndexer(scale_value=w["scale"], sparse_count=2048,
                                                     teacher_from_backward=f) for f in (False, True)}

        def make_step(fused):
            def step():
                for t in leaves.values():
                    t.grad = None
                out, loss = layers[fused](leaves["q"], leaves["k"], leaves["qr"], leaves["kr"],
                                          leaves["qi"], leaves["ki"], leaves["w"])
                ((out * g_out).float().sum() + loss).backward()
            return step
        fn = make_step(False)
        pairs = int(np.minimum(np.arange(1, S + 1), 2048).sum())   # causal top-2048 pairs
        lip = S * (S + 1) // 2
        flops = (lip * 2 * 64 * 128 + pairs * (FWD_FLOP_PER_PAIR + BWD_FLOP_PER_PAIR)
                 + pairs * 2 * (64 * 128 * 3 + 128 * 576))
        nbytes = pairs * (GATHER_BYTES_PER_PAIR * 3 + 256)
        metric, unit, wl = ("DSA layer training step TFLOP/s", "TFLOP/s",
                            "config 4/5 geometry: indexer top-2048 (64 heads x 128) -> sparse attention "
                            "(S1=S2=8192, N1=128, D=512+64) fwd + bwd -> indexer KL loss")
        extra_fns = {"teacher_from_backward": make_step(True)}
    elif args.workload == "dense":
        # config-5 geometry, one key head: the KL loss over every visible key (33.6 M
        # causal pairs); the teacher's softmax statistics are those of full causal attention,
        # from the forward over all keys
        from dsa_triton_ascend_b200.synthetic import sli_prefill
        w = sli_prefill(device=dev, seed=0)
        S = w["q"].shape[1]
        ids = torch.arange(S, dtype=torch.int32, device=dev).view(1, 1, 1, S).expand(1, S, 1, S).contiguous()
        _, mx_d, sm_d = dsa.sparse_flash_attention_triton(
            w["q"], w["k"], w["k"], ids, w["scale"], query_rope=w["qr"], key_rope=w["kr"],
            sparse_mode=3, return_softmax_lse=True)
        del ids
        fn = lambda: dsa.dense_loss_backward_triton(
            w["q"], w["k"], w["qi"], w["ki"], w["w"], mx_d, sm_d, scale_value=w["scale"],
            query_rope=w["qr"], key_rope=w["kr"])
        pairs = S * (S + 1) // 2
        flops, nbytes = pairs * 2 * (64 * 128 * 3 + 128 * 576), pairs * (GATHER_BYTES_PER_PAIR + 256)
        metric, unit, wl = ("dense indexer KL-grad TFLOP/s", "TFLOP/s",
                            "config 5 geometry, dense (every visible key; S1=S2=8192, N1=128, N2=1, Nidx1=64)")
    else:
        return run_sli(args, rank, world, local)
    timing = "CUDA events around each call"
    if args.workload == "decode":
        # A decode step is ~70 us of GPU work, about as long as the Python call that enqueues
        # it, so the call is captured once into a CUDA graph and replayed (as a serving loop
        # does); the warm-up calls fill the per-device caches the capture relies on.
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            fn, timing = graph.replay, "CUDA graph replay of the public call, CUDA events"
        except RuntimeError as e:   # capture refused: keep eager timing and say so
            timing = f"CUDA events around each call (graph capture failed: {str(e)[:80]})"
    ms = _timed(fn, args.steps, max(args.warmup, 3), stream)
    dsa.check_device_errors(dev)
    extra = {}
    for name, f2 in (extra_fns.items() if "extra_fns" in locals() else []):
        ms2 = _timed(f2, args.steps, max(args.warmup, 3), stream)
        dsa.check_device_errors(dev)
        extra[name] = {"ms_per_step": ms2, "value": flops / (ms2 * 1e-3) / 1e12, "unit": unit}
    t_b, t_f = nbytes / (hbm_peak * 1e9), flops / (tf_peak * 1e12)
    bound = "hbm" if t_b >= t_f else "tensor"
    line = {"metric": metric, "value": flops / (ms * 1e-3) / 1e12 * world, "unit": unit,
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3" if args.workload == "li_fp8" else "bf16",
            "data": "synthetic", "config": {"workload": wl, "timing": timing},
            "roofline": {"bound": bound, "achieved": (nbytes / (ms * 1e-3) / 1e9) if bound == "hbm"
                         else flops / (ms * 1e-3) / 1e12,
                         "peak": hbm_peak if bound == "hbm" else tf_peak,
                         "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
                         "frac": max(t_b, t_f) / (ms * 1e-3),
                         "traffic": WORKLOAD_DRAM_BYTES.get(args.workload),
                         "peak_source": peak_kind}}
    line.update(extra)
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
