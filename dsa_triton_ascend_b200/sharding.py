"""Query-row sharding of the DSA hot path across GPUs (host logic, no GPU code).

The unit of work is one query row (b, s1).  Rows are split into contiguous ranges of
about equal work, a row's valid (query, key) pairs plus a fixed per-row cost -- causal
rows near the start see fewer keys, so equal row counts would leave the first rank idle,
and equal pair counts give it twice the rows of the others.  KV is replicated on every rank;
the forward and the query gradients need no exchange, the key gradients (fp32
accumulators) are summed across ranks before the final cast.

A contiguous row range [r0, r1) of a causal (sparse_mode 3) BSND batch is itself a BSND
query of r1 - r0 rows whose actual query length is S1 - r0: the kernel's window
act_k - act_q + s1 + 1 then equals the window of the original row r0 + s1.
"""
from __future__ import annotations

import numpy as np


# Fixed cost of one query row in the sparse-attention kernels (a CTA pair's prologue and
# epilogue in the forward and in each backward kernel), in valid pairs: at config 4 on 8
# GPUs, equal pair counts gave the rank of the short causal rows (about 1,900 rows against
# 900) a 15 % longer step, 0.5 us per extra row at 0.54 M pairs per ms.
SFA_ROW_COST = 256


def shard_rows(pairs_per_row, world: int, rank: int, row_cost: int = 0):
    """Contiguous row range [r0, r1) of `rank` with ~1/world of the work, a row's work being
    its valid pairs plus ``row_cost`` (rows with pairs only)."""
    pairs = np.asarray(pairs_per_row, dtype=np.int64)
    if row_cost:
        pairs = pairs + np.where(pairs > 0, int(row_cost), 0)
    cum = np.concatenate([[0], np.cumsum(pairs)])
    total = cum[-1]
    bounds = [int(np.searchsorted(cum, total * r / world, side="left")) for r in range(world + 1)]
    bounds[0], bounds[-1] = 0, len(pairs)
    for i in range(1, world + 1):            # keep ranges ordered
        bounds[i] = max(bounds[i], bounds[i - 1])
    return bounds[rank], bounds[rank + 1]


def shard_act_q(s1_total: int, r0: int) -> int:
    """Actual query length to pass for the row range starting at r0 (causal mode)."""
    return s1_total - r0
