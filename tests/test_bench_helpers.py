"""bench.py's count of the key rows the backward's scatter reduces (CPU).

The backward groups adjacent query rows and reduces a key the group's rows share once;
bench.py reports the scatter bytes from that count.  Checked here against a plain
set-union count over random index rows with -1 tails and row counts that leave a short
last group.
"""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _plain(si, group):
    n = 0
    for r0 in range(0, si.shape[0], group):
        keys = set()
        for r in range(r0, min(r0 + group, si.shape[0])):
            keys |= {int(k) for k in si[r] if k >= 0}
        n += len(keys)
    return n


def test_reduced_key_rows_matches_set_union():
    import bench
    rng = np.random.default_rng(5)
    for rows, topk, span in [(1, 8, 20), (5, 16, 40), (8, 32, 64), (11, 64, 100)]:
        si = np.full((rows, topk), -1, np.int32)
        for r in range(rows):
            n = int(rng.integers(0, topk + 1))
            si[r, :n] = rng.choice(span, n, replace=False)
        t = torch.from_numpy(si)
        for group in (1, 2, 4):
            assert bench.reduced_key_rows(t, group) == _plain(si, group), (rows, topk, group)
