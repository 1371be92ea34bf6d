"""Helpers to read the golden fixtures (tests only)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def from_bits16(bits, dtype):
    bits = np.asarray(bits, np.uint16)
    if dtype == "fp16":
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
