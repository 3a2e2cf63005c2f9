"""Seeded synthetic inputs for benchmarks and tests.

bf16 weights ~ N(0, std) are drawn by hashing (seed, tensor stream, element
index) with the SplitMix64 finalizer (Steele, Lea & Flood, 2014) and using
the low 16 bits to index a table of 65536 bf16 quantiles of the normal
distribution at (u + 0.5) / 65536.  The device generator (layout.cu) and any
CPU consumer produce identical bits from the same table.
"""

from __future__ import annotations

from functools import lru_cache
from statistics import NormalDist

import numpy as np


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bias = ((b >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    return ((b + bias) >> np.uint64(16)).astype(np.uint16)


@lru_cache(maxsize=8)
def normal_table_bits(std: float) -> np.ndarray:
    """65536 bf16 bit patterns of N(0, std) quantiles."""
    nd = NormalDist(0.0, 1.0)
    q = np.array([nd.inv_cdf((u + 0.5) / 65536.0) for u in range(65536)], dtype=np.float64)
    bits = _bf16_bits((q * std).astype(np.float32))
    bits.setflags(write=False)
    return bits


# Tensor streams of the synthetic model (layer l, part p -> ((l + 1) << 8) + p).
PART_Q, PART_K, PART_V, PART_O, PART_GATE, PART_UP, PART_DOWN = range(7)
STREAM_EMBED, STREAM_LM_HEAD = 0xE0000, 0xE0002
STREAM_TOKENS = 0x70CE


def layer_stream(layer: int, part: int) -> int:
    return ((layer + 1) << 8) + part
