"""Seeded synthetic inputs for the benchmark workloads (numpy only, no oracle).

The reference publishes no attention dataset, so the benchmark draws its inputs: context
lengths uniform in [lo, hi] and N(0,1) values, both from splitmix64 so that a host with
only numpy reproduces them.  These are the same sequences the test oracle's generators
give (the CPU test suite checks that), kept here so that the benchmark's GPU arm never
loads the oracle.
"""
from __future__ import annotations

import math

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(seed: int, idx: np.ndarray) -> np.ndarray:
    """Output `idx` of the splitmix64 stream seeded with `seed` (uint64)."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (idx.astype(np.uint64) + np.uint64(1)) * _GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform_int(seed: int, n: int, lo: int, hi: int, offset: int = 0) -> np.ndarray:
    """n int32 values uniform in [lo, hi] (inclusive), e.g. per-sequence context lengths."""
    i = np.arange(offset, offset + n, dtype=np.uint64)
    z = splitmix64(seed ^ 0x5EED, i)
    return (lo + (z % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int32)


def normal(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """n float32 standard normals (Box-Muller over splitmix64 draws 2i and 2i+1)."""
    i = np.arange(offset, offset + n, dtype=np.uint64)
    a = splitmix64(seed, 2 * i)
    b = splitmix64(seed, 2 * i + 1)
    u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
    u2 = (b >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    return (np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)).astype(np.float32)


def stratified_sample(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of k entries of `values` taken at the midpoints of k equal quantile bins, so
    that the sample's mean tracks the whole set's (used to time a CPU baseline on a
    bounded sample of a batch with the batch's length mix)."""
    order = np.argsort(values, kind="stable")
    n = len(values)
    pos = ((np.arange(k) + 0.5) * n / k).astype(np.int64)
    return np.sort(order[np.minimum(pos, n - 1)])
