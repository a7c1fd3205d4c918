"""Vectorised form of the reference tests' input generator (tests/test_attention.cpp:15-24 of
prathameshpranjale/paged-kv-cache-manager): s <- s * 6364136223846793005 + 1442695040888963407 (mod 2^64),
output (s >> 33) as uint32, uniform = (out % 20001) / 10000 - 1 in float32.

The n-th state is A^n * s0 + c * (1 + A + ... + A^(n-1)), evaluated for a whole range of n at once with
wrapping uint64 arithmetic, so fixtures regenerate in milliseconds instead of a Python loop per value.
"""
import numpy as np

A = np.uint64(6364136223846793005)
CINC = np.uint64(1442695040888963407)
M64 = (1 << 64) - 1


class VecLcg:
    def __init__(self, seed: int, mul: int = 0x9E3779B97F4A7C15, add: int = 1):
        self.s = (seed * mul + add) & M64

    def raw(self, n: int) -> np.ndarray:
        """The next n outputs (uint32 as uint64)."""
        if n == 0:
            return np.zeros(0, dtype=np.uint64)
        with np.errstate(over="ignore"):
            powers = np.full(n, A, dtype=np.uint64)
            powers = np.cumprod(powers, dtype=np.uint64)          # A^1 .. A^n
            geo = np.concatenate([[np.uint64(1)], powers[:-1]])    # A^0 .. A^(n-1)
            geo = np.cumsum(geo, dtype=np.uint64)                   # 1 + ... + A^(k-1), k = 1..n
            states = powers * np.uint64(self.s) + CINC * geo
        self.s = int(states[-1])
        return states >> np.uint64(33)

    def uniform(self, n: int) -> np.ndarray:
        r = (self.raw(n) % np.uint64(20001)).astype(np.float32)
        return r / np.float32(10000.0) - np.float32(1.0)
