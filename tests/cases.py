"""Case lists and input recipes shared by the golden-fixture generator and the tests.

They restate the reference tests' own recipes (prathameshpranjale/paged-kv-cache-manager,
tests/test_attention.cpp:15-101 and cuda/test_paged_attention.cu:165-175): an LCG for inputs, block tables
produced by a KVManager, prefix sharing between sequences.
"""
from __future__ import annotations

import numpy as np

from lcg import VecLcg


class Lcg:
    """tests/test_attention.cpp:15-24 of the reference (seed * golden-ratio constant + 1, PCG-style LCG)."""

    def __init__(self, seed: int, mul: int = 0x9E3779B97F4A7C15, add: int = 1):
        self.s = (seed * mul + add) & 0xFFFFFFFFFFFFFFFF

    def next(self) -> int:
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return (self.s >> 33) & 0xFFFFFFFF

    def uniform(self) -> float:
        return np.float32(self.next() % 20001) / np.float32(10000.0) - np.float32(1.0)

    def range(self, lo: int, hi: int) -> int:
        return lo + self.next() % (hi - lo + 1)


def attention_inputs(seed, nh, kvh, hd, B, lens, share, mgr_cls):
    """Inputs of test_attention.cpp run_case (:28-50): KVManager tables, LCG K, V, then Q*2."""
    rng = VecLcg(seed)
    ns = len(lens)
    max_blocks = max((n + B - 1) // B for n in lens)
    kv = mgr_cls(ns * max_blocks + 4, B)
    for i, n in enumerate(lens):
        if share and i > 0 and n >= B:
            ok = kv.admit_with_prefix(i, 0, min(lens[0], n), n)
        else:
            ok = kv.admit(i, n)
        assert ok
    nblk = kv.total_blocks()
    kv_elems = nblk * B * kvh * hd
    K = rng.uniform(kv_elems).reshape(nblk, B, kvh, hd)
    V = rng.uniform(kv_elems).reshape(nblk, B, kvh, hd)
    Q = (rng.uniform(ns * nh * hd) * np.float32(2.0)).reshape(ns, nh, hd)
    tables = np.zeros((ns, max_blocks), dtype=np.int32)
    for i in range(ns):
        t = kv.block_table(i)
        tables[i, : len(t)] = t
    return Q, K, V, tables, np.asarray(lens, dtype=np.int32)


def attention_cases():
    """The case list of tests/test_attention.cpp:62-101."""
    cases = []
    for B in (1, 4, 8, 16, 32):
        lens = [n for n in (1, B - 1, B, B + 1, 2 * B, 3 * B + 1, 97, 130) if n >= 1]
        for P in (1, 4, 8):
            cases.append(dict(seed=B * 100 + P, nh=8, kvh=2, hd=64, B=B, lens=lens, share=False, P=P))
    cases.append(dict(seed=5, nh=4, kvh=4, hd=32, B=16, lens=[1], share=False, P=8))
    cases.append(dict(seed=6, nh=4, kvh=4, hd=32, B=16, lens=[2, 3, 5], share=False, P=32))
    for nh, kvh in ((8, 8), (8, 2), (8, 1), (14, 2)):
        cases.append(dict(seed=77, nh=nh, kvh=kvh, hd=64, B=16, lens=[70, 70, 55, 33, 16], share=True, P=4))
    for seed in range(1, 61):
        r = Lcg(seed)
        hd = 32 * r.range(1, 4)
        B = 1 << r.range(0, 5)
        n = r.range(1, 6)
        lens = [r.range(1, 200) for _ in range(n)]
        P = r.range(1, 8)
        share = r.range(0, 1) == 1
        cases.append(dict(seed=seed, nh=8, kvh=2, hd=hd, B=B, lens=lens, share=share, P=P))
    return cases



def cuda_test_cases():
    """The GPU case list of cuda/test_paged_attention.cu:165-175 (nh, kvh, hd, B, lens, share)."""
    cases = []
    for B in (1, 8, 16, 32):
        lens = [1, B - 1 if B - 1 > 0 else 1, B, B + 1, 2 * B, 3 * B + 1, 97, 130]
        cases.append((8, 2, 64, B, lens, False))
        cases.append((8, 2, 128, B, lens, False))
        cases.append((32, 8, 128, B, [70, 70, 55, 33, 16], True))
    cases.append((14, 2, 64, 16, [33, 64, 65, 300], False))
    cases.append((4, 4, 32, 16, [1, 2, 3], False))
    cases.append((8, 8, 256, 16, [100, 17], False))
    return cases
