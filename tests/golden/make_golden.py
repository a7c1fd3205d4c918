"""Generates the golden fixtures in this directory from the reference itself.

The reference (prathameshpranjale/paged-kv-cache-manager) keeps no stored vectors: its tests regenerate
inputs from seeded LCGs.  This script runs the reference's own C++ code, compiled from its sources by
oracle/Makefile into oracle/_ref/libkvpage_ref.so, on

  * attention_cases.npz -- the input-generation recipe of tests/test_attention.cpp:15-57 (LCG uniform
    [-1, 1], Q scaled by 2, block tables from the real KVManager, optional prefix sharing) for the cases
    of :62-101, with the outputs of reference_attention and paged_attention_cpu(partitions);
  * kv_traces.json -- seeded random KVManager operation sequences in the style of tests/test_random.cpp:30-128
    (admit / admit_with_prefix / fork / append / cache / free), with every result, and the final tables,
    refcounts and stats.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

sys.path.insert(0, os.path.dirname(HERE))
from cases import Lcg, attention_cases, attention_inputs  # noqa: E402


def make_attention(path):
    arrays = {}
    meta = []
    for ci, c in enumerate(attention_cases()):
        Q, K, V, T, L = attention_inputs(c["seed"], c["nh"], c["kvh"], c["hd"], c["B"], c["lens"], c["share"],
                                         oracle.RefKVManager)
        ref = oracle.reference_attention(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L, impl="ref")
        pag = oracle.paged_attention_cpu(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L, partitions=c["P"],
                                         impl="ref")
        arrays[f"c{ci}_ref"] = ref
        arrays[f"c{ci}_paged"] = pag
        arrays[f"c{ci}_tables"] = T
        meta.append(c)
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(path, **arrays)


def kv_trace(seed: int, nops: int):
    """A random op sequence in the style of tests/test_random.cpp:30-128, recorded with its results."""
    rng = Lcg(seed, mul=2862933555777941757, add=3037000493)
    B = rng.range(1, 8)
    total = rng.range(4, 40)
    kv = oracle.RefKVManager(total, B)
    kv.set_check_each_op(True)
    live = []  # sorted live ids (the reference test iterates a std::map)
    next_id = 0
    ops = []
    for _ in range(nops):
        c = rng.range(0, 99)

        def pick():
            return live[rng.range(0, len(live) - 1)] if live else None

        if c < 20:
            prompt = rng.range(0, 5 * B)
            got = kv.admit(next_id, prompt)
            ops.append(["admit", next_id, prompt, int(got)])
            if got:
                live.append(next_id)
            next_id += 1
        elif c < 35:
            p = pick()
            if p is None:
                continue
            shared, prompt = rng.range(0, kv.num_tokens(p) + B), rng.range(0, 6 * B)
            got = kv.admit_with_prefix(next_id, p, shared, prompt)
            ops.append(["admit_with_prefix", next_id, p, shared, prompt, int(got)])
            if got:
                live.append(next_id)
            next_id += 1
        elif c < 40:
            p = pick()
            if p is None:
                continue
            got = kv.fork(next_id, p)
            ops.append(["fork", next_id, p, int(got)])
            live.append(next_id)
            next_id += 1
        elif c < 46:
            p = pick()
            if p is None:
                continue
            key, tokens = rng.range(0, 3), rng.range(0, 4 * B)
            got = kv.cache_prefix(key, p, tokens)
            ops.append(["cache_prefix", key, p, tokens, int(got)])
        elif c < 54:
            key, shared, prompt = rng.range(0, 3), rng.range(0, 4 * B), rng.range(0, 6 * B)
            got = kv.admit_with_cached_prefix(next_id, key, shared, prompt)
            ops.append(["admit_with_cached_prefix", next_id, key, shared, prompt, int(got)])
            if got:
                live.append(next_id)
            next_id += 1
        elif c < 84:
            p = pick()
            if p is None:
                continue
            got = kv.append_token(p)
            ops.append(["append_token", p, int(got)])
        else:
            p = pick()
            if p is None:
                continue
            if rng.range(0, 29) == 0:
                kv.clear_cache()
                ops.append(["clear_cache"])
            else:
                kv.free(p)
                ops.append(["free", p])
                live.remove(p)
        live.sort()
    final = {
        "tables": {str(r): kv.block_table(r) for r in live},
        "tokens": {str(r): kv.num_tokens(r) for r in live},
        "refcounts": [kv.refcount(b) for b in range(total)],
        "stats": kv.stats(),
        "free_blocks": kv.free_blocks(),
    }
    return {"seed": seed, "B": B, "total": total, "ops": ops, "final": final}


def make_traces(path, seeds=range(1, 121), nops=200):
    with open(path, "w") as f:
        json.dump([kv_trace(s, nops) for s in seeds], f, separators=(",", ":"))


if __name__ == "__main__":
    oracle.build()
    make_attention(os.path.join(HERE, "attention_cases.npz"))
    make_traces(os.path.join(HERE, "kv_traces.json"))
    for f in sorted(os.listdir(HERE)):
        print(f, os.path.getsize(os.path.join(HERE, f)))
