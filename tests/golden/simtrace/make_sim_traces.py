"""Generates tests/golden/sim_traces.npz: the reference's own scheduler simulation recorded as decision streams.

The reference (prathameshpranjale/paged-kv-cache-manager) simulates continuous batching over its KVManager in
src/simulator.cpp:80-289 (run_paged) but moves no data.  This script compiles that simulator, the reference's
workload generator, metrics and its own KVManager / BlockAllocator from their sources under /root/reference,
with tracing_kv_manager.h force-included into simulator.cpp only, runs the scenarios of sim_trace_main.cpp and
stores, per scenario:

  <name>_requests  int64 [n][8]  id, arrival, prompt_len, output_len, prefix_group, prefix_len, fork_of, priority
  <name>_config    int64 [11]    num_blocks, block_size, policy, watermark, max_running, preempt_mode,
                                 swap_capacity_blocks, prefill_tokens_per_step, swap_blocks_per_step,
                                 prefix_cache, fork_sharing
  <name>_metrics   int64 [11]    total_steps, tokens_generated, preemptions, recomputed_tokens, cow_copies,
                                 swap_out_blocks, swap_in_blocks, cache_hits, cache_evictions,
                                 prefill_tokens_computed, requests_completed
  <name>_trace     int64 [m][7]  op, a, b, c, d, result, flag (paged-kv-cache-manager_b200/dataplane.py's
                                 TRACE_* codes)

Each KVManager mutation the simulator made is a row with its arguments and result; each end-of-step stats()
call is a STEP row carrying the reference's (requests, allocated_blocks, cow_copies, cache_evictions).  The
two stats() calls run_paged makes after its loop are dropped, so STEP rows = total_steps.  A FREE row
carries the request's tokens (b), and its flag says why it was freed: finished (tokens = prompt + output),
preempted into the CPU swap pool, or preempted for recomputation -- the simulator's rule at
src/simulator.cpp:117-133 (swap mode and room in the pool).  An admission flagged 1 is the swap-in of a
swapped request (:231-241).  The script checks the stream against the reference's metrics.

Run from the repository root:  python tests/golden/simtrace/make_sim_traces.py
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
REF = "/root/reference"
OUT = os.path.join(os.path.dirname(HERE), "sim_traces.npz")

STEP, ADMIT_PREFIX, ADMIT_CACHED, CACHE_PREFIX, FORK, APPEND, FREE, CLEAR = range(8)
FREE_FINISHED, FREE_SWAPPED, FREE_DROPPED = 0, 1, 2


def build_and_run(tmp: str) -> str:
    inc = ["-I", os.path.join(REF, "include"), "-I", HERE]
    sim_o = os.path.join(tmp, "simulator.o")
    subprocess.run(["g++", "-std=c++17", "-O2", *inc, "-include", os.path.join(HERE, "tracing_kv_manager.h"),
                    "-c", os.path.join(REF, "src", "simulator.cpp"), "-o", sim_o], check=True)
    exe = os.path.join(tmp, "sim_trace")
    srcs = [os.path.join(REF, "src", f) for f in ("workload.cpp", "metrics.cpp", "kv_manager.cpp",
                                                  "block_allocator.cpp")]
    subprocess.run(["g++", "-std=c++17", "-O2", *inc, os.path.join(HERE, "sim_trace_main.cpp"), sim_o, *srcs,
                    "-o", exe], check=True)
    return subprocess.run([exe], check=True, capture_output=True, text=True).stdout


def parse(text: str) -> dict:
    out, cur = {}, None
    for line in text.splitlines():
        p = line.split()
        if not p:
            continue
        if p[0] == "scenario":
            cur = out[p[1]] = {"requests": [], "rows": []}
        elif p[0] == "config":
            cur["config"] = [int(x) for x in p[1:]]
        elif p[0] == "request":
            cur["requests"].append([int(x) for x in p[1:]])
        elif p[0] == "metrics":
            cur["metrics"] = [int(x) for x in p[1:]]
        elif p[0] == "row":
            cur["rows"].append([int(x) for x in p[1:]])
    return out


def annotate(sc: dict) -> np.ndarray:
    cfg = sc["config"]
    B, preempt_mode, capacity = cfg[1], cfg[5], cfg[6]
    req = {r[0]: r for r in sc["requests"]}
    rows = sc["rows"]
    # run_paged ends with stats(), stats(), clear_cache() after its loop: drop those two STEP rows.
    assert rows[-1][0] == CLEAR and rows[-2][0] == STEP and rows[-3][0] == STEP
    rows = rows[:-3] + rows[-1:]
    out, cpu_used, swapped = [], 0, {}
    for op, a, b, c, d, res in rows:
        flag = 0
        if op == FREE:
            r = req[a]
            blocks = -(-b // B)
            if b == r[2] + r[3]:
                flag = FREE_FINISHED
            elif preempt_mode == 1 and cpu_used + blocks <= capacity:
                flag = FREE_SWAPPED
                cpu_used += blocks
                swapped[a] = blocks
            else:
                flag = FREE_DROPPED
        elif op == ADMIT_PREFIX and res and a in swapped:
            flag = 1
            cpu_used -= swapped.pop(a)
        out.append([op, a, b, c, d, res, flag])
    assert cpu_used == 0 and not swapped
    return np.asarray(out, dtype=np.int64)


def check(sc: dict, t: np.ndarray):
    (steps, generated, preemptions, recomputed, cow, swap_out, swap_in, hits, evictions, prefill,
     completed) = sc["metrics"]
    B = sc["config"][1]
    req = {r[0]: r for r in sc["requests"]}
    op, res, flag = t[:, 0], t[:, 5], t[:, 6]
    assert (op == STEP).sum() == steps
    assert ((op == APPEND) & (res == 1)).sum() == generated
    frees = t[op == FREE]
    assert (frees[:, 6] == FREE_FINISHED).sum() == completed
    assert (frees[:, 6] != FREE_FINISHED).sum() == preemptions
    assert frees[frees[:, 6] == FREE_DROPPED, 2].sum() == recomputed
    assert (-(-frees[frees[:, 6] == FREE_SWAPPED, 2] // B)).sum() == swap_out
    assert t[op == STEP][-1, 3] == cow and t[op == STEP][-1, 4] == evictions
    assert ((op == ADMIT_PREFIX) & (res == 1) & (flag == 1)).sum() == (frees[:, 6] == FREE_SWAPPED).sum()
    assert swap_in == swap_out
    del hits, prefill, req  # prefill tokens and cache hits are checked by the replay (they need the state)


def main():
    if not os.path.isdir(os.path.join(REF, "src")):
        sys.exit("the reference sources are needed to regenerate the traces")
    with tempfile.TemporaryDirectory() as tmp:
        scen = parse(build_and_run(tmp))
    arrays = {}
    for name, sc in scen.items():
        t = annotate(sc)
        check(sc, t)
        arrays[f"{name}_requests"] = np.asarray(sc["requests"], dtype=np.int64)
        arrays[f"{name}_config"] = np.asarray(sc["config"], dtype=np.int64)
        arrays[f"{name}_metrics"] = np.asarray(sc["metrics"], dtype=np.int64)
        arrays[f"{name}_trace"] = t
        print(name, "rows", len(t), "metrics", sc["metrics"])
    arrays["names"] = np.frombuffer(json.dumps(sorted(scen)).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
