"""The reference's own scheduler simulation driving the device data plane.

tests/golden/sim_traces.npz holds decision streams recorded from the reference's run_paged
(src/simulator.cpp:80-289) over the reference's own KVManager (tests/golden/simtrace/make_sim_traces.py), with
the reference's metrics, in three scenarios: FCFS with swap preemption, a persistent prefix cache and two
samples per request (fork + copy-on-write); shortest-prompt-first with recompute preemption and shared
prefixes; priority classes with displacement, a swap pool too small for every victim, and block size 8.

CPU: this package's KVManager re-makes every decision with the recorded result, matches every end-of-step
statistics marker, and the replay's totals (tokens, prefill tokens, cache hits, copy-on-write copies, swapped
blocks) equal the reference's metrics.

GPU: DataPlane replays the same streams with real K/V (synthetic rows that respect prefix groups and fork
lineage): prefill writes, copy-on-write copies, swap-out / swap-in through a pinned pool, and per-layer paged
attention with the new token fused in (or scattered first).  Every 20 steps (60 on the serving-scale stream)
each live request's context, gathered from the pools through its table, equals its logical rows bit for bit;
sampled attention batches match the fp64 oracle over the logical contexts (2e-3 abs + 2e-3 rel)."""
import importlib
import json
import os

import numpy as np
import pytest

from conftest import PKG

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sim_traces.npz")
NAMES = json.loads(bytes(np.load(GOLDEN)["names"]).decode())
L, KVH, D, NH = 2, 2, 64, 8


def _load(name):
    z = np.load(GOLDEN)
    return {k: z[f"{name}_{k}"] for k in ("requests", "config", "metrics", "trace")}


def _dp(kvb):
    return importlib.import_module(PKG + ".dataplane")


def _metrics(sc):
    keys = ("steps", "generated", "preemptions", "recomputed", "cow", "swap_out", "swap_in", "hits", "evictions",
            "prefill", "completed")
    return dict(zip(keys, (int(x) for x in sc["metrics"])))


def _max_swapped_blocks(dp, trace, B):
    """Host slots the replay needs: the peak of blocks sitting in the swap pool."""
    used = peak = 0
    held = {}
    for row in trace:
        if row[0] == dp.TRACE_FREE and row[6] == dp.FREE_SWAPPED:
            held[int(row[1])] = -(-int(row[2]) // B)
            used += held[int(row[1])]
            peak = max(peak, used)
        elif row[0] == dp.TRACE_ADMIT_PREFIX and row[6] == 1:
            used -= held.pop(int(row[1]))
    return peak


def test_fixture_covers_the_paths():
    for name in NAMES:
        m = _metrics(_load(name))
        assert m["completed"] > 30 and m["preemptions"] > 5
    by = {n: _metrics(_load(n)) for n in NAMES}
    assert any(m["swap_out"] > 0 for m in by.values()) and any(m["recomputed"] > 0 for m in by.values())
    assert any(m["cow"] > 0 for m in by.values()) and any(m["hits"] > 0 for m in by.values())
    assert any(m["evictions"] > 0 for m in by.values())


@pytest.mark.parametrize("name", NAMES)
def test_decisions_match_reference_simulation(kvb, name):
    dp = _dp(kvb)
    sc = _load(name)
    nb, B = (int(x) for x in sc["config"][:2])
    mgr = kvb.KVManager(nb, B)
    n = dp.replay_decisions(mgr, sc["trace"])
    m = _metrics(sc)
    assert (n.steps, n.tokens_generated, n.cow_copies) == (m["steps"], m["generated"], m["cow"])
    assert (n.swap_out_blocks, n.swap_in_blocks) == (m["swap_out"], m["swap_in"])
    assert (n.prefill_tokens, n.cache_hits) == (m["prefill"], m["hits"])
    assert mgr.validate() == "" and mgr.free_blocks() == nb


def test_a_wrong_decision_is_reported(kvb):
    dp = _dp(kvb)
    sc = _load(NAMES[0])
    nb, B = (int(x) for x in sc["config"][:2])
    t = sc["trace"].copy()
    i = int(np.nonzero((t[:, 0] == dp.TRACE_APPEND) & (t[:, 5] == 1))[0][5])
    t[i, 5] = 0  # plant a wrong recorded result
    with pytest.raises(dp.TraceMismatch):
        dp.replay_decisions(kvb.KVManager(nb, B), t)


def _oracle_check(ora, content, rids, q, out, B):
    ctx = [content(np.full(int(n), r, dtype=np.int64), np.arange(int(n), dtype=np.int64)) for r, n in rids]
    nblk = [-(-int(n) // B) for _, n in rids]
    tables = np.zeros((len(rids), max(nblk)), np.int32)
    lens = np.asarray([int(n) for _, n in rids], np.int32)
    b0 = 0
    for i, nbk in enumerate(nblk):
        tables[i, :nbk] = np.arange(b0, b0 + nbk)
        b0 += nbk
    for layer in range(L):
        K = np.zeros((b0 * B, KVH, D), np.float32)
        V = np.zeros_like(K)
        for i, (k, v) in enumerate(ctx):
            s = int(tables[i, 0]) * B
            K[s:s + lens[i]] = k[layer].float().cpu().numpy()
            V[s:s + lens[i]] = v[layer].float().cpu().numpy()
        ref = ora.reference_attention(NH, KVH, D, B, q[layer].float().cpu().numpy(), K.reshape(b0, B, KVH, D),
                                      V.reshape(b0, B, KVH, D), tables, lens)
        got = out[layer].float().cpu().numpy()
        assert (np.abs(got - ref) <= 2e-3 + 2e-3 * np.abs(ref)).all(), (layer, np.abs(got - ref).max())


def _contexts_check(plane, content):
    import torch
    torch.cuda.synchronize()
    for r in sorted(plane.tokens):
        n = plane.mgr.num_tokens(r)
        assert n == plane.tokens[r]
        idx = torch.tensor(plane.mgr.block_table(r), dtype=torch.long, device=plane.dev)
        gk = plane.k[:, idx].reshape(L, -1, KVH, D)[:, :n]
        gv = plane.v[:, idx].reshape(L, -1, KVH, D)[:, :n]
        ek, ev = content(np.full(n, r, dtype=np.int64), np.arange(n, dtype=np.int64))
        assert torch.equal(gk.view(torch.int16), ek.view(torch.int16)), f"K of request {r}"
        assert torch.equal(gv.view(torch.int16), ev.view(torch.int16)), f"V of request {r}"


@pytest.mark.gpu
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "scatter"])
@pytest.mark.parametrize("name", NAMES)
def test_replay_on_device(kvb, ora, cuda, name, fused):
    import torch
    dp = _dp(kvb)
    sc = _load(name)
    nb, B = (int(x) for x in sc["config"][:2])
    content = dp.SyntheticContent(sc["requests"], layers=L, kv_heads=KVH, head_dim=D, num_heads=NH, device=cuda,
                                  seed=5)
    batches = {"n": 0, "checked": 0}
    big = _metrics(sc)["steps"] > 400  # the serving-scale stream: sparser checks
    every_batch, every_step = (25, 60) if big else (9, 20)

    def on_attention(rids, q, out, tables, lens):
        batches["n"] += 1
        if batches["n"] % every_batch == 1:
            _oracle_check(ora, content, list(zip(rids, lens)), q, out, B)
            batches["checked"] += 1

    plane = dp.DataPlane(nb, B, layers=L, num_heads=NH, kv_heads=KVH, head_dim=D, source=content,
                         queries=content.queries, device=cuda, swap_slots=_max_swapped_blocks(dp, sc["trace"], B),
                         fused_append=fused, on_attention=on_attention)
    steps_checked = []

    def on_step(i):
        if i % every_step == 0:
            _contexts_check(plane, content)
            steps_checked.append(i)

    n = plane.run(sc["trace"], on_step=on_step)
    assert plane.status_word() == 0
    _contexts_check(plane, content)
    m = _metrics(sc)
    assert (n.steps, n.tokens_generated, n.cow_copies) == (m["steps"], m["generated"], m["cow"])
    assert (n.swap_out_blocks, n.swap_in_blocks) == (m["swap_out"], m["swap_in"])
    assert (n.prefill_tokens, n.cache_hits) == (m["prefill"], m["hits"])
    assert n.attention_rows == m["generated"]
    assert plane.mgr.free_blocks() == nb and not plane.tokens
    assert batches["checked"] >= 5 and len(steps_checked) >= 8
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_replay_llama_heads_with_strided_queries(kvb, ora, cuda):
    """The first 40 scheduler steps of the serving-scale stream at the Llama-3-8B head shape (32/8 heads,
    head_dim 128, 4 layers, bf16), with the queries of each batch a strided view of a larger bank (each layer's
    rows contiguous, the layers 512 rows apart), as the data-plane benchmark passes them: contexts bit-exact
    every 10 steps, and three rows of every fifth attention batch against the fp64 oracle on layers 0 and 3."""
    import torch
    dp = _dp(kvb)
    sc = _load("serving_fcfs_swap")
    nb, B = (int(x) for x in sc["config"][:2])
    t = sc["trace"]
    cut = int(np.nonzero(t[:, 0] == dp.TRACE_STEP)[0][39]) + 1
    trace = t[:cut]
    Lq, nh, kvh, Dq = 4, 32, 8, 128
    content = dp.SyntheticContent(sc["requests"], layers=Lq, kv_heads=kvh, head_dim=Dq, num_heads=nh, device=cuda,
                                  seed=9)
    bank = torch.randn((Lq, 512, nh, Dq), device=cuda).to(torch.bfloat16)
    seen = {"n": 0, "checked": 0}

    def queries(rids):
        return bank[:, :len(rids)]

    def on_attention(rids, q, out, tables, lens):
        seen["n"] += 1
        if seen["n"] % 5 != 1:
            return
        n = len(rids)
        for i in sorted({0, n // 2, n - 1}):
            ln = int(lens[i])
            k, v = content(np.full(ln, rids[i], dtype=np.int64), np.arange(ln, dtype=np.int64))
            nbk = -(-ln // B)
            for layer in (0, Lq - 1):
                K = np.zeros((nbk * B, kvh, Dq), np.float32)
                V = np.zeros_like(K)
                K[:ln] = k[layer].float().cpu().numpy()
                V[:ln] = v[layer].float().cpu().numpy()
                ref = ora.reference_attention(nh, kvh, Dq, B, q[layer, i:i + 1].float().cpu().numpy(),
                                              K.reshape(nbk, B, kvh, Dq), V.reshape(nbk, B, kvh, Dq),
                                              np.arange(nbk, dtype=np.int32)[None], np.asarray([ln], np.int32))
                got = out[layer, i:i + 1].float().cpu().numpy()
                assert (np.abs(got - ref) <= 2e-3 + 2e-3 * np.abs(ref)).all(), (layer, i, np.abs(got - ref).max())
        seen["checked"] += 1

    plane = dp.DataPlane(nb, B, layers=Lq, num_heads=nh, kv_heads=kvh, head_dim=Dq, source=content, queries=queries,
                         device=cuda, swap_slots=max(1, _max_swapped_blocks(dp, trace, B)), on_attention=on_attention)

    def contexts(i):
        if i % 10 == 0:
            torch.cuda.synchronize()
            for r in sorted(plane.tokens):
                n = plane.mgr.num_tokens(r)
                idx = torch.tensor(plane.mgr.block_table(r), dtype=torch.long, device=plane.dev)
                gk = plane.k[:, idx].reshape(Lq, -1, kvh, Dq)[:, :n]
                ek, _ = content(np.full(n, r, dtype=np.int64), np.arange(n, dtype=np.int64))
                assert torch.equal(gk.view(torch.int16), ek.view(torch.int16)), f"K of request {r}"

    n = plane.run(trace, on_step=contexts)
    assert plane.status_word() == 0
    assert n.steps == 40 and n.tokens_generated > 200 and seen["checked"] >= 6
