"""Parity at the benchmark's own scale: the decode step bench.py times (bench.DecodeStep -- fused append, the
balanced schedule over one zero-filled workspace with KVP_ATTN_WORKSPACE_CLEAN, early load, one CUDA graph per
step) run over the full batch of 256 requests, with sampled outputs checked against the fp64 oracle
(reference_attention, src/paged_attention.cpp:25-66) on the K/V the pool holds after the step, and the rows
the fused append wrote checked against the new K/V bit for bit.

Tolerance: |got - ref| <= 2e-3 + (2e-3 + 2^-8) |ref| (bf16 outputs add half an ulp), as in
test_attention_gpu.check_close.
"""
import ctypes

import numpy as np
import pytest

from test_attention_gpu import check_close

pytestmark = pytest.mark.gpu


def _workload(kvb, cfg, lens, steps, seed):
    import torch
    import bench
    dev = torch.device("cuda:0")
    mgr, kc, vc, nb = bench.setup_shard(kvb, cfg, lens, steps, dev, seed=seed)
    st = bench.DecodeStep(kvb, cfg, mgr, kc, vc, nb, len(lens), steps, dev, seed=seed + 1, rows_per_step=True)
    return st, dev


def _check_step(ora, st, s, layers, what):
    cfg = st.cfg
    idx = st.sample_rows(s, n=16, seed=s)
    smp = st.parity_sample(s, layers, idx)
    for l, d in smp["layers"].items():
        assert d["appended_ok"], f"{what}: step {s} layer {l}: the fused append's rows differ from the new K/V"
        ref = ora.reference_attention(cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"], d["q"], d["k"], d["v"],
                                      smp["tables"], smp["lens"])
        check_close(d["out"], ref, out_dtype=cfg["dtype"], what=f"{what}: step {s} layer {l}")
    return smp["lens"]


def _cfg(name, layers):
    import bench
    cfg = dict(bench.CONFIGS[name])
    cfg["L"] = layers
    cfg["pool_gb"], cfg["pool_blocks"] = None, None  # pool sized to the shard
    return cfg


@pytest.mark.parametrize("short", [False, True], ids=["bench-lengths", "with-one-tile-requests"])
def test_llama3_8b_shape_full_batch(kvb, ora, cuda, short):
    """The Llama-3-8B-shaped step at its full batch: 256 requests with the bench's own lengths (log-normal,
    median 4096, clipped to 32768, seed 1000), 2 layers, 3 eager steps then the graphs of all 6 steps replayed --
    the bench's warm-up and timed sequence -- checked after the last eager step and after the last replay.  The
    second variant gives four requests short contexts (1, 15, 16 and 17 tokens before the steps), so the sample
    also holds a sequence that fits one tile."""
    import torch
    import bench
    cfg = _cfg("llama3-8b", 2)
    lens = bench.sample_lens(cfg, cfg["ns"], seed=1000)
    if short:
        lens[:4] = [1, 15, 16, 17]
    W, K = 3, 3
    st, dev = _workload(kvb, cfg, lens, W + K, seed=11)
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for s in range(W):
        st.launch(s, sp)
    torch.cuda.synchronize()
    assert int(st.status.item()) == 0
    _check_step(ora, st, W - 1, [0, 1], "eager")
    graphs = st.capture(range(W + K))
    for s in range(W + K):
        graphs[s].replay()
    torch.cuda.synchronize()
    assert int(st.status.item()) == 0
    got_lens = _check_step(ora, st, W + K - 1, [0, 1], "graph replay")
    if short:
        assert got_lens.min() <= 16  # the sample holds the shortest request: a context of one tile
    del graphs


def test_tinyllama_shape_128_step_loop(kvb, ora, cuda):
    """The TinyLlama-shaped decode loop as specified: 256 requests (log-normal, median 1024, clipped to 2048),
    all 22 layers, 128 steps replayed from CUDA graphs with a fused append every step (different new K/V each
    step), checked every 32 steps (first and last layer, 16 requests including the longest and shortest)."""
    import torch
    import bench
    cfg = _cfg("tinyllama-1.1b", 22)
    lens = bench.sample_lens(cfg, cfg["ns"], seed=1000)
    steps = 128
    st, dev = _workload(kvb, cfg, lens, steps, seed=21)
    graphs = st.capture(range(steps))
    for s in range(steps):
        graphs[s].replay()
        if (s + 1) % 32 == 0:
            torch.cuda.synchronize()
            assert int(st.status.item()) == 0, s
            _check_step(ora, st, s, [0, cfg["L"] - 1], "128-step loop")
    del graphs
