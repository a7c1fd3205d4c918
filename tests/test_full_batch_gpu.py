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


def test_decoder_pipelined_tinyllama_shape(kvb, ora, cuda):
    """The end-to-end leg of bench.py at the TinyLlama shape, checked: 256 requests (log-normal lengths, median
    1024), 22 layers, bf16, through the decoder with its packed pinned inputs and pipelined steps (submit, plan
    the next step, wait), 6 steps with new inputs each step.  After the last step, 16 sampled requests'
    outputs of the first and the last layer against the fp64 oracle on the pools and tables as the decoder
    left them, and their newest K/V rows equal to the last step's inputs."""
    import torch
    import bench
    cfg = _cfg("tinyllama-1.1b", 22)
    L, nh, kvh, D, B = cfg["L"], cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"]
    lens = bench.sample_lens(cfg, cfg["ns"], seed=1000)
    ns, steps = len(lens), 6
    dev = torch.device("cuda:0")
    mgr, kc, vc, nb = bench.setup_shard(kvb, cfg, lens, steps + 2, dev, seed=31)
    max_blocks = (int(lens.max()) + steps + 2 + B) // B
    dec = kvb.Decoder(mgr, kc, vc, nh, max_seqs=ns, max_blocks_per_seq=max_blocks)
    rids = np.arange(ns, dtype=np.int64)
    pq, pk, pv = dec.host_inputs(ns)
    out = torch.empty((L, ns, nh, D), dtype=torch.bfloat16).pin_memory()
    g = torch.Generator().manual_seed(5)
    dec.plan(rids)
    for s in range(steps):
        q = torch.randn((L, ns, nh, D), generator=g).to(torch.bfloat16)
        kn = torch.randn((L, ns, kvh, D), generator=g).to(torch.bfloat16)
        vn = torch.randn((L, ns, kvh, D), generator=g).to(torch.bfloat16)
        pq.copy_(q), pk.copy_(kn), pv.copy_(vn)
        dec.submit(rids, pq, pk, pv, out)
        if s + 1 < steps:
            dec.plan(rids)
        dec.wait()
    assert dec.status() == 0
    idx = [int(np.argmax(lens)), int(np.argmin(lens))] + \
        [int(i) for i in np.random.default_rng(2).choice(ns, 14, replace=False)]
    tables, got_lens = mgr.dense_tables([int(i) for i in idx], max_blocks)
    assert (got_lens == lens[idx] + steps).all()
    nblk = (got_lens + B - 1) // B
    T = np.zeros((len(idx), int(nblk.max())), np.int32)
    blocks, off = [], 0
    for j in range(len(idx)):
        blocks.extend(tables[j, :nblk[j]].tolist())
        T[j, :nblk[j]] = np.arange(off, off + nblk[j])
        off += int(nblk[j])
    bidx = torch.tensor(blocks, dtype=torch.long, device=dev)
    for layer in (0, L - 1):
        k = kc[layer].index_select(0, bidx)
        v = vc[layer].index_select(0, bidx)
        for j, i in enumerate(idx):  # the fused append of the last step: position len - 1
            p = int(got_lens[j]) - 1
            blk = int(T[j, p // B])
            assert torch.equal(k[blk, p % B].cpu(), kn[layer, i]) and torch.equal(v[blk, p % B].cpu(), vn[layer, i])
        ref = ora.reference_attention(nh, kvh, D, B, q[layer, idx].float().numpy(), k.float().cpu().numpy(),
                                      v.float().cpu().numpy(), T, got_lens)
        check_close(out[layer, idx].float().numpy(), ref, out_dtype="bf16", what=f"decoder layer {layer}")
