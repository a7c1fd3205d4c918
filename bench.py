"""Decode-step benchmark of the paged KV-cache data plane on B200.

A step = one decode step of every request of this GPU's shard: the host KVManager appends one token per
request (slots, copy-on-write pairs, new table entries), and one paged decode attention launch per layer
writes the layer's new K/V into its slot (fused append) and attends over every context.  Default workload: the Llama-3-8B-shaped
request-sharded config (32 query / 8 kv heads, head_dim 128, 32 layers, block 16, bf16, 256 requests per
GPU, context lengths log-normal with median 4096 clipped to 32768, a pool of about 150 GB per GPU).
Inputs are synthetic, seeded N(0,1).

  value : decode tokens/s over all GPUs with every input already resident in HBM (device timed; each step's
          per-layer launches replayed from a CUDA graph, or launched from Python with --eager)
  e2e   : the same step through the C ABI with host buffers: per-layer queries and new K/V copied from pinned
          host memory, the host KVManager step, and the attention output copied back, inside the timed region
          (the requests regrown to the value run's starting lengths; each step's bookkeeping planned while the
          previous step runs)
  roofline : the attention kernel's algorithmic bytes (unique K/V bytes of the contexts) per launch / its
          average duration (CUDA events around each launch with --eager; otherwise the replayed steps' CUDA-event
          time over their launches, gaps between launches included), against the measured HBM copy peak
  cpu_baseline : the reference's own CPU paged_attention_cpu (oracle/_ref) on a bounded sample, all host cores
  --impl reference : that CPU baseline as its own line, plus (reference_gpu_kernel) the reference's own GPU
          kernel built from its source, timed on one layer of a 32-request sample of the same workload

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config llama3-8b|...]
       python bench.py --op migrate|cow|swap   (block movers: one process; migrate reads GPU 1's pool into
                                                GPU 0's over NVLink when two GPUs are visible; swap moves blocks
                                                to a pinned host pool and back)
       python bench.py --op sim                (the reference scheduler's recorded serving stream replayed by
                                                the data plane: prefill, append, copy-on-write, swap, attention)
       python bench.py --op latency            (per-call latency of the small 8-sequence case, the drop-in
                                                entry point included)
Multi-GPU: launched under torch.distributed.run, one process per GPU, requests sharded with no collective
on the data path (weak scaling); timings are the max over ranks.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: heads, kv heads, head_dim, layers, block, requests per GPU, kv dtype, length sampler, pool target
    "llama3-8b": dict(nh=32, kvh=8, D=128, L=32, B=16, ns=256, dtype="bf16", lens=("lognormal", 4096, 0.35, 32768),
                      pool_gb=150.0),
    "qwen2.5-0.5b": dict(nh=14, kvh=2, D=64, L=24, B=16, ns=64, dtype="f16", lens=("uniform", 512, 4096),
                         pool_blocks=65536),
    "tinyllama-1.1b": dict(nh=32, kvh=4, D=64, L=22, B=16, ns=256, dtype="bf16", lens=("lognormal", 1024, 0.5, 2048),
                           pool_gb=None),
}
DEFAULT = "llama3-8b"


def sample_lens(cfg, ns, seed):
    rng = np.random.default_rng(seed)
    kind = cfg["lens"][0]
    if kind == "uniform":
        return rng.integers(cfg["lens"][1], cfg["lens"][2] + 1, size=ns).astype(np.int64)
    _, med, sigma, cap = cfg["lens"]
    x = np.round(rng.lognormal(math.log(med), sigma, size=ns))
    return np.clip(x, 1, cap).astype(np.int64)


def block_bytes_all_layers(cfg):
    return 2 * cfg["L"] * cfg["B"] * cfg["kvh"] * cfg["D"] * 2


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.p is not None:
            time.sleep(0.25)
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()
                out, _ = self.p.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU baseline
def _random_sample(cfg, sl, seed, pool_blocks=None):
    """A CPU-side sample of the workload: requests of context lengths `sl`, N(0,1) fp32 K/V/Q.  Without
    `pool_blocks` each request's blocks are a random permutation of a pool of exactly their blocks; with it,
    tables draw ids from a smaller shared pool (filled by tiling a 64 MB random chunk), which keeps host memory
    and set-up time bounded while every request still reads blocks scattered over DRAM."""
    nh, kvh, D, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"]
    rng = np.random.default_rng(seed)
    sl = np.asarray(sl, np.int32)
    ns = len(sl)
    nblk = (sl + B - 1) // B
    T = np.zeros((ns, int(nblk.max())), np.int32)
    if pool_blocks is None:
        pool = int(nblk.sum())
        K = rng.standard_normal((pool, B, kvh, D), dtype=np.float32)
        V = rng.standard_normal((pool, B, kvh, D), dtype=np.float32)
        perm = rng.permutation(pool).astype(np.int32)
        o = 0
        for i in range(ns):
            T[i, : nblk[i]] = perm[o: o + nblk[i]]
            o += int(nblk[i])
    else:
        pool = int(pool_blocks)
        K = np.empty((pool, B, kvh, D), np.float32)
        V = np.empty((pool, B, kvh, D), np.float32)
        for t in (K, V):
            chunk = rng.standard_normal(min(t.size, 16 << 20), dtype=np.float32)
            flat = t.reshape(-1)
            for o in range(0, flat.size, chunk.size):
                m = min(chunk.size, flat.size - o)
                flat[o:o + m] = chunk[:m]
        for i in range(ns):
            T[i, : nblk[i]] = rng.integers(0, pool, size=nblk[i], dtype=np.int32)
    Q = rng.standard_normal((ns, nh, D), dtype=np.float32)
    return Q, K, V, T, sl


def _time_cpu(cfg, Q, K, V, T, sl, target_s, impl, cores):
    """Seconds per paged_attention_cpu call (partitions 1, `cores` threads) over about target_s."""
    import oracle
    nh, kvh, D, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"]
    oracle.paged_attention_cpu(nh, kvh, D, B, Q, K, V, T, sl, partitions=1, nthreads=cores, impl=impl)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.paged_attention_cpu(nh, kvh, D, B, Q, K, V, T, sl, partitions=1, nthreads=cores, impl=impl)
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s or reps >= 1000:
            break
    return el / reps, reps, el


def check_parity(cfg, sample):
    """The GPU's outputs of the timed step's last launch for the sampled requests against the fp64
    reference_attention (the reference library's own function when it is built, else the oracle's C
    restatement) on the same K/V, queries and tables; and the rows the fused append wrote.  Tolerance:
    |got - ref| <= 2e-3 + (2e-3 + half an ulp of the output dtype) |ref|."""
    import oracle
    nh, kvh, D, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"]
    impl = "ref" if oracle.have_ref() else "c"
    half_ulp = {"bf16": 2.0 ** -8, "f16": 2.0 ** -11}[cfg["dtype"]]
    worst_abs, worst_excess, appended = 0.0, -1.0, True
    for l, d in sample["layers"].items():
        ref = oracle.reference_attention(nh, kvh, D, B, d["q"], d["k"], d["v"], sample["tables"], sample["lens"],
                                         impl=impl)
        got = d["out"]
        finite = bool(np.isfinite(got).all())
        err = np.abs(got - ref)
        worst_abs = max(worst_abs, float(err.max()) if finite else float("inf"))
        worst_excess = max(worst_excess, float((err - (2e-3 + (2e-3 + half_ulp) * np.abs(ref))).max())
                           if finite else float("inf"))
        appended &= d["appended_ok"]
    n = len(sample["lens"])
    return {"checked": n * len(sample["layers"]), "requests": n, "layers": sorted(sample["layers"]),
            "context_tokens": [int(sample["lens"].min()), int(sample["lens"].max())],
            "max_abs_err": worst_abs, "max_excess_over_tolerance": worst_excess, "appended_rows_ok": appended,
            "ok": bool(worst_excess <= 0 and appended),
            "oracle": "reference_attention (fp64) of the " + ("reference library" if impl == "ref" else
                                                               "oracle's C restatement"),
            "tolerance": "2e-3 abs + (2e-3 + half an ulp of the output dtype) rel"}


def cpu_layer_workload(cfg, lens):
    """What the reference's CPU code is timed on: one layer of every request of the shard, its own context
    length, N(0,1) fp32 data, tables drawing their blocks from a shared pool of at most 16,384 blocks (so host
    memory and set-up stay bounded while every request still reads blocks scattered over DRAM).  One call is
    1/L of a decode step, and every host thread has many requests to work through."""
    pool = min(int(((lens + cfg["B"] - 1) // cfg["B"]).sum()), 16384)
    return _random_sample(cfg, lens, seed=77, pool_blocks=pool), pool


def cpu_baseline(cfg, lens, target_s=12.0, kind_pref="reference", sample=None):
    """Times the reference's paged_attention_cpu (the reference library built here, else the oracle's
    restatement) on all host cores over cpu_layer_workload() for about target_s (at least one call), and scales
    it to decode tok/s = requests / (L x seconds per call).  With `sample` (DecodeStep.parity_sample of the last
    timed step: 16 of its requests, the first and last layer, copied off the device after the timed region) this
    leg also checks the GPU's outputs for those requests (check_parity).  Returns (baseline, parity)."""
    import oracle
    kind = "reference" if (kind_pref == "reference" and oracle.have_ref()) else "port"
    impl = "ref" if kind == "reference" else "c"
    kvh, D = cfg["kvh"], cfg["D"]
    cores = os.cpu_count() or 1
    parity = check_parity(cfg, sample) if sample is not None else None
    (Q, K, V, T, sl), pool = cpu_layer_workload(cfg, lens)
    per_call, reps, el = _time_cpu(cfg, Q, K, V, T, sl, target_s, impl, cores)
    gbs = float(sl.sum()) * kvh * D * 2 * 2 / per_call / 1e9  # the GPU's byte formula
    return {"value": len(lens) / (cfg["L"] * per_call), "unit": "tok/s", "cores": cores, "kind": kind,
            "gb_s": round(gbs, 3),
            "sample": f"one layer of all {len(sl)} requests per call ({int(sl.sum())} context tokens; tables over a "
                      f"shared pool of {pool} blocks), {reps} timed calls over {el:.1f}s, x {cfg['L']} layers"}, parity


def reference_gpu_kernel(cfg, lens, nseq=32):
    """The reference's own GPU kernel (cuda/paged_attention.cu, built from its source into oracle/_ref; fp16
    only) timed on one layer of a bounded sample of this workload -- `nseq` requests drawn from the same
    lengths, random block tables over a pool of exactly their blocks -- with CUDA events, at 4 and 8 warps
    (the better is reported).  Reported beside the CPU baseline as extra context; None without a GPU or the
    built kernel."""
    try:
        import torch
        import oracle
    except Exception:
        return None
    if not torch.cuda.is_available() or not oracle.have_ref_gpu():
        return None
    nh, kvh, D, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"]
    rng = np.random.default_rng(78)
    sl = rng.choice(lens, size=nseq, replace=True).astype(np.int32)
    nblk = (sl + B - 1) // B
    pool = int(nblk.sum())
    perm = rng.permutation(pool).astype(np.int32)
    T = np.zeros((nseq, int(nblk.max())), np.int32)
    o = 0
    for i in range(nseq):
        T[i, :nblk[i]] = perm[o:o + nblk[i]]
        o += int(nblk[i])
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    k = torch.randn((pool, B, kvh, D), generator=g, device=dev).half()
    v = torch.randn((pool, B, kvh, D), generator=g, device=dev).half()
    q = torch.randn((nseq, nh, D), generator=g, device=dev).half()
    out = torch.empty_like(q)
    t, ln = torch.from_numpy(T).to(dev), torch.from_numpy(sl).to(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    for warps in (4, 8):
        def call():
            rc = oracle.ref_gpu_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), t.data_ptr(), ln.data_ptr(),
                                          out.data_ptr(), nseq, nh, kvh, D, B, T.shape[1], warps, stream.cuda_stream)
            assert rc == 0, rc
        call()
        torch.cuda.synchronize(dev)
        reps = 5
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        if best is None or ms < best[0]:
            best = (ms, warps)
    ms, warps = best
    sample_bytes = float(sl.sum()) * kvh * D * 2 * 2
    gbs = sample_bytes / (ms / 1e3) / 1e9
    step_bytes = float(lens.sum()) * kvh * D * 2 * 2 * cfg["L"]
    return {"value": round(len(lens) / (step_bytes / (gbs * 1e9)), 2), "unit": "tok/s", "gb_s": round(gbs, 1),
            "ms_per_layer_sample": round(ms, 3), "warps": warps, "dtype": "f16",
            "sample": f"{nseq} requests x 1 layer ({int(sl.sum())} tokens, lengths drawn from the workload), fp16 "
                      f"(the kernel's only type; same bytes as bf16), scaled to {len(lens)} requests x {cfg['L']} "
                      f"layers by its GB/s"}


# ----------------------------------------------------------------------------- GPU workload
def setup_shard(kvb, cfg, lens, steps_total, dev, seed):
    """Pool, manager and fragmented block tables for one GPU's shard."""
    import torch
    B, L, kvh, D = cfg["B"], cfg["L"], cfg["kvh"], cfg["D"]
    ns = len(lens)
    need_blocks = int(((lens + steps_total + B) // B + 1).sum()) + 64
    free, _ = torch.cuda.mem_get_info(dev)
    bb = block_bytes_all_layers(cfg)
    if cfg.get("pool_blocks"):
        nb = int(cfg["pool_blocks"])
    elif cfg.get("pool_gb"):
        nb = int(cfg["pool_gb"] * 1e9 // bb)
    else:
        nb = need_blocks
    nb = max(nb, need_blocks)
    cap = int((free - 14e9) // bb)
    if nb > cap:
        nb = cap
    if nb < need_blocks:
        raise RuntimeError(f"pool of {nb} blocks cannot hold the shard ({need_blocks} needed)")
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    kc = torch.empty((L, nb, B, kvh, D), dtype=tdt, device=dev)
    vc = torch.empty((L, nb, B, kvh, D), dtype=tdt, device=dev)
    # Fill the pools with N(0,1): a 2 GiB random chunk, tiled (generating 150 GB with the RNG would dominate).
    g = torch.Generator(device=dev).manual_seed(seed)
    chunk = torch.randn(min(1 << 30, kc.numel()), generator=g, device=dev, dtype=torch.float32).to(tdt)
    for t in (kc, vc):
        flat = t.view(-1)
        for o in range(0, flat.numel(), chunk.numel()):
            n = min(chunk.numel(), flat.numel() - o)
            flat[o: o + n].copy_(chunk[:n])
    del chunk
    torch.cuda.empty_cache()
    mgr = kvb.KVManager(nb, B)
    grow_requests(mgr, lens, B, seed + 1)
    return mgr, kc, vc, nb


def grow_requests(mgr, lens, B, seed):
    """Requests 0 .. len(lens)-1 admitted empty, then grown block by block in a random interleaving to their
    lengths, so tables are fragmented the way a long-running server's are."""
    for r in range(len(lens)):
        assert mgr.admit(r, 0)
    rng = np.random.default_rng(seed)
    remaining = np.asarray(lens).copy()
    while remaining.max() > 0:
        order = rng.permutation(np.nonzero(remaining > 0)[0])
        rids = []
        for r in order:
            k = int(min(B, remaining[r]))
            rids.extend([int(r)] * k)
            remaining[r] -= k
        done, _, _ = mgr.append_batch(rids)
        assert done == len(rids)


class DecodeStep:
    """The timed decode step of one GPU shard, built once and reused by the benchmark and by the full-batch
    tests (so both run the same launch plan): the host KVManager is advanced `n_steps` steps up front (one
    append per request per step, lengths recorded per step; the table after the last step serves every step,
    as entries past a sequence are never read), and step s is one kvp_paged_attention launch per layer with the
    fused append of the layer's new K/V at position len - 1, the balanced schedule over one zero-filled
    workspace (KVP_ATTN_WORKSPACE_CLEAN) and early load (each layer's launch may start and load K/V during the
    previous one).  `rows_per_step`: the new K/V rows differ from step to step (else one set serves all)."""

    def __init__(self, kvb, cfg, mgr, kc, vc, nb, ns, n_steps, dev, seed, split=0, wph=0, stages=0,
                 seq_start_tiles=0, rows_per_step=False):
        import ctypes
        import torch
        nh, kvh, D, L, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["L"], cfg["B"]
        self.kvb, self.cfg, self.kc, self.vc, self.nb, self.dev, self.ns = kvb, cfg, kc, vc, nb, dev, ns
        rids = list(range(ns))
        self.lens_all = np.empty((n_steps, ns), np.int32)
        for s in range(n_steps):
            done, _, pairs = mgr.append_batch(rids)
            assert done == ns and len(pairs) == 0
            self.lens_all[s] = [mgr.num_tokens(r) for r in rids]
        self.max_blocks = (int(self.lens_all[-1].max()) + B - 1) // B + 1
        self.tables, _ = mgr.dense_tables(rids, self.max_blocks, pad=0)
        self.d_tables = torch.from_numpy(self.tables).to(dev)
        self.d_lens = torch.from_numpy(self.lens_all).to(dev)
        tdt = kc.dtype
        g = torch.Generator(device=dev).manual_seed(seed)
        self.q = torch.randn((L, ns, nh, D), generator=g, device=dev).to(tdt)
        nrows = n_steps if rows_per_step else 1
        self.knew = torch.randn((nrows, L, ns, kvh, D), generator=g, device=dev).to(tdt)
        self.vnew = torch.randn((nrows, L, ns, kvh, D), generator=g, device=dev).to(tdt)
        self.out = torch.empty((L, ns, nh, D), device=dev, dtype=tdt)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.split = split
        a0 = kvb.attention_args(self.q[0], kc[0], vc[0], self.d_tables, self.d_lens[0], self.out[0], nh, kvh,
                                num_blocks=nb, split_tiles=split, warps_per_kv_head=wph, stages=stages,
                                seq_start_tiles=seq_start_tiles)
        self.ws = torch.zeros(max(kvb.workspace_bytes(a0), 256), dtype=torch.uint8, device=dev)
        # Launch arguments are built once; a step only repoints the lengths and new rows, so the timed loop
        # measures the kernels, not Python.
        self.args = []
        for l in range(L):
            a = kvb.attention_args(self.q[l], kc[l], vc[l], self.d_tables, self.d_lens[0], self.out[l], nh, kvh,
                                   num_blocks=nb, split_tiles=split, status=self.status, warps_per_kv_head=wph,
                                   stages=stages, seq_start_tiles=seq_start_tiles, k_new=self.knew[0, l],
                                   v_new=self.vnew[0, l])
            a.workspace, a.workspace_bytes = self.ws.data_ptr(), self.ws.numel()
            # zero-filled once, every call leaves the counters zero; lengths and tables are never written by a
            # kernel and a layer's kernel writes only its own pool, so each layer's launch may start and load K/V
            # during the previous one
            a.flags = kvb.KVP_ATTN_WORKSPACE_CLEAN | kvb.KVP_ATTN_EARLY_LOAD
            self.args.append(a)
        self.lib = kvb.lib()
        self._ct = ctypes
        self.lens_row = self.d_lens.stride(0) * 4
        # launches per layer: one (balanced schedule, or unsplit contexts), two with fixed splits (+ merge)
        self.per_layer = 1 if split == 0 or split >= (self.max_blocks * B + 15) // 16 or split < 0 else 2

    def launch(self, s, stream_ptr, ev=None, stream=None):
        """Step s's per-layer launches on a stream (events around each launch when `ev` is given)."""
        lp = self.d_lens.data_ptr() + s * self.lens_row
        row = s if self.knew.shape[0] > 1 else 0
        for l, a in enumerate(self.args):
            a.seq_lens = lp
            a.k_new, a.v_new = self.knew[row, l].data_ptr(), self.vnew[row, l].data_ptr()
            if ev is not None:
                ev[l][0].record(stream)
            rc = self.lib.kvp_paged_attention(self._ct.byref(a), stream_ptr)
            assert rc == 0, self.kvb.last_error()
            if ev is not None:
                ev[l][1].record(stream)

    def capture(self, steps):
        """One CUDA graph per step (its lengths row and new rows are baked into the launches)."""
        import torch
        graphs = []
        cap = torch.cuda.Stream(self.dev)
        for s in steps:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap, capture_error_mode="thread_local"):
                self.launch(s, self._ct.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream))
            graphs.append(g)
        return graphs

    def sample_rows(self, s, n=16, seed=0):
        """Requests whose outputs a parity check reads after step s: the longest and the shortest context,
        the rest drawn at random (seeded)."""
        lens = self.lens_all[s]
        pick = [int(np.argmax(lens)), int(np.argmin(lens))]
        rest = [i for i in np.random.default_rng(seed).permutation(self.ns).tolist() if i not in pick]
        return pick + rest[:max(0, n - 2)]

    def parity_sample(self, s, layers, idx):
        """What a CPU check of step s needs, copied out of the device after it ran (no checking here): per
        layer, the sampled requests' queries and outputs (fp32), their K/V blocks gathered into a compact pool
        (fp32, exact) with the tables renumbered into it, and whether the pool holds the step's new K/V rows at
        each sampled request's position len - 1 (the fused append's writes)."""
        import torch
        B = self.cfg["B"]
        lens = self.lens_all[s][idx].astype(np.int32)
        nblk = (lens + B - 1) // B
        T = np.zeros((len(idx), int(nblk.max())), np.int32)
        blocks, off = [], 0
        for j, i in enumerate(idx):
            blocks.extend(self.tables[i, :nblk[j]].tolist())
            T[j, :nblk[j]] = np.arange(off, off + nblk[j])
            off += int(nblk[j])
        bidx = torch.tensor(blocks, dtype=torch.long, device=self.dev)
        ridx = torch.tensor(idx, dtype=torch.long, device=self.dev)
        pos = lens - 1
        slot_blk = torch.tensor([int(self.tables[i, p // B]) for i, p in zip(idx, pos)], dtype=torch.long,
                                device=self.dev)
        slot_off = torch.tensor((pos % B).tolist(), dtype=torch.long, device=self.dev)
        row = s if self.knew.shape[0] > 1 else 0
        out = {"lens": lens, "tables": T, "layers": {}}
        for l in layers:
            kc, vc = self.kc[l], self.vc[l]
            out["layers"][l] = {
                "q": self.q[l].index_select(0, ridx).float().cpu().numpy(),
                "out": self.out[l].index_select(0, ridx).float().cpu().numpy(),
                "k": kc.index_select(0, bidx).float().cpu().numpy(),
                "v": vc.index_select(0, bidx).float().cpu().numpy(),
                "appended_ok": bool(torch.equal(kc[slot_blk, slot_off], self.knew[row, l].index_select(0, ridx)) and
                                    torch.equal(vc[slot_blk, slot_off], self.vnew[row, l].index_select(0, ridx))),
            }
        return out


def _per_rank_ms(ms, world, dev):
    """Every rank's device-timed milliseconds (one entry per rank, in rank order)."""
    if world == 1:
        return [ms]
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def run_ours(args, cfg, rank, world, dev):
    import ctypes
    import torch
    import torch.distributed as dist
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
    kvb.lib()
    nh, kvh, D, L, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["L"], cfg["B"]
    # The whole job's requests (ns per GPU) are sampled once and sharded by context length, longest first
    # (sharding.assign_requests); each rank serves its shard with its own pool and KVManager.
    sh = importlib.import_module("paged-kv-cache-manager_b200.sharding")
    all_lens = sample_lens(cfg, cfg["ns"] * world, seed=1000)
    rank_of = sh.assign_requests(all_lens.tolist(), world)
    lens = all_lens[sh.shard_of(rank_of, rank)]
    ns = len(lens)
    W, K = args.warmup, args.steps
    steps_total = W + K + 2  # the value run's steps; the e2e run regrows the requests and takes W + K + 1
    mgr, kc, vc, nb = setup_shard(kvb, cfg, lens, steps_total, dev, seed=rank * 7 + 1)
    tdt = kc.dtype
    rids = list(range(ns))
    max_len = int(lens.max()) + steps_total + 1
    max_blocks = (max_len + B - 1) // B
    # Device-resident inputs for the value run; each step's attention launch writes the new token of its layer
    # into the slot at position len - 1 (fused append).
    stepper = DecodeStep(kvb, cfg, mgr, kc, vc, nb, ns, W + K, dev, seed=99 + rank, split=args.split,
                         wph=args.wph, stages=args.stages, seq_start_tiles=args.seq_start_tiles)
    lens_all, split, per_layer, status = stepper.lens_all, stepper.split, stepper.per_layer, stepper.status
    stream = torch.cuda.current_stream(dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    for s in range(W):
        stepper.launch(s, sptr)
    torch.cuda.synchronize(dev)
    # A step's per-layer launches are replayed from a CUDA graph (one per step), so launch-bound small steps are
    # not timed at the host's launch rate.
    graphs = []
    if not args.eager:
        graphs = stepper.capture(range(W + K))
        for s in range(W):
            graphs[s].replay()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
           for _ in range(K)] if args.eager else None
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device() if dev.index is None else dev.index) as clk:
        t_start.record(stream)
        for s in range(K):
            if args.eager:
                stepper.launch(W + s, sptr, evs[s], stream)
            else:
                graphs[W + s].replay()
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    ms_total = t_start.elapsed_time(t_end)
    # per launch: CUDA events around each launch (eager), or the replayed step time over its launches
    attn_ms = ([e0.elapsed_time(e1) for row in evs for (e0, e1) in row] if args.eager else [ms_total / (K * L)])
    del graphs
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    # algorithmic bytes per attention launch: unique K/V bytes of every context, averaged over the steps
    elem = 2
    bytes_per_launch = float(lens_all[W:].astype(np.float64).sum(axis=1).mean()) * kvh * D * 2 * elem
    # What the CPU-baseline leg checks the last timed step against (copied out after the timed region, before
    # the end-to-end leg moves the pools on): 16 requests, the first and the last layer.
    sample = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        last = W + K - 1
        sample = stepper.parity_sample(last, sorted({0, L - 1}), stepper.sample_rows(last))
    per_rank = _per_rank_ms(ms_total, world, dev)

    if args.no_e2e:
        vals = torch.tensor([ms_total, ms_total, float(np.mean(attn_ms))], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ms_total, e2e_ms, attn_avg = [float(x) for x in vals.cpu()]
        gpu_launches = K * L * per_layer
        return dict(ms_total=ms_total, e2e_ms=e2e_ms, attn_avg_ms=attn_avg, bytes_per_launch=bytes_per_launch,
                    clocks=clk.summary(), ns=ns, nb=nb, split=split, gpu_launches=gpu_launches, h2d=0, d2h=0,
                    lens_mean=float(lens.mean()), per_rank_ms=per_rank, sample=sample), lens

    # ---------------------------------------------------------------- e2e through the C ABI, host buffers
    # Per decode step through the decoder's C ABI: host KVManager appends, metadata upload, new K/V and per-layer
    # queries copied in from pinned host memory, copy-on-write + fused append/attention for every layer, and
    # each layer's output copied back, with the copies overlapping the attention of other layers; the next
    # step's appends are planned while the step runs (kvp_decoder_submit / plan / wait).
    h_q = torch.randn((L, ns, nh, D), generator=torch.Generator().manual_seed(5)).to(tdt).pin_memory()
    h_k = torch.randn((L, ns, kvh, D), generator=torch.Generator().manual_seed(6)).to(tdt).pin_memory()
    h_v = torch.randn((L, ns, kvh, D), generator=torch.Generator().manual_seed(7)).to(tdt).pin_memory()
    h_out = torch.empty((L, ns, nh, D), dtype=tdt).pin_memory()
    del stepper
    torch.cuda.empty_cache()
    # The requests are freed and regrown to their starting lengths (new fragmented tables over the same pool),
    # so the e2e run's W + K steps attend over the same context lengths as the value run's.
    for r in rids:
        mgr.free(r)
    grow_requests(mgr, lens, B, seed=rank * 7 + 3)
    dec = kvb.Decoder(mgr, kc, vc, nh, max_seqs=ns, max_blocks_per_seq=max_blocks)
    rids = np.arange(ns, dtype=np.int64)  # the batch as the C ABI takes it (no per-step conversion)
    # the step's inputs produced in place in the decoder's pinned input buffers (a layer's queries and new K/V
    # adjacent, so each group of layers goes up in one copy)
    p_q, p_k, p_v = dec.host_inputs(ns)
    p_q.copy_(h_q), p_k.copy_(h_k), p_v.copy_(h_v)

    def e2e_step():
        # a serving loop's step: submit it (inputs copied up, launches), plan the next step's bookkeeping while
        # it runs, then wait for its outputs to reach the host
        dec.submit(rids, p_q, p_k, p_v, h_out)
        dec.plan(rids)
        dec.wait()

    dec.plan(rids)
    for _ in range(W):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    wall_ms = (time.perf_counter() - t0) * 1e3
    # the decoder works on its own streams and returns after its outputs reached the host: the host wall clock
    # over the K steps is the end-to-end time (the events on the default stream bracket the same interval)
    e2e_ms = max(wall_ms, e0.elapsed_time(e1))
    assert dec.status() == 0
    h2d = int(h_q.numel() * 2 + h_k.numel() * 2 + h_v.numel() * 2 + (ns * max_blocks + ns) * 4)

    # max over ranks (device-timed)
    vals = torch.tensor([ms_total, e2e_ms, float(np.mean(attn_ms))], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms, attn_avg = [float(x) for x in vals.cpu()]
    clocks = clk.summary()
    gpu_launches = K * L * per_layer  # the device-timed value region
    res = dict(ms_total=ms_total, e2e_ms=e2e_ms, attn_avg_ms=attn_avg, bytes_per_launch=bytes_per_launch,
               clocks=clocks, ns=ns, nb=nb, split=split, gpu_launches=gpu_launches,
               h2d=h2d, d2h=int(h_out.numel() * 2), lens_mean=float(lens.mean()), per_rank_ms=per_rank,
               sample=sample)
    return res, lens


def run_swap(args, cfg):
    """Swap (preemption) traffic, device timed: a step swaps 512 random config blocks (every layer, K and V) out
    to a pinned host pool (kvp_swap_out) and back into fresh block ids (kvp_swap_in), on a side stream as the
    decode runtime issues them.  Reports GB/s per direction against the host link."""
    import torch
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
    L, B, kvh, D = cfg["L"], cfg["B"], cfg["kvh"], cfg["D"]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    nblk, nb = 512, 2048
    dev = torch.device("cuda", 0)
    k = torch.empty((L, nb, B, kvh, D), dtype=tdt, device=dev)
    v = torch.empty_like(k)
    k.view(torch.int16).random_(-30000, 30000)
    v.view(torch.int16).random_(-30000, 30000)
    slot = kvb.host_slot_bytes(L, B, kvh, D)
    pool = torch.empty(slot * nblk, dtype=torch.uint8).pin_memory()
    rng = np.random.default_rng(0)
    side = torch.cuda.Stream(dev)
    steps = args.warmup + args.steps
    outs = [rng.permutation(nb)[:nblk].tolist() for _ in range(steps)]
    ins = [rng.permutation(nb)[:nblk].tolist() for _ in range(steps)]
    slots = list(range(nblk))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    t_out = t_in = 0.0
    with ClockSampler(0) as clk:
        for i in range(steps):
            ev[0].record(side)
            kvb.swap_out(k, v, outs[i], slots, pool, stream=side)
            ev[1].record(side)
            kvb.swap_in(k, v, ins[i], slots, pool, stream=side)
            ev[2].record(side)
            side.synchronize()
            if i >= args.warmup:
                t_out += ev[0].elapsed_time(ev[1])
                t_in += ev[1].elapsed_time(ev[2])
    # bit-exact round trip of the last step: each block swapped in equals its host slot's K and V
    bb = B * kvh * D * 2
    for j in range(8):
        hk = pool[j * slot:j * slot + L * bb].view(torch.int16).view(L, B, kvh, D)
        hv = pool[j * slot + L * bb:(j + 1) * slot].view(torch.int16).view(L, B, kvh, D)
        assert torch.equal(k[:, ins[-1][j]].view(torch.int16).cpu(), hk)
        assert torch.equal(v[:, ins[-1][j]].view(torch.int16).cpu(), hv)
    moved = nblk * block_bytes_all_layers(cfg)
    g_out = moved / (t_out / args.steps / 1e3) / 1e9
    g_in = moved / (t_in / args.steps / 1e3) / 1e9
    line = {"metric": "block swap bandwidth (out, in)", "value": round(min(g_out, g_in), 1), "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "op": "swap",
            "out_gbs": round(g_out, 1), "in_gbs": round(g_in, 1),
            "ms_per_step": round((t_out + t_in) / args.steps, 3), "dtype": cfg["dtype"], "data": "synthetic random bits",
            "config": {"workload": f"{args.config}-shaped blocks ({block_bytes_all_layers(cfg)} bytes, every layer, K "
                                   f"and V), {nblk} random blocks out and {nblk} back in per step, pinned host pool",
                       "copies": "one cudaMemcpy2DAsync per (block, K|V), layers strided"},
            "gpu_launches": 0, "clocks": clk.summary()}
    print(json.dumps(line))


class _BankContent:
    """The data-plane benchmark's K/V source: each row is a row of a seeded random bank (4096 rows of every
    layer's K and V), picked by a hash of the row's origin and position -- the prefix and fork sharing of
    dataplane.SyntheticContent at the cost of one gather (content does not matter for timing)."""

    def __init__(self, requests, cfg, dev, tdt, max_rows):
        import torch
        dp = importlib.import_module("paged-kv-cache-manager_b200.dataplane")
        L, kvh, D, nh = cfg["L"], cfg["kvh"], cfg["D"], cfg["nh"]
        self.origins = dp.SyntheticContent(requests, layers=1, kv_heads=1, head_dim=1, num_heads=1,
                                           device=dev).origins
        g = torch.Generator(device=dev).manual_seed(11)
        self.bank = torch.randn((2, L, 4096, kvh, D), generator=g, device=dev).to(tdt)
        self.qbank = torch.randn((L, max_rows, nh, D), generator=g, device=dev).to(tdt)
        self.dev = dev

    def __call__(self, rids, positions):
        import torch
        key = (self.origins(rids, positions) * 1000003 + np.asarray(positions) * 7919) % 4096
        idx = torch.from_numpy(key).pin_memory().to(self.dev, non_blocking=True)
        return self.bank[0].index_select(1, idx), self.bank[1].index_select(1, idx)

    def queries(self, rids):
        return self.qbank[:, :len(rids)]


def run_sim(args, cfg):
    """Scheduler-driven data plane: the reference simulator's recorded decision stream at serving scale
    (tests/golden/sim_traces.npz, `serving_fcfs_swap`: 256 requests, long-tail prompts up to 3072 tokens, shared
    prefixes + prefix cache, FCFS, swap preemption, 3072 blocks of 16 tokens) replayed by dataplane.DataPlane at
    this config's head shape: prefill writes, copy-on-write, swap-out / swap-in through a pinned pool, and
    per-layer fused append + attention of every generating request, all decisions re-made by the KVManager.
    One warm-up replay, then `--sim-replays` timed replays, each on fresh pools; wall time includes the host."""
    import time
    import torch
    dp = importlib.import_module("paged-kv-cache-manager_b200.dataplane")
    z = np.load(os.path.join(ROOT, "tests", "golden", "sim_traces.npz"))
    name = "serving_fcfs_swap"
    trace, req, conf, met = (z[f"{name}_{k}"] for k in ("trace", "requests", "config", "metrics"))
    nb, B = int(conf[0]), int(conf[1])
    L, kvh, D, nh = cfg["L"], cfg["kvh"], cfg["D"], cfg["nh"]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    held, used, peak = {}, 0, 0
    for row in trace:
        if row[0] == dp.TRACE_FREE and row[6] == dp.FREE_SWAPPED:
            held[int(row[1])] = -(-int(row[2]) // B)
            used += held[int(row[1])]
            peak = max(peak, used)
        elif row[0] == dp.TRACE_ADMIT_PREFIX and row[6] == 1:
            used -= held.pop(int(row[1]))
    content = _BankContent(req, cfg, dev, tdt, max_rows=512)
    tok_bytes = L * kvh * D * 2 * (2 if tdt != torch.float32 else 4)

    def replay():
        plane = dp.DataPlane(nb, B, layers=L, num_heads=nh, kv_heads=kvh, head_dim=D, source=content,
                             queries=content.queries, dtype=tdt, device=dev, swap_slots=peak)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        n = plane.run(trace)
        st = plane.status_word()  # synchronises
        wall = time.perf_counter() - t0
        assert st == 0, st
        secs, attn_bytes = plane.attention_time()
        return n, wall, secs, attn_bytes

    replay()
    runs = []
    with ClockSampler(0) as clk:
        for _ in range(args.sim_replays):
            runs.append(replay())
    n = runs[-1][0]
    assert (n.steps, n.tokens_generated, n.swap_out_blocks, n.prefill_tokens) == \
        (int(met[0]), int(met[1]), int(met[5]), int(met[9]))
    wall = float(np.mean([r[1] for r in runs]))
    attn_s = float(np.mean([r[2] for r in runs]))
    attn_bytes = runs[-1][3]
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak_hbm = float(peaks.get("hbm_gbs", 6650.0))
    achieved = attn_bytes / attn_s / 1e9
    blk = B * tok_bytes
    line = {"metric": "scheduler-driven decode replay throughput", "value": round(n.tokens_generated / wall, 1),
            "unit": "tok/s", "n_gpus": 1, "steps": args.sim_replays, "warmup": 1,
            "ms_per_step": round(1e3 * wall, 2), "higher_is_better": True, "op": "sim", "dtype": cfg["dtype"],
            "data": "reference simulator decision stream; synthetic K/V rows",
            "config": {"workload": f"{args.config}-shaped heads, {L} layers; {name}: {len(trace)} decisions, "
                                   f"{n.steps} scheduler steps, {nb} blocks x {B} tokens",
                       "step": "one replay of the whole decision stream (host decisions included)"},
            "scheduler_steps_per_s": round(n.steps / wall, 1),
            "attention": {"launches": n.attention_launches, "seconds": round(attn_s, 4),
                          "algorithmic_bytes": attn_bytes, "share_of_wall": round(attn_s / wall, 3)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_hbm, "unit": "GB/s",
                         "frac": round(achieved / peak_hbm, 4), "traffic": None,
                         "kernel": "paged_decode_streamk_kernel inside the replay (event time per batch)",
                         "peak_source": "measured" if "hbm_gbs" in peaks else "fallback"},
            "data_plane_bytes": {"prefill": n.prefill_tokens * tok_bytes, "appended": n.tokens_generated * tok_bytes,
                                 "cow_copied": n.cow_copies * blk, "swap_out": n.swap_out_blocks * blk,
                                 "swap_in": n.swap_in_blocks * blk},
            "counters": n.as_dict(), "gpu_launches": n.attention_launches, "clocks": clk.summary()}
    print(json.dumps(line))


def _drop_in_fn(kvb):
    """The drop-in launch_paged_attention (C++ symbol) from the library, bound with ctypes."""
    import ctypes as C
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", kvb.LIB_PATH], capture_output=True, text=True).stdout
    name = [ln.split()[-1] for ln in out.splitlines() if "launch_paged_attention" in ln][0]
    f = getattr(kvb.lib(), name)
    f.restype = C.c_int
    f.argtypes = [C.c_void_p] * 6 + [C.c_int] * 7 + [C.c_void_p]
    return f


def run_latency(args):
    """The small 8-sequence correctness case, timed for latency: 8 sequences, 8/8 heads, head_dim 64, block
    16, lengths U{1..512} (seeded), fp32 queries, fp16 K/V in a 1024-block pool (each request's blocks a random
    permutation of pool ids), fp32 output, one layer -- about 4 MB per call, L2-resident and launch-bound.
    Times kvp_paged_attention (per call back to back on a stream, replayed from a CUDA graph, and one call
    alone between events) and the drop-in launch_paged_attention (fp16 in and out, the reference's signature),
    with the reference's paged_attention_cpu on the same input beside it."""
    import ctypes as C
    import time
    import torch
    import oracle
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
    nh, kvh, D, B, ns, nb = 8, 8, 64, 16, 8, 1024
    rng = np.random.default_rng(1)
    lens = rng.integers(1, 513, size=ns).astype(np.int32)
    nblk = (lens + B - 1) // B
    mb = int(nblk.max())
    perm = rng.permutation(nb).astype(np.int32)
    T = np.zeros((ns, mb), np.int32)
    o = 0
    for i in range(ns):
        T[i, :nblk[i]] = perm[o:o + nblk[i]]
        o += int(nblk[i])
    Q = rng.standard_normal((ns, nh, D), dtype=np.float32)
    K = rng.standard_normal((nb, B, kvh, D), dtype=np.float32).astype(np.float16)
    V = rng.standard_normal((nb, B, kvh, D), dtype=np.float32).astype(np.float16)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v = torch.from_numpy(Q).to(dev), torch.from_numpy(K).to(dev), torch.from_numpy(V).to(dev)
    t, ln = torch.from_numpy(T).to(dev), torch.from_numpy(lens).to(dev)
    out = torch.empty((ns, nh, D), dtype=torch.float32, device=dev)
    a = kvb.attention_args(q, k, v, t, ln, out, nh, kvh, num_blocks=nb)
    ws = torch.zeros(max(kvb.workspace_bytes(a), 256), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes, a.flags = ws.data_ptr(), ws.numel(), kvb.KVP_ATTN_WORKSPACE_CLEAN
    fn = kvb.lib().kvp_paged_attention
    stream = torch.cuda.Stream(dev)
    sp = C.c_void_p(stream.cuda_stream)

    def launch():
        rc = fn(C.byref(a), sp)
        assert rc == 0, kvb.last_error()

    n_b2b = 200
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]

    def back_to_back(body):
        vals = []
        for _ in range(args.steps):
            ev[0].record(stream)
            body()
            ev[1].record(stream)
            stream.synchronize()
            vals.append(ev[0].elapsed_time(ev[1]) * 1e3 / n_b2b)
        return float(np.median(vals))

    with torch.cuda.stream(stream):
        for _ in range(args.warmup * 20):
            launch()
        stream.synchronize()
        with ClockSampler(0) as clk:
            us_stream = back_to_back(lambda: [launch() for _ in range(n_b2b)])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(n_b2b):
                    launch()
            g.replay()
            stream.synchronize()
            us_graph = back_to_back(g.replay)
            single = []
            for _ in range(max(args.steps, 20)):
                stream.synchronize()
                ev[0].record(stream)
                launch()
                ev[1].record(stream)
                stream.synchronize()
                single.append(ev[0].elapsed_time(ev[1]) * 1e3)
            us_single = float(np.median(single))
            # the drop-in entry point: fp16 queries and output, the reference's signature
            f = _drop_in_fn(kvb)
            qh = q.half()
            oh = torch.empty((ns, nh, D), dtype=torch.float16, device=dev)

            def drop_in():
                rc = f(qh.data_ptr(), k.data_ptr(), v.data_ptr(), t.data_ptr(), ln.data_ptr(), oh.data_ptr(), ns, nh,
                       kvh, D, B, mb, 4, stream.cuda_stream)
                assert rc == 0
            for _ in range(20):
                drop_in()
            us_drop_in = back_to_back(lambda: [drop_in() for _ in range(n_b2b)])
        del g
    # the reference's CPU function on the same input (fp32 copies of the fp16 K/V), 1 thread and all cores
    impl = "ref" if oracle.have_ref() else "c"
    cores = os.cpu_count() or 1
    Kf, Vf = K.astype(np.float32), V.astype(np.float32)
    cpu = {}
    for nthreads in (1, cores):
        oracle.paged_attention_cpu(nh, kvh, D, B, Q, Kf, Vf, T, lens, partitions=1, nthreads=nthreads, impl=impl)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 2.0:
            oracle.paged_attention_cpu(nh, kvh, D, B, Q, Kf, Vf, T, lens, partitions=1, nthreads=nthreads, impl=impl)
            reps += 1
        cpu[nthreads] = (time.perf_counter() - t0) / reps * 1e6
    algo = float(lens.sum()) * kvh * D * 2 * 2
    line = {"metric": "paged decode-attn latency (8 sequences, 8/8 heads, D 64)", "value": round(us_stream, 2), "unit": "us",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us_stream / 1e3, 5),
            "higher_is_better": False, "op": "latency", "dtype": "f16", "data": "synthetic N(0,1), seeded",
            "config": {"workload": "small correctness case: 8 sequences, 8/8 heads, head_dim 64, block 16, lengths U{1..512}, "
                                   "fp32 q / fp16 K,V / fp32 out, 1024-block pool, one layer",
                       "context_tokens": int(lens.sum()), "kv_bytes": int(algo),
                       "l2": "L2-resident (about 4 MB per call): a latency, not a bandwidth, figure"},
            "us_per_call": {"stream_back_to_back": round(us_stream, 2), "cuda_graph": round(us_graph, 2),
                            "single_call_between_events": round(us_single, 2),
                            "drop_in_launch_paged_attention_back_to_back": round(us_drop_in, 2)},
            "cpu_baseline": {"value": round(cpu[cores], 1), "unit": "us", "cores": cores,
                             "one_thread_us": round(cpu[1], 1),
                             "kind": "reference" if impl == "ref" else "port",
                             "sample": "the same 8 sequences, paged_attention_cpu (partitions 1), timed over 2 s"},
            "gpu_launches": n_b2b * args.steps, "clocks": clk.summary()}
    print(json.dumps(line))


class OpMix:
    """The KV-management op mix on one GPU (BASELINE config 5 at its stated scale by default): a shared
    `prefix`-token prompt admitted once (the parent), `requests` requests admitted with admit_with_prefix on it
    (prompt = prefix + a seeded suffix of 1..255 tokens, never block-aligned, so the request's last block is
    partial), each forked into `samples` samples (the request plus samples - 1 forks); then decode steps: every
    live sample appends one token (KVManager.append_batch on the host), the copy-on-write pairs those appends
    decided are copied (kvp_cow_copy; the first append of all but one of the samples sharing a partial block),
    and every sample's new K/V row of every layer is written to its slot (kvp_append_scatter).  After every
    `swap_every`-th step, samples drawn at random (seeded) until their tables hold `swap_frac` of the allocated
    blocks are swapped out to a pinned host pool (kvp_swap_out on a side stream, then freed, as the reference's
    simulator preempts, src/simulator.cpp:117-133); they sit out the next step, whose allocations reuse the freed
    blocks, and are swapped back in after it (admitted with fresh ids and no sharing, kvp_swap_in;
    src/simulator.cpp:193, 231-241).

    Content model: the K (V) row of position p written on behalf of `origin` is row key(origin, p) of a seeded
    N(0,1) bank, where origin is the parent for the prefix, the request for its suffix and the sample for its
    decode tokens -- so the context any live sample must see through its table is known, and check() compares
    it on the device bit for bit.  `on_op(name, args, result)` sees every KVManager call in order (a test replays
    them on the reference's KVManager)."""

    BANK = 8192

    def __init__(self, kvb, cfg, dev, requests=512, samples=8, prefix=2048, steps=64, swap_every=16,
                 swap_frac=0.1, seed=5, on_op=None):
        import torch
        self.kvb, self.cfg, self.dev = kvb, cfg, dev
        self.L, self.B, self.kvh, self.D = cfg["L"], cfg["B"], cfg["kvh"], cfg["D"]
        self.tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
        self.requests, self.samples, self.prefix = requests, samples, prefix
        self.swap_every, self.swap_frac, self.on_op = swap_every, swap_frac, on_op
        self.rng = np.random.default_rng(seed)
        B = self.B
        self.suffix = self.rng.integers(1, 256, size=requests)
        self.suffix[(prefix + self.suffix) % B == 0] += 1  # keep every request's last block partial
        # pool: prefix + suffix blocks, one copy-on-write block per sample, the decode growth, the swap-in copies
        n_s = requests * samples
        grow = n_s * (steps // B + 2)
        need = prefix // B + int(((self.suffix + B - 1) // B).sum()) + n_s + grow
        swap_cap = int(swap_frac * need) + (prefix + 256 + steps) // B + 8
        rounds = steps // swap_every + 1
        self.nb = need + rounds * swap_cap + 64
        self.swap_cap = swap_cap
        self.k = torch.empty((self.L, self.nb, B, self.kvh, self.D), dtype=self.tdt, device=dev)
        self.v = torch.empty_like(self.k)
        g = torch.Generator(device=dev).manual_seed(seed)
        self.bank_k = torch.randn((self.L, self.BANK, self.kvh, self.D), generator=g, device=dev).to(self.tdt)
        self.bank_v = torch.randn((self.L, self.BANK, self.kvh, self.D), generator=g, device=dev).to(self.tdt)
        self.mgr = kvb.KVManager(self.nb, B)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.compute = torch.cuda.current_stream(dev)
        self.side = torch.cuda.Stream(dev)
        self.slot_bytes = kvb.host_slot_bytes(self.L, B, self.kvh, self.D, self.k.element_size())
        self.host = torch.empty(self.slot_bytes * swap_cap, dtype=torch.uint8, pin_memory=True)
        self.parent = -1
        # Sample identities are 0 .. requests * samples - 1 (request r's are r * samples + s); a sample keeps its
        # identity (and so its content) when a swap gives it a new manager id.
        self.mid = {}
        self.tokens = np.zeros(n_s, np.int64)
        self.live = []        # identities decoding this step
        self.away = []        # identities swapped out: (identity, tokens, host slots)
        self.next_id = 10 ** 7
        self.counters = dict(cow_pairs=0, cow_bytes=0, cow_ms=0.0, scatter_rows=0, scatter_bytes=0, scatter_ms=0.0,
                             swap_out_blocks=0, swap_in_blocks=0, swap_out_ms=0.0, swap_in_ms=0.0, swap_rounds=0,
                             steps=0)
        self._events = []

    # ---------------------------------------------------------------- helpers
    def _op(self, name, *args):
        res = getattr(self.mgr, name)(*args)
        if self.on_op is not None:
            self.on_op(name, args, res)
        return res

    def _key(self, origin, pos):
        return (np.asarray(origin, np.int64) * 1000003 + np.asarray(pos, np.int64) * 7919) % self.BANK

    def _origin(self, ident, pos):
        """Who wrote position pos of sample ident (arrays broadcast): the parent, the request, or the sample."""
        ident, pos = np.asarray(ident, np.int64), np.asarray(pos, np.int64)
        req = ident // self.samples
        prompt = self.prefix + self.suffix[req]
        return np.where(pos < self.prefix, self.parent, np.where(pos < prompt, req * self.samples, ident))

    def _write(self, keys, slots, timed=False):
        """Bank rows `keys` into `slots` (every layer, K and V) with kvp_append_scatter on the compute stream."""
        import torch
        idx = torch.from_numpy(np.asarray(keys, np.int64)).to(self.dev)
        kn = self.bank_k.index_select(1, idx)
        vn = self.bank_v.index_select(1, idx)
        d_slots = torch.from_numpy(np.asarray(slots, np.int32)).to(self.dev)
        if timed:
            e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            e[0].record(self.compute)
        self.kvb.append_scatter(kn, vn, self.k, self.v, d_slots, status=self.status, stream=self.compute)
        if timed:
            e[1].record(self.compute)
            self._events.append(("scatter", e, len(slots)))

    def _prompt_rows(self, ident, start, end):
        tbl = self.mgr.block_table(self.mid[ident])
        pos = np.arange(start, end)
        slots = np.asarray(tbl, np.int64)[pos // self.B] * self.B + pos % self.B
        self._write(self._key(self._origin(ident, pos), pos), slots)

    # ---------------------------------------------------------------- workload
    def setup(self):
        """Parent prefix, the requests' prompts (their suffix rows written), the forks."""
        self.parent = self.next_id
        self.next_id += 1
        assert self._op("admit", self.parent, self.prefix)
        pos = np.arange(self.prefix)
        tbl = np.asarray(self.mgr.block_table(self.parent), np.int64)
        self._write(self._key(np.full(self.prefix, self.parent), pos), tbl[pos // self.B] * self.B + pos % self.B)
        for r in range(self.requests):
            lead = r * self.samples
            prompt = self.prefix + int(self.suffix[r])
            self.mid[lead] = lead
            assert self._op("admit_with_prefix", lead, self.parent, self.prefix, prompt)
            self._prompt_rows(lead, self.prefix, prompt)
            self.live.append(lead)
            for s in range(1, self.samples):
                ident = lead + s
                self.mid[ident] = ident
                assert self._op("fork", ident, lead)
                self.live.append(ident)
            self.tokens[lead:lead + self.samples] = prompt
        self.compute.synchronize()

    def step(self):
        """One decode step of every live sample; then, on swap steps, the swap-in of the previous round's
        samples and the swap-out of this round's."""
        import torch
        live = self.live
        rids = [self.mid[i] for i in live]
        done, slots, pairs = self._op("append_batch", rids)
        assert done == len(rids), "the pool ran out of blocks"
        if len(pairs):
            e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            e[0].record(self.compute)
            self.kvb.cow_copy(self.k, self.v, torch.from_numpy(np.ascontiguousarray(pairs)).to(self.dev),
                              status=self.status, stream=self.compute)
            e[1].record(self.compute)
            self._events.append(("cow", e, len(pairs)))
        ids = np.asarray(live, np.int64)
        pos = self.tokens[ids]  # the new token's position
        self.tokens[ids] += 1
        self._write(self._key(self._origin(ids, pos), pos), slots, timed=True)
        self.counters["steps"] += 1
        if self.away:
            self._swap_in()
        if self.counters["steps"] % self.swap_every == 0:
            self._swap_out()

    def _swap_out(self):
        import torch
        allocated = self.mgr.total_blocks() - self.mgr.free_blocks()
        order = self.rng.permutation(len(self.live))
        victims, blocks, held = [], [], 0
        for j in order:
            ident = self.live[int(j)]
            tbl = self.mgr.block_table(self.mid[ident])
            if held + len(tbl) > self.swap_cap:
                continue
            victims.append(ident)
            blocks.append(tbl)
            held += len(tbl)
            if held >= self.swap_frac * allocated:
                break
        flat = [b for t in blocks for b in t]
        self.side.wait_stream(self.compute)  # the rows written so far go out with the blocks
        e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        e[0].record(self.side)
        self.kvb.swap_out(self.k, self.v, flat, list(range(len(flat))), self.host, stream=self.side)
        e[1].record(self.side)
        self._events.append(("swap_out", e, len(flat)))
        self.compute.wait_stream(self.side)  # freed blocks are rewritten only after they went out
        o = 0
        for ident, tbl in zip(victims, blocks):
            tokens = int(self.tokens[ident])
            self._op("free", self.mid[ident])
            self.away.append((ident, tokens, list(range(o, o + len(tbl)))))
            o += len(tbl)
        gone = set(victims)
        self.live = [i for i in self.live if i not in gone]
        self.counters["swap_rounds"] += 1

    def _swap_in(self):
        import torch
        fresh, slots = [], []
        for ident, tokens, hs in self.away:
            new = self.next_id
            self.next_id += 1
            assert self._op("admit", new, tokens), "no room to swap back in"
            self.mid[ident] = new
            tbl = self.mgr.block_table(new)
            assert len(tbl) == len(hs)
            fresh.extend(tbl)
            slots.extend(hs)
            self.live.append(ident)
        e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        e[0].record(self.side)
        self.kvb.swap_in(self.k, self.v, fresh, slots, self.host, stream=self.side)
        e[1].record(self.side)
        self._events.append(("swap_in", e, len(fresh)))
        self.compute.wait_stream(self.side)  # the next step appends into the fresh blocks
        self.away = []

    def settle(self):
        """Waits for the device, folds the op events into the counters; returns the status word."""
        import torch
        torch.cuda.synchronize(self.dev)
        blk = 2 * self.L * self.B * self.kvh * self.D * self.k.element_size()
        row = 2 * self.L * self.kvh * self.D * self.k.element_size()
        c = self.counters
        for kind, (e0, e1), n in self._events:
            ms = e0.elapsed_time(e1)
            if kind == "cow":
                c["cow_pairs"] += n
                c["cow_bytes"] += 2 * n * blk
                c["cow_ms"] += ms
            elif kind == "scatter":
                c["scatter_rows"] += n
                c["scatter_bytes"] += 2 * n * row
                c["scatter_ms"] += ms
            elif kind == "swap_out":
                c["swap_out_blocks"] += n
                c["swap_out_ms"] += ms
            else:
                c["swap_in_blocks"] += n
                c["swap_in_ms"] += ms
        self._events = []
        return int(self.status.item())

    def check(self, idents=None):
        """Every given live sample's context, gathered from the device through its table, equals the content
        model bit for bit (K and V, every layer).  Returns the number of rows checked."""
        import torch
        torch.cuda.synchronize(self.dev)
        rows = 0
        for ident in (self.live if idents is None else idents):
            mid = self.mid[ident]
            n = self.mgr.num_tokens(mid)
            tbl = np.asarray(self.mgr.block_table(mid), np.int64)
            pos = np.arange(n)
            blk = torch.from_numpy(tbl[pos // self.B]).to(self.dev)
            off = torch.from_numpy(pos % self.B).to(self.dev)
            key = torch.from_numpy(self._key(self._origin(ident, pos), pos)).to(self.dev)
            for pool, bank in ((self.k, self.bank_k), (self.v, self.bank_v)):
                got = pool[:, blk, off]
                assert torch.equal(got, bank.index_select(1, key)), f"sample {ident}: context differs"
            rows += n
        return rows


def run_mix(args, cfg):
    """The KV-management op mix (OpMix) at its stated scale: 512 requests x 8 samples on a 2048-token shared
    prefix, Llama-3-8B-shaped blocks (32 layers, 8 kv heads x 128, bf16, 16 tokens: 2 MiB per block), a swap
    round every 16 steps.  `--warmup` steps run first (the copy-on-write burst of the first append is among
    them), then `--steps` timed steps; steps/s is the host + device wall time per timed step.  Reported beside
    it: copy-on-write, append-scatter and swap bandwidths from CUDA events around each of those launches over the
    whole run.  Verified after the run: every live sample's context equals the content model (a sample of 256
    with --mix-check-all not given)."""
    import torch
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    total = args.warmup + args.steps
    mix = OpMix(kvb, cfg, dev, requests=args.mix_requests, steps=total, seed=5)
    mix.setup()
    for _ in range(args.warmup):
        mix.step()
    torch.cuda.synchronize(dev)
    with ClockSampler(0) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            mix.step()
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
    assert mix.settle() == 0
    assert mix.mgr.validate() == ""
    live = list(mix.live)
    pick = live if args.mix_check_all else [live[int(i)] for i in np.random.default_rng(9).permutation(len(live))[:256]]
    rows = mix.check(pick)
    c = mix.counters
    blk = 2 * mix.L * mix.B * mix.kvh * mix.D * 2
    st = mix.mgr.stats()
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))

    def rate(b, ms):
        return round(b / (ms / 1e3) / 1e9, 1) if ms > 0 else None

    line = {"metric": "KV-op mix decode steps per second", "value": round(args.steps / wall, 2), "unit": "steps/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * wall / args.steps, 3),
            "higher_is_better": True, "op": "mix", "dtype": cfg["dtype"], "data": "synthetic N(0,1) bank rows, seeded",
            "config": {"workload": f"KV-op mix: {args.mix_requests} requests x {mix.samples} samples on a {mix.prefix}-token "
                                   f"shared prefix (admit_with_prefix + fork), {mix.L} layers x {mix.kvh} kv heads x "
                                   f"{mix.D}, bf16, block {mix.B}; copy-on-write on the first append; every "
                                   f"{mix.swap_every} steps {int(100 * mix.swap_frac)}% of the allocated blocks swapped "
                                   f"out to pinned host memory and back in after one step",
                       "step": "host append_batch of every live sample + copy-on-write + append scatter (+ swaps)"},
            "cow": {"pairs": c["cow_pairs"], "gb_s": rate(c["cow_bytes"], c["cow_ms"]),
                    "frac_of_hbm_peak": round(c["cow_bytes"] / (c["cow_ms"] / 1e3) / 1e9 / peak, 4) if c["cow_ms"] else None,
                    "bytes": "read + write of 2 MiB per pair"},
            "scatter": {"rows": c["scatter_rows"], "gb_s": rate(c["scatter_bytes"], c["scatter_ms"]),
                        "frac_of_hbm_peak": round(c["scatter_bytes"] / (c["scatter_ms"] / 1e3) / 1e9 / peak, 4)},
            "swap": {"rounds": c["swap_rounds"], "out_blocks": c["swap_out_blocks"], "in_blocks": c["swap_in_blocks"],
                     "out_gb_s": rate(c["swap_out_blocks"] * blk, c["swap_out_ms"]),
                     "in_gb_s": rate(c["swap_in_blocks"] * blk, c["swap_in_ms"])},
            "kv_stats": dict(st), "pool_blocks": mix.nb,
            "verified": {"samples": len(pick), "rows": rows, "bit_exact": True},
            "gpu_launches": args.steps * 2 + c["swap_rounds"], "clocks": clk.summary()}
    print(json.dumps(line))


def run_block_mover(args, cfg):
    """Whole-block movers of the data plane, device timed: `migrate` copies blocks from a second GPU's pool into
    this GPU's pool (kvp_migrate_blocks, peer loads over NVLink; two pools on one GPU when only one is
    visible), `cow` copies blocks within one pool (kvp_cow_copy).  A step moves `blocks` random (src, dst)
    pairs of config blocks (every layer, K and V)."""
    import torch
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
    L, B, kvh, D = cfg["L"], cfg["B"], cfg["kvh"], cfg["D"]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    nblk = args.pairs
    nb = 2 * nblk
    two = args.op == "migrate" and torch.cuda.device_count() >= 2
    dst_dev = torch.device("cuda", 0)
    src_dev = torch.device("cuda", 1) if two else dst_dev

    def pool(dev):
        t = torch.empty((L, nb, B, kvh, D), dtype=tdt, device=dev)
        t.view(torch.int16).random_(-30000, 30000)
        return t

    dk, dv = pool(dst_dev), pool(dst_dev)
    sk, sv = (pool(src_dev), pool(src_dev)) if args.op == "migrate" else (dk, dv)
    rng = np.random.default_rng(0)
    steps_total = args.warmup + args.steps
    pairs = []
    for _ in range(steps_total):
        src = rng.permutation(nb)[:nblk]
        dst = rng.permutation(nb)[:nblk] if args.op == "migrate" else np.setdiff1d(np.arange(nb), src)
        pairs.append(torch.from_numpy(np.stack([src, rng.permutation(dst)], 1).astype(np.int32)).to(dst_dev))
    st = torch.zeros(1, dtype=torch.int32, device=dst_dev)
    stream = torch.cuda.current_stream(dst_dev)

    def one(i):
        if args.op == "migrate":
            kvb.migrate_blocks(sk, sv, dk, dv, pairs[i], status=st, stream=stream)
        else:
            kvb.cow_copy(dk, dv, pairs[i], status=st, stream=stream)

    for i in range(args.warmup):
        one(i)
    torch.cuda.synchronize(dst_dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record(stream)
        for i in range(args.steps):
            one(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize(dst_dev)
    assert int(st.item()) == 0
    # bit-exact spot check of the last step
    p = pairs[-1][:64].long()
    assert torch.equal(dk[:, p[:, 1].to(dst_dev)].view(torch.int16).cpu(), sk[:, p[:, 0].to(src_dev)].view(torch.int16).cpu())
    ms = e0.elapsed_time(e1) / args.steps
    moved = nblk * block_bytes_all_layers(cfg)  # bytes copied per step
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    if two:
        bound, peak, unit, algo = "nvlink", 770.0, "GB/s", moved  # measured peer-copy bandwidth per direction
        peak_src = "measured peer copy per direction"
    else:
        bound, peak, unit, algo = "hbm", float(peaks.get("hbm_gbs", 6650.0)), "GB/s", 2 * moved  # read + write
        peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    achieved = algo / (ms / 1e3) / 1e9
    line = {"metric": f"block {args.op} bandwidth", "value": round(moved / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "n_gpus": 2 if two else 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "op": args.op, "dtype": cfg["dtype"], "data": "synthetic random bits",
            "config": {"workload": f"{args.config}-shaped blocks ({block_bytes_all_layers(cfg)} bytes, every layer, "
                                   f"K and V), {nblk} random pairs per step",
                       "src": str(src_dev), "dst": str(dst_dev)},
            "roofline": {"bound": bound, "achieved": round(achieved, 1), "peak": peak, "unit": unit,
                         "frac": round(achieved / peak, 4), "peak_source": peak_src},
            "gpu_launches": args.steps, "clocks": clk.summary()}
    print(json.dumps(line))


def reference_arm(args, cfg, config, metric):
    """The reference's own CPU implementation of the path (paged_attention_cpu from the reference library built
    here, else the oracle's C restatement) on all host cores.  A timed step is one layer of every request of
    the shard (the same length distribution; tables draw their blocks from a shared pool of up to 16,384
    blocks, N(0,1) fp32 data): 1/L of a decode step, so `ms_per_step` x `steps` is what actually ran, and the
    decode rate is requests / (L x seconds per step)."""
    import oracle
    kind = "reference" if oracle.have_ref() else "port"
    impl = "ref" if kind == "reference" else "c"
    cores = os.cpu_count() or 1
    lens = sample_lens(cfg, cfg["ns"], seed=1000)
    (Q, K, V, T, sl), pool = cpu_layer_workload(cfg, lens)
    nh, kvh, D, B = cfg["nh"], cfg["kvh"], cfg["D"], cfg["B"]

    def one():
        t0 = time.perf_counter()
        oracle.paged_attention_cpu(nh, kvh, D, B, Q, K, V, T, sl, partitions=1, nthreads=cores, impl=impl)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        one()
    t_run = time.perf_counter()
    secs = [one() for _ in range(args.steps)]
    wall = time.perf_counter() - t_run
    per_step = float(np.mean(secs))
    v = len(sl) / (cfg["L"] * per_step)
    gbs = float(sl.sum()) * kvh * D * 2 * 2 / per_step / 1e9
    cb = {"value": v, "unit": "tok/s", "cores": cores, "kind": kind, "gb_s": round(gbs, 3),
          "sample": f"one layer of all {len(sl)} requests per step ({int(sl.sum())} context tokens; tables over a "
                    f"shared pool of {pool} blocks), {args.steps} timed steps over {wall:.1f}s"}
    line = {"metric": metric, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * per_step, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)", "config": config,
            "impl": "reference", "cpu_baseline": cb,
            "step": {"what": f"one layer of the decode step (1/{cfg['L']} of it) for every request, all host cores",
                     "layers_per_decode_step": cfg["L"], "timed_wall_s": round(wall, 2),
                     "ms_per_decode_step": round(1e3 * per_step * cfg["L"], 1)},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    ref_gpu = reference_gpu_kernel(cfg, lens)
    if ref_gpu is not None:
        line["reference_gpu_kernel"] = ref_gpu
    return line


def run_scatter(args, cfg):
    """The append scatter alone (kvp_append_scatter: every layer's K and V row of each new token into its
    slot), device timed with CUDA events around each launch and L2 flushed before it (a 256 MB buffer written
    outside the events), at two shapes of this config: `decode` -- one new token for each of the shard's
    requests (a random slot in each of `requests` distinct random blocks) -- and `prompt` -- `prompt_rows`
    consecutive positions of one request (its blocks a random permutation of pool ids), the prefill write.
    Bytes: read + write of 2 (K, V) x layers x rows x kv_heads x head_dim x 2.  The line's value is the prompt
    shape's GB/s; both shapes are checked bit-exact on a sample of rows."""
    import torch
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
    L, B, kvh, D = cfg["L"], cfg["B"], cfg["kvh"], cfg["D"]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prompt_rows = args.prompt_rows
    ns = cfg["ns"]
    nb = 2 * max(ns, (prompt_rows + B - 1) // B) + 16
    k = torch.zeros((L, nb, B, kvh, D), dtype=tdt, device=dev)
    v = torch.zeros_like(k)
    rng = np.random.default_rng(3)
    shapes = {}
    blocks = rng.permutation(nb)[:ns]
    shapes["decode"] = (blocks * B + rng.integers(0, B, size=ns)).astype(np.int32)
    pos = np.arange(prompt_rows)
    table = rng.permutation(nb)[:(prompt_rows + B - 1) // B]
    shapes["prompt"] = (table[pos // B] * B + pos % B).astype(np.int32)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    res = {}
    with ClockSampler(0) as clk:
        for name, slots in shapes.items():
            n = len(slots)
            g = torch.Generator(device=dev).manual_seed(5)
            kn = torch.randn((L, n, kvh, D), generator=g, device=dev).to(tdt)
            vn = torch.randn((L, n, kvh, D), generator=g, device=dev).to(tdt)
            d_slots = torch.from_numpy(slots).to(dev)
            ms = []
            for i in range(args.warmup + args.steps):
                flush.fill_(i & 0xff)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                kvb.append_scatter(kn, vn, k, v, d_slots, status=st, stream=stream)
                e1.record(stream)
                if i >= args.warmup:
                    ms.append((e0, e1))
            torch.cuda.synchronize(dev)
            assert int(st.item()) == 0
            pick = torch.from_numpy(rng.permutation(n)[:64]).to(dev)
            sl = d_slots[pick].long()
            assert torch.equal(k[:, sl // B, sl % B], kn[:, pick]) and torch.equal(v[:, sl // B, sl % B], vn[:, pick])
            t = float(np.mean([a.elapsed_time(b) for a, b in ms]))
            moved = 2 * 2 * L * n * kvh * D * 2  # read + write, K and V
            res[name] = {"rows": n, "us_per_launch": round(t * 1e3, 2), "bytes": moved,
                         "gb_s": round(moved / (t / 1e3) / 1e9, 1), "frac": round(moved / (t / 1e3) / 1e9 / peak, 4)}
    line = {"metric": "append scatter bandwidth (read + write)", "value": res["prompt"]["gb_s"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(res["prompt"]["us_per_launch"] / 1e3, 5),
            "higher_is_better": True, "op": "scatter", "dtype": cfg["dtype"], "data": "synthetic N(0,1), seeded",
            "config": {"workload": f"{args.config}-shaped rows ({kvh} kv heads x {D}, {L} layers, K and V): a prompt "
                                   f"of {prompt_rows} consecutive positions (value) and a decode step of one row for "
                                   f"each of {ns} requests",
                       "l2": "flushed before every launch (256 MB write outside the events)"},
            "shapes": res,
            "roofline": {"bound": "hbm", "achieved": res["prompt"]["gb_s"], "peak": peak, "unit": "GB/s",
                         "frac": res["prompt"]["frac"], "kernel": "append_scatter_kernel<4>",
                         "peak_source": "measured" if "hbm_gbs" in peaks else "fallback"},
            "gpu_launches": 2 * args.steps, "clocks": clk.summary()}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=DEFAULT, choices=sorted(CONFIGS))
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--split", type=int, default=0, help="tiles per context split (0: balanced persistent grid)")
    ap.add_argument("--wph", type=int, default=0, help="tuning: consumer warps per kv head (0: automatic)")
    ap.add_argument("--stages", type=int, default=0, help="tuning: pipeline stages (0: automatic)")
    ap.add_argument("--seq-start-tiles", type=int, default=0,
                    help="tuning: start cost charged per sequence in the balanced partition, in tiles (0: automatic, "
                         "<0: none)")
    ap.add_argument("--no-e2e", action="store_true", help="tuning runs: skip the end-to-end leg")
    ap.add_argument("--eager", action="store_true", help="launch every layer from Python instead of a CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--requests", type=int, default=0, help="profiling: requests per GPU (pool sized to need)")
    ap.add_argument("--layers", type=int, default=0, help="profiling: number of layers (pool sized to need)")
    ap.add_argument("--prompt-rows", type=int, default=4096, help="scatter: positions of the prompt shape")
    ap.add_argument("--pairs", type=int, default=2048, help="cow / migrate: block pairs per step")
    ap.add_argument("--mix-requests", type=int, default=512, help="mix: requests (8 samples each)")
    ap.add_argument("--mix-check-all", action="store_true", help="mix: verify every live sample, not 256")
    ap.add_argument("--op", default="decode",
                    choices=["decode", "migrate", "cow", "swap", "sim", "latency", "scatter", "mix"],
                    help="decode step (default), a whole-block mover measured alone, the scheduler-driven "
                         "data plane (sim), or the small 8-sequence case's per-call latency (latency)")
    ap.add_argument("--sim-replays", type=int, default=2, help="sim: timed replays of the decision stream")
    args = ap.parse_args()
    assert args.warmup >= 3, "at least 3 warm-up steps"
    cfg = dict(CONFIGS[args.config])
    if args.requests or args.layers:
        cfg["ns"] = args.requests or cfg["ns"]
        cfg["L"] = args.layers or cfg["L"]
        cfg["pool_gb"], cfg["pool_blocks"] = None, None
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "paged decode-attn achieved HBM TB/s & % peak; decode tok/s at 1/2/4/8 GPUs"
    reduced = " (reduced profiling case)" if (args.requests or args.layers) else ""
    config = {"workload": f"{args.config}-shaped decode step: fused append + paged decode attention, all layers"
                          + reduced,
              "heads": cfg["nh"], "kv_heads": cfg["kvh"], "head_dim": cfg["D"], "layers": cfg["L"],
              "block_size": cfg["B"], "requests_per_gpu": cfg["ns"], "lengths": list(cfg["lens"]),
              "kv_dtype": cfg["dtype"], "l2": "inputs larger than L2 (every step reads the whole context)",
              "launch": "per-layer launches from Python" if args.eager else
                        "CUDA graph per step (one launch per layer, early start)",
              "parallelism": f"request-sharded x{args.gpus}, no collective"}

    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(reference_arm(args, cfg, config, metric)))
        return

    if args.op == "swap":
        run_swap(args, cfg)
        return
    if args.op == "sim":
        run_sim(args, cfg)
        return
    if args.op == "latency":
        run_latency(args)
        return
    if args.op == "scatter":
        run_scatter(args, cfg)
        return
    if args.op == "mix":
        run_mix(args, cfg)
        return
    if args.op != "decode":
        run_block_mover(args, cfg)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    res, lens = run_ours(args, cfg, rank, world, dev)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak_gbs = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    ns_total = cfg["ns"] * world  # every rank serves a balanced shard of the job's requests
    ms_step = res["ms_total"] / args.steps
    value = ns_total / (ms_step / 1e3)
    achieved = res["bytes_per_launch"] / (res["attn_avg_ms"] / 1e3) / 1e9
    # DRAM traffic per launch: the ncu-measured (read + write) / algorithmic ratio of this kernel on a reduced
    # case of the same workload (profiles/traffic.json), scaled to this launch's algorithmic bytes.
    traffic = None
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        if args.config == DEFAULT:
            traffic = round(tr["dram_read_plus_write_over_algorithmic"] * res["bytes_per_launch"])
    except Exception:
        pass
    e2e_ms_step = res["e2e_ms"] / args.steps
    line = {"metric": metric, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic N(0,1), seeded", "config": config,
            "hbm_tb_s": round(achieved / 1e3, 3), "pct_of_measured_peak": round(100 * achieved / peak_gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(achieved / peak_gbs, 4), "traffic": traffic,
                         "kernel": ("paged_decode_streamk_kernel (fused append, in-kernel merge)" if res["split"] == 0
                                    else "paged_decode_kernel (fused append; + split merge)"),
                         "peak_source": peak_src},
            "e2e": {"value": round(ns_total / (e2e_ms_step / 1e3), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
            "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
            "shard": {"pool_blocks": res["nb"], "split_tiles": res["split"], "mean_context": res["lens_mean"]}}
    if world > 1:
        tok = [cfg["ns"] / (ms / args.steps / 1e3) for ms in res["per_rank_ms"]]
        line["per_rank"] = {"tok_s": [round(x, 1) for x in tok],
                            "ms_per_step": [round(ms / args.steps, 4) for ms in res["per_rank_ms"]],
                            "imbalance_max_over_mean": round(max(res["per_rank_ms"]) /
                                                             float(np.mean(res["per_rank_ms"])), 4)}
    parity_ok = True
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"], parity = cpu_baseline(cfg, lens, target_s=args.cpu_seconds, sample=res["sample"])
        line["parity"] = parity
        parity_ok = parity is None or parity["ok"]
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not parity_ok:
        sys.exit("parity check of the timed step failed")


if __name__ == "__main__":
    main()
