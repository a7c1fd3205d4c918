"""kvp_paged_attention_noalloc: the attention entry point for callers that cannot allocate device memory
(a serving engine whose memory manager has reserved the HBM for the KV pool, or a plugin whose enqueue
callback may not allocate).  It keeps the split partials in a fixed array inside the library instead of a
caller-provided workspace.  Checked through the C ABI against the fp64 oracle and against kvp_paged_attention
with a workspace, on two calls in a row (the second sees whatever the first left in the shared array).  This file is collected
last so that a run stopping at its first failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-3


def _inputs(seed, lens, nh=32, kvh=8, D=128, B=16):
    import torch
    rng = np.random.default_rng(seed)
    nblk = [(n + B - 1) // B for n in lens]
    pool = sum(nblk) + 3
    perm = rng.permutation(pool)
    T = np.zeros((len(lens), max(nblk)), np.int32)
    o = 0
    for i, nb in enumerate(nblk):
        T[i, :nb] = perm[o: o + nb]
        o += nb
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn((pool, B, kvh, D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((pool, B, kvh, D), generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((len(lens), nh, D), generator=g, device=dev).to(torch.bfloat16)
    return q, k, v, torch.from_numpy(T).to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), nh, kvh


def _with_workspace(kvb, q, k, v, t, l, nh, kvh, split):
    import torch
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=q.device)
    a = kvb.attention_args(q, k, v, t, l, out, nh, kvh, split_tiles=split)
    ws = torch.empty(max(kvb.workspace_bytes(a), 256), dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    assert kvb.lib().kvp_paged_attention(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    return out


def _no_alloc(kvb, q, k, v, t, l, nh, kvh, split):
    import torch
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=q.device)
    status = torch.zeros(1, dtype=torch.int32, device=q.device)
    a = kvb.attention_args(q, k, v, t, l, out, nh, kvh, split_tiles=split, status=status)
    rc = kvb.lib().kvp_paged_attention_noalloc(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, kvb.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out


def _close(got, want):
    g, w = got.cpu().numpy(), want.cpu().numpy()
    assert np.isfinite(g).all()
    assert (np.abs(g - w) <= ATOL + RTOL * np.abs(w)).all(), float(np.abs(g - w).max())


def test_no_alloc_matches_workspace_entry_point_twice(kvb, ora, cuda):
    # Two consecutive calls with different inputs and split sizes (and one with the balanced schedule), each
    # checked against the fp64 oracle and against the entry point that takes a caller-allocated workspace.
    from test_attention_gpu import check_close
    for seed, lens, split in ((1, [700, 3000, 17, 1500, 64], 4), (2, [33, 4096, 2048, 1], 3), (3, [900, 5, 2500], 0)):
        args = _inputs(seed, lens)
        got = _no_alloc(kvb, *args, split)
        q, k, v, t, l, nh, kvh = args
        ref = ora.reference_attention(nh, kvh, q.shape[2], k.shape[1], q.float().cpu().numpy(),
                                      k.float().cpu().numpy(), v.float().cpu().numpy(), t.cpu().numpy(),
                                      l.cpu().numpy())
        check_close(got.cpu().numpy(), ref, what=f"no-alloc call (split {split})")
        want = _with_workspace(kvb, *args, split)
        _close(got, want)


def test_no_alloc_automatic_split_fits_and_oversize_is_rejected(kvb, cuda):
    import torch
    args = _inputs(3, [5000] * 40)
    want = _with_workspace(kvb, *args, 1)
    got = _no_alloc(kvb, *args, 0)  # automatic: the balanced schedule's partials fit the fixed scratch
    _close(got, want)
    # one tile per split: 40 x 313 splits x 32 heads x (D + 2) floats is beyond the 32 MiB array
    q, k, v, t, l, nh, kvh = args
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    a = kvb.attention_args(q, k, v, t, l, out, nh, kvh, split_tiles=1)
    rc = kvb.lib().kvp_paged_attention_noalloc(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == kvb.KVP_ENOSPACE
    assert "no-allocation scratch" in kvb.last_error()


def test_no_alloc_balanced_call_after_fixed_splits(kvb, cuda):
    # A call with fixed splits leaves partials where the next balanced call keeps its merge counters; the
    # balanced call must still merge correctly, even when its caller claims a clean workspace (the flag is
    # ignored here: every call clears its counters).
    import torch
    args = _inputs(4, [3000, 1200, 4096, 77, 2500])
    want = _with_workspace(kvb, *args, 0)
    _no_alloc(kvb, *args, 2)  # fills the start of the shared array with partials
    q, k, v, t, l, nh, kvh = args
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=q.device)
    a = kvb.attention_args(q, k, v, t, l, out, nh, kvh)
    a.flags = kvb.KVP_ATTN_WORKSPACE_CLEAN
    rc = kvb.lib().kvp_paged_attention_noalloc(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, kvb.last_error()
    torch.cuda.synchronize()
    _close(out, want)


def test_no_alloc_coarsens_when_balanced_partials_do_not_fit(kvb, cuda):
    # 2,500 short sequences at the Llama-3-8B head shape: the balanced schedule would need about 44 MB of partials,
    # more than the 32 MiB array, so the automatic call switches to fixed splits coarse enough to fit.
    import torch
    lens = np.random.default_rng(6).integers(200, 400, size=2500).tolist()
    args = _inputs(6, lens)
    q, k, v, t, l, nh, kvh = args
    probe = kvb.attention_args(q, k, v, t, l, torch.empty(q.shape, dtype=torch.float32, device=q.device), nh, kvh)
    assert kvb.workspace_bytes(probe) > kvb.KVP_NOALLOC_SCRATCH_BYTES
    fits = []
    for split in (16, 32, 64, 128):
        probe.split_tiles = split
        fits.append(kvb.workspace_bytes(probe) <= kvb.KVP_NOALLOC_SCRATCH_BYTES)
    assert any(fits)
    want = _with_workspace(kvb, *args, 0)
    for _ in range(2):
        _close(_no_alloc(kvb, *args, 0), want)
