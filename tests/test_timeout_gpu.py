"""Failure detection of the attention kernel's bounded pipeline waits, without a GPU fault.

kvp_attention_wait_test arms the first CTA's first pipeline stage for a copy that is never issued (a flag
nothing sets) and limits every wait to a short number of clock cycles.  That CTA's wait runs out: the kernel
must report KVP_STATUS_TIMEOUT in the status word, return without a copy in flight and leave the context
usable -- the next normal launch on the same buffers must be correct (checked against the fp64 oracle).  The
reference's nearest analogue is the simulator's livelock guard (src/simulator.cpp:136).
"""
import ctypes as C
import time

import numpy as np
import pytest

from test_attention_gpu import _normal_case, _round, check_close

pytestmark = pytest.mark.gpu

LIMIT = 2_000_000  # clock cycles: about 1 ms at B200 clocks


@pytest.mark.parametrize("B,split", [(16, 0), (16, -1), (8, 0), (16, 2)],
                         ids=["balanced", "unsplit", "two-runs-per-tile", "fixed-splits"])
def test_wait_runs_out_reports_timeout_and_context_stays_usable(kvb, ora, cuda, B, split):
    import torch
    nh, kvh, D = 32, 8, 128
    lens = [300, 4096, 77, 1500, 33, 2500]
    nb = sum((n + B - 1) // B for n in lens) + 11
    Q, K, V, T, L = _normal_case(5, len(lens), nh, kvh, D, B, lens, nb)
    dev = torch.device("cuda:0")
    qt, qf = _round(Q, "bf16")
    kt, kf = _round(K, "bf16")
    vt, vf = _round(V, "bf16")
    keep = [qt.to(dev), kt.to(dev), vt.to(dev), torch.from_numpy(T).to(dev), torch.from_numpy(L).to(dev)]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.full((len(lens), nh, D), float("nan"), dtype=torch.float32, device=dev)
    a = kvb.attention_args(*keep, out, nh, kvh, split_tiles=split, status=status)
    ws = torch.zeros(max(kvb.workspace_bytes(a), 256), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = kvb.lib()

    t0 = time.perf_counter()
    assert lib.kvp_attention_wait_test(C.byref(a), sp, LIMIT, 1) == 0, kvb.last_error()
    torch.cuda.synchronize()
    stalled_s = time.perf_counter() - t0
    assert int(status.item()) & kvb.KVP_STATUS_TIMEOUT, f"status {int(status.item())}"
    assert stalled_s < 5.0, f"the stalled launch took {stalled_s:.2f}s"

    # Same buffers, normal launch: the merge counters a timed-out launch may leave nonzero are cleared because
    # the flags do not claim a clean workspace.
    status.zero_()
    out.fill_(float("nan"))
    assert lib.kvp_paged_attention(C.byref(a), sp) == 0, kvb.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = ora.reference_attention(nh, kvh, D, B, qf, kf, vf, T, L)
    check_close(out.cpu().numpy(), ref, what=f"after a timed-out launch (B={B}, split={split})")

    # The same entry point without a stall, at the full limit, is an ordinary launch.
    out.fill_(float("nan"))
    assert lib.kvp_attention_wait_test(C.byref(a), sp, 2_000_000_000, 0) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    check_close(out.cpu().numpy(), ref, what="wait test entry point without a stall")
    del keep


def test_wait_test_rejects_bad_limits(kvb, cuda):
    import torch
    a = kvb.AttnArgs()
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for limit, stall in ((0, 1), (-5, 0), (3_000_000_000, 0), (1000, 2)):
        assert kvb.lib().kvp_attention_wait_test(C.byref(a), sp, limit, stall) == kvb.KVP_EINVAL


@pytest.mark.parametrize("mode", ["nonzero", "epoch"])
@pytest.mark.parametrize("split", [0, 2], ids=["balanced", "fixed-splits"])
def test_inputs_ready_flag(kvb, ora, cuda, split, mode):
    """kvp_attn_args.inputs_ready (queries and new K/V written by a copy on another stream): while the word is
    not ready -- zero, or with inputs_epoch behind the epoch -- the kernel's bounded wait runs out:
    KVP_STATUS_TIMEOUT, and the pools are untouched (the fused append waits for the flag too).  Once it is
    ready (non-zero; or equal to the epoch, here across the 32-bit wrap), the same launch appends the new K/V
    and attends over the appended cache (fp64 oracle)."""
    import torch
    nh, kvh, D, B = 32, 8, 128, 16
    lens = [300, 4096, 77, 1500, 33, 2500]
    nb = sum((n + B - 1) // B for n in lens) + 11
    Q, K, V, T, L = _normal_case(6, len(lens), nh, kvh, D, B, lens, nb)
    rng = np.random.default_rng(7)
    dev = torch.device("cuda:0")
    qt, qf = _round(Q, "bf16")
    kt, kf = _round(K, "bf16")
    vt, vf = _round(V, "bf16")
    knt, knf = _round(rng.standard_normal((len(lens), kvh, D), dtype=np.float32), "bf16")
    vnt, vnf = _round(rng.standard_normal((len(lens), kvh, D), dtype=np.float32), "bf16")
    k_d, v_d = kt.to(dev), vt.to(dev)
    keep = [qt.to(dev), k_d, v_d, torch.from_numpy(T).to(dev), torch.from_numpy(L).to(dev)]
    kn_d, vn_d = knt.to(dev), vnt.to(dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    epoch = torch.full((1,), 2**31 - 1, dtype=torch.int32, device=dev)
    if mode == "epoch":
        flag.fill_(2**31 - 2)  # the previous step's value
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.full((len(lens), nh, D), float("nan"), dtype=torch.float32, device=dev)
    a = kvb.attention_args(*keep, out, nh, kvh, split_tiles=split, status=status, k_new=kn_d, v_new=vn_d,
                           inputs_ready=flag)
    if mode == "epoch":
        a.inputs_epoch = epoch.data_ptr()
    ws = torch.zeros(max(kvb.workspace_bytes(a), 256), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = kvb.lib()
    k0, v0 = k_d.clone(), v_d.clone()

    t0 = time.perf_counter()
    assert lib.kvp_attention_wait_test(C.byref(a), sp, LIMIT, 0) == 0, kvb.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) & kvb.KVP_STATUS_TIMEOUT, f"status {int(status.item())}"
    assert time.perf_counter() - t0 < 5.0
    assert torch.equal(k_d, k0) and torch.equal(v_d, v0), "the pools changed before the inputs were ready"

    flag.fill_(1 if mode == "nonzero" else -2**31)  # in epoch mode: one past the epoch, wrapped
    status.zero_()
    assert lib.kvp_paged_attention(C.byref(a), sp) == 0, kvb.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for s, n in enumerate(lens):
        blk, off = int(T[s, (n - 1) // B]), (n - 1) % B
        kf[blk, off], vf[blk, off] = knf[s], vnf[s]
    assert torch.equal(k_d.cpu(), torch.from_numpy(kf).to(torch.bfloat16))
    ref = ora.reference_attention(nh, kvh, D, B, qf, kf, vf, T, L)
    check_close(out.cpu().numpy(), ref, what=f"inputs_ready set (split={split})")
    del keep


def test_inputs_ready_rejected_where_unsupported(kvb, cuda):
    """fp32 pools (the CUDA-core kernel) take no inputs_ready; a misaligned word is rejected."""
    import torch
    dev = torch.device("cuda:0")
    q = torch.zeros((1, 8, 64), device=dev)
    kv = torch.zeros((2, 16, 2, 64), device=dev)
    t = torch.zeros((1, 1), dtype=torch.int32, device=dev)
    ln = torch.ones(1, dtype=torch.int32, device=dev)
    word = torch.zeros(2, dtype=torch.int32, device=dev)
    a = kvb.attention_args(q, kv, kv, t, ln, torch.empty_like(q), 8, 2, inputs_ready=word)
    assert kvb.lib().kvp_paged_attention(C.byref(a), None) == kvb.KVP_EINVAL
    kb = kv.to(torch.bfloat16)
    a = kvb.attention_args(q.to(torch.bfloat16), kb, kb, t, ln, torch.empty_like(q), 8, 2)
    a.inputs_ready = word.data_ptr() + 2
    assert kvb.lib().kvp_paged_attention(C.byref(a), None) == kvb.KVP_EINVAL
