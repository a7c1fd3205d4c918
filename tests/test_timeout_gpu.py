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
