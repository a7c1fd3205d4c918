"""fp32 pools and the host-buffer entry points with the reference's CPU signatures.

The reference's CPU attention (include/kvpage/paged_attention.h:25-35, src/paged_attention.cpp:25-114) takes
fp32 host buffers; its test (tests/test_attention.cpp:62-111) accepts a max abs difference of 1e-5 (2e-5 for
the random cases) against its fp64 reference_attention.  This library serves that signature on the GPU
(kvp_paged_attention_host; kvp::paged_attention_cpu / kvp::reference_attention; kvpage_py's functions) with an
fp32 CUDA-core kernel, which is held to the reference test's own bound here: max |got - fp64 oracle| <= 2e-5.
"""
import os
import subprocess

import numpy as np
import pytest

from cases import attention_cases, attention_inputs

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BOUND = 2e-5


def test_fp32_pools_through_the_device_entry_point(kvb, ora, cuda):
    """All 81 cases of tests/test_attention.cpp (block sizes 1..32, boundary lengths, GQA 8/8, 8/2, 8/1, 14/2,
    shared prefix blocks, random shapes) with fp32 device pools through kvp_paged_attention, fp32 queries and
    outputs; no workspace is needed."""
    import torch
    dev = torch.device("cuda:0")
    worst = 0.0
    for c in attention_cases():
        Q, K, V, T, L = attention_inputs(c["seed"], c["nh"], c["kvh"], c["hd"], c["B"], c["lens"], c["share"],
                                         kvb.KVManager)
        ref = ora.reference_attention(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L)
        out = torch.full(Q.shape, float("nan"), dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        a = kvb.attention_args(torch.from_numpy(Q).to(dev), torch.from_numpy(K).to(dev), torch.from_numpy(V).to(dev),
                               torch.from_numpy(T).to(dev), torch.from_numpy(L).to(dev), out, c["nh"], c["kvh"],
                               status=status)
        assert kvb.workspace_bytes(a) == 0
        kvb._launch(dev, kvb.lib().kvp_paged_attention, a, None)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = float(np.abs(out.cpu().numpy() - ref).max())
        assert err <= BOUND, (c, err)
        worst = max(worst, err)
    print(f"worst abs error {worst:.2e}")


def test_host_entry_point_reference_cases(kvb, ora, cuda):
    """kvpage_py.paged_attention_cpu / reference_attention (the reference binding's signatures, host numpy
    arrays) on the same 81 cases, with each case's partition count passed through."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "paged-kv-cache-manager_b200"))
    import kvpage_py as kp
    for c in attention_cases():
        Q, K, V, T, L = attention_inputs(c["seed"], c["nh"], c["kvh"], c["hd"], c["B"], c["lens"], c["share"],
                                         kvb.KVManager)
        ref = ora.reference_attention(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L)
        got = kp.paged_attention_cpu(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L, c["P"])
        assert float(np.abs(got - ref).max()) <= BOUND, c
        got = kp.reference_attention(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L)
        assert float(np.abs(got - ref).max()) <= BOUND, c


def test_host_entry_point_against_torch_sdpa(kvb, cuda):
    """The case list of the reference's python/attention_check.py (N(0,1) data, scattered blocks) against
    torch's scaled_dot_product_attention on contiguous K/V, at that script's bound (1e-5)."""
    import torch
    rng = np.random.default_rng(0)
    for nh, kvh, hd, B, lens in [(8, 2, 64, 16, [1, 15, 16, 17, 100]), (14, 2, 64, 8, [33, 64, 65]),
                                 (8, 8, 128, 32, [5, 128, 129]), (4, 1, 32, 1, [3, 9]), (16, 4, 128, 16, [200, 7])]:
        ns = len(lens)
        mb = max((n + B - 1) // B for n in lens)
        nblocks = ns * mb + 3
        K = rng.standard_normal((nblocks, B, kvh, hd), dtype=np.float32)
        V = rng.standard_normal((nblocks, B, kvh, hd), dtype=np.float32)
        Q = rng.standard_normal((ns, nh, hd), dtype=np.float32)
        perm = rng.permutation(nblocks)
        T = np.zeros((ns, mb), dtype=np.int32)
        for i, n in enumerate(lens):
            T[i, :(n + B - 1) // B] = perm[i * mb: i * mb + (n + B - 1) // B]
        got = kvb.paged_attention_host(nh, kvh, hd, B, Q, K, V, T, np.asarray(lens, np.int32), 4)
        for i, n in enumerate(lens):
            blk = torch.from_numpy(T[i, :(n + B - 1) // B]).long()
            k = torch.from_numpy(K)[blk].reshape(-1, kvh, hd)[:n].permute(1, 0, 2).repeat_interleave(nh // kvh, 0)
            v = torch.from_numpy(V)[blk].reshape(-1, kvh, hd)[:n].permute(1, 0, 2).repeat_interleave(nh // kvh, 0)
            q = torch.from_numpy(Q[i])[:, None, :].double()
            want = torch.nn.functional.scaled_dot_product_attention(q, k.double(), v.double())[:, 0].numpy()
            assert float(np.abs(got[i] - want).max()) < 1e-5, (nh, kvh, hd, B, lens, i)


def test_host_entry_point_rejects_like_the_reference(kvb, cuda):
    """The reference's checks (src/paged_attention.cpp:12-17, 72) raise ValueError with its messages; a negative
    block id (out of bounds in the reference) is rejected too; an empty batch is a no-op."""
    x = np.zeros((1, 8, 64), np.float32)
    kv = np.zeros((2, 16, 2, 64), np.float32)
    t = np.zeros((1, 1), np.int32)
    one = np.ones(1, np.int32)
    with pytest.raises(ValueError, match="num_heads % kv_heads"):
        kvb.paged_attention_host(8, 3, 64, 16, x, kv, kv, t, one)
    with pytest.raises(ValueError, match="bad seq_len"):
        kvb.paged_attention_host(8, 2, 64, 16, x, kv, kv, t, np.zeros(1, np.int32))
    with pytest.raises(ValueError, match="bad seq_len"):
        kvb.paged_attention_host(8, 2, 64, 16, x, kv, kv, t, np.full(1, 17, np.int32))  # two blocks, one entry
    with pytest.raises(ValueError, match="partitions"):
        kvb.paged_attention_host(8, 2, 64, 16, x, kv, kv, t, one, 0)
    with pytest.raises(ValueError, match="negative block id"):
        kvb.paged_attention_host(8, 2, 64, 16, x, kv, kv, np.full((1, 1), -1, np.int32), one)
    empty = kvb.paged_attention_host(8, 2, 64, 16, np.zeros((0, 8, 64), np.float32), kv, kv,
                                     np.zeros((0, 1), np.int32), np.zeros(0, np.int32))
    assert empty.shape == (0, 8, 64)


def test_reference_attention_test_binary(cuda):
    """The reference's own tests/test_attention.cpp, unchanged, built by oracle/Makefile: its
    paged_attention_cpu calls run this library's device path, its reference_attention oracle is the
    reference's own fp64 source; the test's own bounds (1e-5, 2e-5) apply."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_attention_test")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/ref_attention_test not built (needs the reference sources at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "5 tests run, 0 failed" in r.stdout, r.stdout
