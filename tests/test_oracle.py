"""Pins the oracle: the C restatement of the reference's attention against fixtures produced by the
reference's own code (tests/golden/make_golden.py) and, where it was built here, against that code live."""
import json

import numpy as np
import pytest

from cases import attention_cases, attention_inputs

GOLDEN = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "attention_cases.npz")


@pytest.fixture(scope="module")
def golden():
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["meta"]).decode())
    return z, meta


def test_case_list_matches_fixture(golden):
    _, meta = golden
    assert meta == attention_cases()


def test_c_oracle_matches_reference_golden(golden, ora, kvb):
    """reference_attention (double) and paged_attention_cpu (fp32, P partitions) restated in C reproduce
    the reference's outputs on all 81 cases of tests/test_attention.cpp:62-101."""
    z, meta = golden
    worst_ref = worst_paged = 0.0
    for ci, c in enumerate(meta):
        Q, K, V, T, L = attention_inputs(c["seed"], c["nh"], c["kvh"], c["hd"], c["B"], c["lens"], c["share"],
                                         kvb.KVManager)
        # The product KVManager hands out the same block ids as the reference did for the fixture.
        np.testing.assert_array_equal(T, z[f"c{ci}_tables"])
        ref = ora.reference_attention(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L)
        pag = ora.paged_attention_cpu(c["nh"], c["kvh"], c["hd"], c["B"], Q, K, V, T, L, partitions=c["P"])
        worst_ref = max(worst_ref, float(np.abs(ref - z[f"c{ci}_ref"]).max()))
        worst_paged = max(worst_paged, float(np.abs(pag - z[f"c{ci}_paged"]).max()))
        # the reference's own acceptance bound between its two functions (test_attention.cpp:71, 98)
        assert float(np.abs(pag - ref).max()) < 2e-5
    assert worst_ref <= 1e-6, worst_ref
    assert worst_paged <= 1e-6, worst_paged


def test_c_oracle_rejects_what_reference_rejects(ora):
    """test_attention.cpp:103-111: num_heads % kv_heads != 0 and seq_len 0 are rejected."""
    q = np.zeros((1, 8, 64), np.float32)
    k = np.zeros((1, 16, 3, 64), np.float32)
    with pytest.raises(ValueError):
        ora.reference_attention(8, 3, 64, 16, q, k, k, np.zeros((1, 1), np.int32), np.ones(1, np.int32))
    k2 = np.zeros((1, 16, 2, 64), np.float32)
    with pytest.raises(ValueError):
        ora.reference_attention(8, 2, 64, 16, q, k2, k2, np.zeros((1, 1), np.int32), np.zeros(1, np.int32))
    with pytest.raises(ValueError):  # ceil(len / B) > max_blocks
        ora.reference_attention(8, 2, 64, 16, q, k2, k2, np.zeros((1, 1), np.int32), np.array([17], np.int32))


def test_c_oracle_matches_live_reference(ora, kvb):
    """Same inputs through the reference library compiled from its sources (when present here)."""
    if not ora.have_ref():
        pytest.skip("reference library not built on this machine")
    rng = np.random.default_rng(7)
    for nh, kvh, hd, B, lens in [(14, 2, 64, 16, [33, 64, 65, 300]), (32, 8, 128, 16, [70, 70, 55, 33, 16]),
                                 (8, 8, 256, 16, [100, 17]), (4, 1, 32, 1, [3, 9]), (16, 4, 96, 8, [200, 7])]:
        ns = len(lens)
        mb = max((n + B - 1) // B for n in lens)
        nb = ns * mb + 3
        K = rng.standard_normal((nb, B, kvh, hd), dtype=np.float32)
        V = rng.standard_normal((nb, B, kvh, hd), dtype=np.float32)
        Q = rng.standard_normal((ns, nh, hd), dtype=np.float32)
        perm = rng.permutation(nb)
        T = np.zeros((ns, mb), np.int32)
        for i, n in enumerate(lens):
            T[i, : (n + B - 1) // B] = perm[i * mb: i * mb + (n + B - 1) // B]
        L = np.asarray(lens, np.int32)
        a = ora.reference_attention(nh, kvh, hd, B, Q, K, V, T, L)
        b = ora.reference_attention(nh, kvh, hd, B, Q, K, V, T, L, impl="ref")
        assert float(np.abs(a - b).max()) <= 1e-6
        for P in (1, 3):
            c1 = ora.paged_attention_cpu(nh, kvh, hd, B, Q, K, V, T, L, partitions=P, nthreads=2)
            c2 = ora.paged_attention_cpu(nh, kvh, hd, B, Q, K, V, T, L, partitions=P, nthreads=3, impl="ref")
            assert float(np.abs(c1 - c2).max()) <= 1e-6


def test_bf16_conversion_is_round_to_nearest_even(ora):
    import torch
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1e-40, 3.4e38, np.inf, -np.inf], np.float32)])
    bits = ora.f32_to_bf16_bits(x)
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(bits, t)
    back = ora.bf16_bits_to_f32(bits)
    np.testing.assert_array_equal(back, torch.from_numpy(x).to(torch.bfloat16).float().numpy())
