"""Fused append + attention (kvp_attn_args.k_new / v_new): one launch that writes each sequence's newest token
into its slot and attends over the context including it must leave the pools and produce outputs bit-identical
to the two-launch form the reference's harness uses -- scatter of the new K/V (python/paged_model.py:145-146),
then attention (python/paged_model.py:147-151) -- under every schedule and shape family."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [  # (num_heads, kv_heads, head_dim, block_size)
    (32, 8, 128, 16),   # Llama-3-8B-like
    (14, 2, 64, 16),    # Qwen2.5-0.5B-like
    (32, 4, 64, 32),
    (16, 1, 128, 3),    # block size not a multiple of 16 (several TMA runs per tile), g = 16
    (8, 8, 256, 16),
    (4, 4, 32, 8),
]


def _step_inputs(kvb, nh, kvh, D, B, seed, dtype):
    """A decode step on a fragmented pool: requests of mixed lengths (including a first token and block
    boundaries), two forks whose next append copies on write; returns everything both paths need."""
    import torch
    rng = np.random.default_rng(seed)
    nb = 4096 if B >= 8 else 8192
    mgr = kvb.KVManager(nb, B)
    junk = list(range(9000, 9000 + 300))
    for r in junk:
        assert mgr.admit(r, int(rng.integers(1, 3 * B)))
    lens_before = [0, 1, B - 1, B, B + 1, 15, 16, 17, 31, 32, 33, 100, 255, 256, 257, 700, 1500]
    lens_before += [int(x) for x in rng.integers(1, 600, size=12)]
    rids = list(range(len(lens_before)))
    for i, r in enumerate(rids):
        if i % 3 == 0 and junk:
            mgr.free(junk.pop(int(rng.integers(len(junk)))))
        assert mgr.admit(r, lens_before[i])
    for child, parent in ((100, 4), (101, 11)):  # partial last blocks shared with the parent
        assert mgr.fork(child, parent)
        rids.append(child)
    done, _, pairs = mgr.append_batch(rids)
    assert done == len(rids)
    assert len(pairs) >= 2  # at least the two forked partial blocks are copied
    mb = max(len(mgr.block_table(r)) for r in rids) + 3
    tables, lens = mgr.dense_tables(rids, mb)
    g = torch.Generator(device="cuda").manual_seed(seed)
    K = torch.randn((nb, B, kvh, D), generator=g, device="cuda").to(dtype)
    V = torch.randn((nb, B, kvh, D), generator=g, device="cuda").to(dtype)
    ns = len(rids)
    q = torch.randn((ns, nh, D), generator=g, device="cuda").to(dtype)
    knew = torch.randn((ns, kvh, D), generator=g, device="cuda").to(dtype)
    vnew = torch.randn((ns, kvh, D), generator=g, device="cuda").to(dtype)
    slots = [mgr.block_table(r)[(n - 1) // B] * B + (n - 1) % B for r, n in zip(rids, lens)]
    return dict(K=K, V=V, q=q, knew=knew, vnew=vnew, tables=torch.from_numpy(tables).cuda(),
                lens=torch.from_numpy(lens).cuda(), pairs=torch.from_numpy(np.asarray(pairs, np.int32).reshape(-1, 2)).cuda(),
                slots=torch.tensor(slots, dtype=torch.int32, device="cuda"), nb=nb)


@pytest.mark.parametrize("split", [0, 1, -1], ids=["balanced", "split1", "nosplit"])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "nh%d-kvh%d-d%d-b%d" % s)
def test_fused_append_matches_scatter_then_attention(kvb, cuda, shape, dtype, split):
    import torch
    nh, kvh, D, B = shape
    dt = torch.float16 if dtype == "f16" else torch.bfloat16
    x = _step_inputs(kvb, nh, kvh, D, B, seed=hash(shape) % 1000 + split, dtype=dt)
    st_a = torch.zeros(1, dtype=torch.int32, device="cuda")
    st_b = torch.zeros(1, dtype=torch.int32, device="cuda")
    # two launches: COW, scatter, attention
    Ka, Va = x["K"].clone(), x["V"].clone()
    kvb.cow_copy(Ka[None], Va[None], x["pairs"], status=st_a)
    kvb.append_scatter(x["knew"][None], x["vnew"][None], Ka[None], Va[None], x["slots"], status=st_a)
    out_a = kvb.paged_attention(x["q"], Ka, Va, x["tables"], x["lens"], nh, kvh, split_tiles=split, status=st_a)
    # fused: COW, then attention that writes the new token itself
    Kb, Vb = x["K"].clone(), x["V"].clone()
    kvb.cow_copy(Kb[None], Vb[None], x["pairs"], status=st_b)
    out_b = kvb.paged_attention(x["q"], Kb, Vb, x["tables"], x["lens"], nh, kvh, split_tiles=split, status=st_b,
                                k_new=x["knew"], v_new=x["vnew"])
    torch.cuda.synchronize()
    assert int(st_a.item()) == 0 and int(st_b.item()) == 0
    assert torch.equal(Ka, Kb) and torch.equal(Va, Vb)
    assert torch.equal(out_a, out_b)
    # the new rows really landed (not just equal because both paths skipped them)
    s = x["slots"].long()
    assert torch.equal(Kb.view(-1, kvh, D)[s], x["knew"]) and torch.equal(Vb.view(-1, kvh, D)[s], x["vnew"])


def test_fused_append_vs_oracle(kvb, ora, cuda):
    """The fused step checked directly against the fp64 reference attention over the appended context."""
    import torch
    nh, kvh, D, B = 8, 2, 64, 16
    x = _step_inputs(kvb, nh, kvh, D, B, seed=7, dtype=torch.bfloat16)
    K, V = x["K"].clone(), x["V"].clone()
    kvb.cow_copy(K[None], V[None], x["pairs"])
    out = kvb.paged_attention(x["q"], K, V, x["tables"], x["lens"], nh, kvh, k_new=x["knew"], v_new=x["vnew"],
                              out_dtype=torch.float32)
    Kr, Vr = x["K"].clone(), x["V"].clone()
    src, dst = x["pairs"][:, 0].long(), x["pairs"][:, 1].long()
    Kr[dst], Vr[dst] = Kr[src], Vr[src]
    s = x["slots"].long()
    Kr.view(-1, kvh, D)[s], Vr.view(-1, kvh, D)[s] = x["knew"], x["vnew"]
    ref = ora.reference_attention(nh, kvh, D, B, x["q"].float().cpu().numpy(), Kr.float().cpu().numpy(),
                                  Vr.float().cpu().numpy(), x["tables"].cpu().numpy(), x["lens"].cpu().numpy())
    got = out.cpu().numpy().reshape(ref.shape)
    np.testing.assert_allclose(got, ref, atol=2e-3, rtol=2e-3)


def test_fused_append_bad_block_is_skipped(kvb, cuda):
    """A table entry outside the pool at the appended position: the kernel reports KVP_STATUS_BAD_BLOCK and
    writes nothing (the pools stay bit-identical)."""
    import torch
    nh, kvh, D, B, nb = 8, 2, 64, 16, 64
    K = torch.randn((nb, B, kvh, D), device="cuda").to(torch.bfloat16)
    V = torch.randn_like(K)
    K0, V0 = K.clone(), V.clone()
    tables = torch.tensor([[3, 5, nb + 7]], dtype=torch.int32, device="cuda")
    lens = torch.tensor([40], dtype=torch.int32, device="cuda")
    q = torch.randn((1, nh, D), device="cuda").to(torch.bfloat16)
    kn = torch.randn((1, kvh, D), device="cuda").to(torch.bfloat16)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    kvb.paged_attention(q, K, V, tables, lens, nh, kvh, k_new=kn, v_new=kn.clone(), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & kvb.KVP_STATUS_BAD_BLOCK
    assert torch.equal(K, K0) and torch.equal(V, V0)


def test_fused_append_argument_checks(kvb, cuda):
    """Host-side refusals (no launch): k_new without v_new, unaligned rows, no pool size to bound the write."""
    import torch
    nh, kvh, D, B, nb = 8, 2, 64, 16, 8
    dev = "cuda"
    K = torch.zeros((nb, B, kvh, D), dtype=torch.bfloat16, device=dev)
    q = torch.zeros((1, nh, D), dtype=torch.bfloat16, device=dev)
    t = torch.zeros((1, 1), dtype=torch.int32, device=dev)
    l = torch.ones(1, dtype=torch.int32, device=dev)
    kn = torch.zeros((1, kvh, D), dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        kvb.paged_attention(q, K, K, t, l, nh, kvh, k_new=kn)
    a = kvb.attention_args(q, K, K.clone(), t, l, torch.empty_like(q), nh, kvh, k_new=kn, v_new=kn.clone())
    a.num_blocks = 0
    with pytest.raises(ValueError, match="num_blocks"):
        kvb._check(kvb.lib().kvp_paged_attention(kvb.C.byref(a), None))
    a = kvb.attention_args(q, K, K.clone(), t, l, torch.empty_like(q), nh, kvh, k_new=kn, v_new=kn.clone())
    a.k_new = kn.data_ptr() + 2
    with pytest.raises(ValueError, match="aligned"):
        kvb._check(kvb.lib().kvp_paged_attention(kvb.C.byref(a), None))
