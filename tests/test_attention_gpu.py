"""Parity of the CUDA decode-attention kernel (through the C ABI) with the oracle.

Tolerance (stated by the task for fp16/bf16 K/V with fp32 accumulation): |got - ref| <= 2e-3 + 2e-3 |ref|
elementwise, where ref is the double-precision reference_attention (src/paged_attention.cpp:25-66) on the
exactly converted inputs (K/V/Q rounded to their storage type first, as cuda/test_paged_attention.cu:61-64
does).  16-bit outputs add half an ulp of their type.  Outputs start NaN-poisoned
(cuda/test_paged_attention.cu:87) so an unwritten element fails.
"""
import ctypes as C

import numpy as np
import pytest

from cases import attention_cases, attention_inputs, cuda_test_cases

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-3


def _tdt(name):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


def _round(x, name):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(_tdt(name))
    return t, t.float().numpy()


def check_close(got, ref, out_dtype="f32", what=""):
    assert np.isfinite(got).all(), f"{what}: non-finite output (unwritten or NaN)"
    extra = {"f32": 0.0, "f16": 2.0 ** -11, "bf16": 2.0 ** -8}[out_dtype]
    err = np.abs(got - ref) - (ATOL + (RTOL + extra) * np.abs(ref))
    worst = float(err.max()) if err.size else -1.0
    assert worst <= 0, f"{what}: max excess over tolerance {worst:.3e}, max abs err {np.abs(got - ref).max():.3e}"
    return float(np.abs(got - ref).max()) if got.size else 0.0


def run_attention(kvb, ora, Q, K, V, T, L, nh, kvh, *, kv="bf16", q="f32", out="f32", split_tiles=0,
                  kvh_cta=0, stages=0, num_blocks=None, ref=None, seq_start_tiles=0):
    import torch
    dev = torch.device("cuda:0")
    kt, kf = _round(K, kv)
    vt, vf = _round(V, kv)
    qt, qf = _round(Q, q)
    if ref is None:
        ref = ora.reference_attention(nh, kvh, K.shape[-1], K.shape[1], qf, kf, vf, T, L)
    o = torch.full(Q.shape, float("nan"), dtype=_tdt(out), device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kvb.paged_attention(qt.to(dev), kt.to(dev), vt.to(dev), torch.from_numpy(T).to(dev),
                        torch.from_numpy(np.asarray(L, np.int32)).to(dev), nh, kvh, out=o, split_tiles=split_tiles,
                        kv_heads_per_cta=kvh_cta, stages=stages, status=status, num_blocks=num_blocks,
                        seq_start_tiles=seq_start_tiles)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return o.float().cpu().numpy(), ref


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_reference_cpu_test_cases(kvb, ora, cuda, kv):
    """All 81 cases of the reference's tests/test_attention.cpp:62-101 (block sizes 1..32, boundary lengths,
    GQA 8/8, 8/2, 8/1, 14/2, 4/4, shared prefix blocks, random shapes), fp32 query, with no split, automatic
    splits and one tile per split (every context split to the maximum, exercising the merge)."""
    worst = 0.0
    for c in attention_cases():
        Q, K, V, T, L = attention_inputs(c["seed"], c["nh"], c["kvh"], c["hd"], c["B"], c["lens"], c["share"],
                                         kvb.KVManager)
        ref = None
        for split in (-1, 0, 1):
            got, ref = run_attention(kvb, ora, Q, K, V, T, L, c["nh"], c["kvh"], kv=kv, split_tiles=split, ref=ref)
            worst = max(worst, check_close(got, ref, what=f"{c} split={split}"))
    print(f"worst abs error {worst:.2e}")


def test_reference_gpu_test_cases(kvb, ora, cuda):
    """The case list of the reference's own GPU test (cuda/test_paged_attention.cu:165-175), with its fp16
    q/K/V/out; also checked against the reference test's own acceptance (1e-2 of max |ref|)."""
    for i, (nh, kvh, hd, B, lens, share) in enumerate(cuda_test_cases()):
        Q, K, V, T, L = attention_inputs(i + 1, nh, kvh, hd, B, lens, share, kvb.KVManager)
        got, ref = run_attention(kvb, ora, Q, K, V, T, L, nh, kvh, kv="f16", q="f16", out="f16")
        check_close(got, ref, out_dtype="f16", what=f"case {i}")
        assert np.abs(got - ref).max() / max(1e-9, np.abs(ref).max()) < 1e-2


def _legacy_fn(kvb):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", kvb.LIB_PATH], capture_output=True, text=True).stdout
    name = [ln.split()[-1] for ln in out.splitlines() if "launch_paged_attention" in ln][0]
    f = getattr(kvb.lib(), name)
    f.restype = C.c_int
    f.argtypes = [C.c_void_p] * 6 + [C.c_int] * 7 + [C.c_void_p]
    return f


def test_drop_in_launch_paged_attention(kvb, ora, cuda):
    """The reference's GPU entry point signature (cuda/paged_attention.cuh:16-19), fp16 everywhere, called by
    its exported C++ symbol; invalid warps / head_dim return cudaErrorInvalidValue (1) like the reference."""
    import torch
    f = _legacy_fn(kvb)
    for i, (nh, kvh, hd, B, lens, share) in enumerate(cuda_test_cases()[:6]):
        Q, K, V, T, L = attention_inputs(100 + i, nh, kvh, hd, B, lens, share, kvb.KVManager)
        kt, kf = _round(K, "f16")
        vt, vf = _round(V, "f16")
        qt, qf = _round(Q, "f16")
        ref = ora.reference_attention(nh, kvh, hd, B, qf, kf, vf, T, L)
        d = [x.cuda() for x in (qt, kt, vt)]
        tt, lt = torch.from_numpy(T).cuda(), torch.from_numpy(L).cuda()
        o = torch.full(Q.shape, float("nan"), dtype=torch.float16, device="cuda")
        for warps in (1, 4, 8):
            rc = f(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), tt.data_ptr(), lt.data_ptr(), o.data_ptr(),
                   len(lens), nh, kvh, hd, B, T.shape[1], warps, None)
            assert rc == 0
            torch.cuda.synchronize()
            check_close(o.float().cpu().numpy(), ref, out_dtype="f16", what=f"legacy case {i} warps {warps}")
        assert f(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), tt.data_ptr(), lt.data_ptr(), o.data_ptr(),
                 len(lens), nh, kvh, hd, B, T.shape[1], 9, None) == 1
        assert f(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), tt.data_ptr(), lt.data_ptr(), o.data_ptr(),
                 len(lens), nh, kvh, 48, B, T.shape[1], 4, None) == 1


def test_matches_the_reference_gpu_kernel(kvb, ora, cuda):
    """The reference's own GPU kernel (cuda/paged_attention.cu, compiled here from its source into oracle/_ref)
    and this library's drop-in, on the same fp16 inputs: the reference's GPU case list plus long contexts at
    the Qwen2.5-0.5B and Llama-3-8B head shapes.  Both are within the fp16 bar of the fp64 reference, hence
    within twice that bar of each other."""
    import torch
    if not ora.have_ref_gpu():
        pytest.skip("the reference's GPU kernel was not built (needs the reference sources)")
    f = _legacy_fn(kvb)
    cases = cuda_test_cases() + [(14, 2, 64, 16, [512, 1999, 4096, 3000], False),
                                 (32, 8, 128, 16, [4096, 777, 8192], False)]
    for i, (nh, kvh, hd, B, lens, share) in enumerate(cases):
        Q, K, V, T, L = attention_inputs(300 + i, nh, kvh, hd, B, lens, share, kvb.KVManager)
        kt, kf = _round(K, "f16")
        vt, vf = _round(V, "f16")
        qt, qf = _round(Q, "f16")
        ref = ora.reference_attention(nh, kvh, hd, B, qf, kf, vf, T, L)
        q, k, v = qt.cuda(), kt.cuda(), vt.cuda()
        t, ln = torch.from_numpy(T).cuda(), torch.from_numpy(L).cuda()
        theirs = torch.full(Q.shape, float("nan"), dtype=torch.float16, device="cuda")
        ours = torch.full_like(theirs, float("nan"))
        args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), t.data_ptr(), ln.data_ptr())
        shape = (len(lens), nh, kvh, hd, B, T.shape[1], 4)
        assert ora.ref_gpu_attention(*args, theirs.data_ptr(), *shape, None) == 0
        assert f(*args, ours.data_ptr(), *shape, None) == 0
        torch.cuda.synchronize()
        a, b = theirs.float().cpu().numpy(), ours.float().cpu().numpy()
        check_close(a, ref, out_dtype="f16", what=f"reference kernel, case {i}")
        check_close(b, ref, out_dtype="f16", what=f"drop-in, case {i}")
        assert (np.abs(a - b) <= 2 * (ATOL + (RTOL + 2.0 ** -11) * np.abs(ref))).all(), i


def _normal_case(seed, ns, nh, kvh, hd, B, lens, pool_blocks):
    """Workload-style inputs: N(0,1) K/V/Q, each request's blocks a random permutation of pool ids."""
    rng = np.random.default_rng(seed)
    mb = max((n + B - 1) // B for n in lens)
    K = rng.standard_normal((pool_blocks, B, kvh, hd), dtype=np.float32)
    V = rng.standard_normal((pool_blocks, B, kvh, hd), dtype=np.float32)
    Q = rng.standard_normal((ns, nh, hd), dtype=np.float32)
    perm = rng.permutation(pool_blocks)
    T = np.zeros((ns, mb), np.int32)
    off = 0
    for i, n in enumerate(lens):
        nb = (n + B - 1) // B
        T[i, :nb] = perm[off: off + nb]
        off += nb
    return Q, K, V, T, np.asarray(lens, np.int32)


def test_eight_sequence_case_full_size(kvb, ora, cuda):
    """The small correctness case at its full size: 8 sequences, 8/8 heads, D=64, B=16, lengths U{1..512},
    fp32 Q, fp16 K/V, 1024-block pool, random block permutation."""
    rng = np.random.default_rng(2024)
    lens = rng.integers(1, 513, size=8).tolist()
    Q, K, V, T, L = _normal_case(1, 8, 8, 8, 64, 16, lens, 1024)
    for split in (-1, 0, 2):
        got, ref = run_attention(kvb, ora, Q, K, V, T, L, 8, 8, kv="f16", q="f32", split_tiles=split)
        check_close(got, ref, what=f"8-sequence case split={split}")


@pytest.mark.parametrize("shape", [
    # (name, nh, kvh, hd, kv dtype, q dtype, lengths)
    ("qwen2.5-0.5b", 14, 2, 64, "f16", "f16", [512, 4096, 1999, 3001]),
    ("tinyllama", 32, 4, 64, "bf16", "bf16", [1, 1024, 2048, 777, 1500, 16]),
    ("llama3-8b", 32, 8, 128, "bf16", "bf16", [4096, 32768, 3000, 17]),
])
def test_config_shapes(kvb, ora, cuda, shape):
    """Configs 2-4 head shapes and dtypes with lengths from their distributions (reduced batch)."""
    name, nh, kvh, hd, kv, q, lens = shape
    nb = sum((n + 15) // 16 for n in lens) + 37
    Q, K, V, T, L = _normal_case(hash(name) % 1000, len(lens), nh, kvh, hd, 16, lens, nb)
    for split in (0, 8):
        got, ref = run_attention(kvb, ora, Q, K, V, T, L, nh, kvh, kv=kv, q=q, split_tiles=split)
        check_close(got, ref, what=f"{name} split={split}")


@pytest.mark.parametrize("kvh_cta,stages", [(1, 2), (2, 3), (4, 4), (8, 2), (2, 8), (1, 12)])
def test_tuning_variants(kvb, ora, cuda, kvh_cta, stages):
    """Every kv-heads-per-CTA / pipeline-depth choice gives the same (correct) result."""
    lens = [700, 16, 33, 1025]
    nb = sum((n + 15) // 16 for n in lens) + 5
    Q, K, V, T, L = _normal_case(9, 4, 32, 8, 128, 16, lens, nb)
    got, ref = run_attention(kvb, ora, Q, K, V, T, L, 32, 8, kv="bf16", q="bf16", kvh_cta=kvh_cta, stages=stages,
                             split_tiles=5)
    check_close(got, ref, what=f"kvh_cta={kvh_cta} stages={stages}")


@pytest.mark.parametrize("q,out", [("f32", "bf16"), ("f16", "f32"), ("bf16", "f16"), ("f32", "f16")])
def test_dtype_combinations(kvb, ora, cuda, q, out):
    lens = [300, 45]
    Q, K, V, T, L = _normal_case(3, 2, 16, 4, 64, 16, lens, 40)
    for kv in ("f16", "bf16"):
        got, ref = run_attention(kvb, ora, Q, K, V, T, L, 16, 4, kv=kv, q=q, out=out)
        check_close(got, ref, out_dtype=out, what=f"q={q} kv={kv} out={out}")


def test_gqa_16_heads_per_kv_head(kvb, ora, cuda):
    lens = [129, 64]
    Q, K, V, T, L = _normal_case(4, 2, 32, 2, 64, 16, lens, 20)
    got, ref = run_attention(kvb, ora, Q, K, V, T, L, 32, 2, kv="bf16", q="bf16", split_tiles=3)
    check_close(got, ref, what="g=16")


def test_layout_invariance_bit_exact(kvb, ora, cuda):
    """The Qwen2.5-0.5B-shaped workload at full size (64 sequences, lengths U{512..4096}, 14/2 heads, D=64, fp16, 64k-block pool):
    relabelling the physical blocks (a different permutation, pool bytes moved accordingly) gives a
    bit-identical output -- the property of the reference's model_check.py:304-330 -- and a sample of
    sequences matches the oracle."""
    import torch
    rng = np.random.default_rng(11)
    ns, nh, kvh, hd, B, P = 64, 14, 2, 64, 16, 65536
    lens = rng.integers(512, 4097, size=ns)
    nblk = (lens + B - 1) // B
    mb = int(nblk.max())
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(5)
    K = torch.randn((P, B, kvh, hd), generator=g, device=dev, dtype=torch.float32).half()
    V = torch.randn((P, B, kvh, hd), generator=g, device=dev, dtype=torch.float32).half()
    Q = torch.randn((ns, nh, hd), generator=g, device=dev, dtype=torch.float32).half()
    perm = rng.permutation(P)
    T = np.zeros((ns, mb), np.int32)
    off = 0
    for i in range(ns):
        T[i, : nblk[i]] = perm[off: off + nblk[i]]
        off += int(nblk[i])
    L = torch.from_numpy(lens.astype(np.int32)).to(dev)
    o1 = kvb.paged_attention(Q, K, V, torch.from_numpy(T).to(dev), L, nh, kvh, out_dtype=torch.float32)
    # relabel: physical block b moves to sigma[b]
    sigma = rng.permutation(P)
    inv = torch.from_numpy(np.argsort(sigma)).to(dev)
    K2, V2 = K[inv], V[inv]
    T2 = sigma[T].astype(np.int32)
    o2 = kvb.paged_attention(Q, K2, V2, torch.from_numpy(T2).to(dev), L, nh, kvh, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    # oracle on a sample of sequences (those blocks only)
    idx = [0, 17, 63]
    blocks = np.unique(T[idx][T[idx] >= 0])
    remap = {int(b): j for j, b in enumerate(blocks)}
    Ts = np.vectorize(lambda b: remap.get(int(b), 0))(T[idx]).astype(np.int32)
    bt = torch.from_numpy(blocks).to(dev)
    ref = ora.reference_attention(nh, kvh, hd, B, Q[idx].float().cpu().numpy(), K[bt].float().cpu().numpy(),
                                  V[bt].float().cpu().numpy(), Ts, lens[idx].astype(np.int32))
    check_close(o1[idx].cpu().numpy(), ref, what="Qwen-shaped sample")


def test_bad_inputs_report_status_without_fault(kvb, ora, cuda):
    """A table entry outside the pool is skipped (zero-filled load) and flagged; a sequence with length 0
    or longer than its table row is flagged and gets zeros; the other sequences are unaffected."""
    import torch
    lens = [100, 40, 0, 999]
    Q, K, V, T, L = _normal_case(8, 4, 8, 2, 64, 16, [100, 40, 1, 1], 30)
    T = np.zeros((4, 7), np.int32) + T[:, :1]
    T[0, :7] = np.arange(7)
    T[1, :3] = [7, 8, 500]  # 500: outside the 30-block pool
    L = np.asarray(lens, np.int32)
    dev = torch.device("cuda:0")
    kt, kf = _round(K, "bf16")
    vt, vf = _round(V, "bf16")
    o = torch.full(Q.shape, float("nan"), dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kvb.paged_attention(torch.from_numpy(Q).to(dev), kt.to(dev), vt.to(dev), torch.from_numpy(T).to(dev),
                        torch.from_numpy(L).to(dev), 8, 2, out=o, status=status, num_blocks=30)
    torch.cuda.synchronize()
    st = int(status.item())
    assert st & kvb.KVP_STATUS_BAD_BLOCK and st & kvb.KVP_STATUS_BAD_LEN
    got = o.cpu().numpy()
    ref0 = ora.reference_attention(8, 2, 64, 16, Q[:1], kf, vf, T[:1], L[:1])
    check_close(got[:1], ref0, what="healthy sequence next to bad ones")
    assert np.all(got[2] == 0) and np.all(got[3] == 0)
    assert np.isfinite(got[1]).all()


def test_empty_batch_is_a_no_op(kvb, cuda):
    import torch
    z = torch.zeros((0, 8, 64), dtype=torch.float32, device="cuda")
    k = torch.zeros((4, 16, 2, 64), dtype=torch.float16, device="cuda")
    t = torch.zeros((0, 1), dtype=torch.int32, device="cuda")
    kvb.paged_attention(z, k, k, t, torch.zeros(0, dtype=torch.int32, device="cuda"), 8, 2, out=z)
    torch.cuda.synchronize()


@pytest.mark.parametrize("start", [0, -1, 40], ids=["start-auto", "start-none", "start-40"])
@pytest.mark.parametrize("lens", [
    [1, 2, 3, 1, 16],                       # fewer tiles than persistent CTAs
    [32768] + [17] * 100,                    # one very long context among many short ones
    [5000] * 3 + [1] * 300 + [700] * 50,     # many sequences, mixed
])
def test_balanced_schedule_edge_cases(kvb, ora, cuda, lens, start):
    """The persistent balanced schedule (automatic split): CTA ranges cut through sequences anywhere (in
    units that charge each sequence's start cost -- automatic, none, or a large 40 tiles, so that some CTAs
    hold only start-cost units), sequences entirely inside one CTA are written directly, the rest merged."""
    nb = sum((n + 15) // 16 for n in lens) + 3
    Q, K, V, T, L = _normal_case(len(lens), len(lens), 32, 8, 128, 16, lens, nb)
    got, ref = run_attention(kvb, ora, Q, K, V, T, L, 32, 8, kv="bf16", q="bf16", split_tiles=0,
                             seq_start_tiles=start)
    check_close(got, ref, what=f"balanced schedule {len(lens)} sequences, start cost {start}")


def test_balanced_schedule_unaligned_query(kvb, ora, cuda):
    """A query buffer that is not 16-byte aligned is read from global memory instead of being bulk-copied."""
    import torch
    lens = [300, 45, 1000]
    Q, K, V, T, L = _normal_case(12, 3, 16, 4, 64, 16, lens, 100)
    kt, kf = _round(K, "f16")
    vt, vf = _round(V, "f16")
    ref = ora.reference_attention(16, 4, 64, 16, Q, kf, vf, T, L)
    buf = torch.empty(Q.size + 1, dtype=torch.float32, device="cuda")
    qv = buf[1:].view(Q.shape)  # 4-byte aligned only
    qv.copy_(torch.from_numpy(Q))
    o = torch.full(Q.shape, float("nan"), dtype=torch.float32, device="cuda")
    kvb.paged_attention(qv, kt.cuda(), vt.cuda(), torch.from_numpy(T).cuda(), torch.from_numpy(L).cuda(), 16, 4, out=o)
    torch.cuda.synchronize()
    check_close(o.cpu().numpy(), ref, what="unaligned query")


def test_balanced_schedule_leaves_workspace_clean(kvb, ora, cuda):
    """The in-kernel merge counters return to zero after every call, so a workspace zero-filled once can be
    reused with KVP_ATTN_WORKSPACE_CLEAN indefinitely (three calls in a row, each checked)."""
    import torch
    lens = [3000, 17, 1200, 5000, 64]
    nb = sum((n + 15) // 16 for n in lens) + 2
    Q, K, V, T, L = _normal_case(21, 5, 32, 8, 128, 16, lens, nb)
    kt, kf = _round(K, "bf16")
    vt, vf = _round(V, "bf16")
    ref = ora.reference_attention(32, 8, 128, 16, Q, kf, vf, T, L)
    q, k, v = torch.from_numpy(Q).cuda(), kt.cuda(), vt.cuda()
    t, l = torch.from_numpy(T).cuda(), torch.from_numpy(L).cuda()
    out = torch.empty(Q.shape, dtype=torch.float32, device="cuda")
    a = kvb.attention_args(q, k, v, t, l, out, 32, 8, num_blocks=nb)
    ws = torch.zeros(kvb.workspace_bytes(a), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes, a.flags = ws.data_ptr(), ws.numel(), kvb.KVP_ATTN_WORKSPACE_CLEAN
    for _ in range(3):
        out.fill_(float("nan"))
        assert kvb.lib().kvp_paged_attention(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        torch.cuda.synchronize()
        check_close(out.cpu().numpy(), ref, what="clean workspace reuse")
        cnt = ws[:8192 * 4].view(torch.int32)  # the counter region: 8192 sequences x 1 kv-head group
        assert int(cnt.abs().sum().item()) == 0


def test_clean_workspace_reuse_across_batch_sizes(kvb, ora, cuda):
    """One workspace, zero-filled once and passed with KVP_ATTN_WORKSPACE_CLEAN, serves calls whose batch size
    changes from call to call (the merge counters sit in a region whose place does not depend on num_seqs):
    long contexts split every sequence across CTAs, so the partials of one call cover the places a
    num_seqs-dependent layout would give the next call's counters.  Each call equals, bit for bit, the same
    call on a fresh workspace, and matches the oracle."""
    import torch
    rng = np.random.default_rng(17)
    nh, kvh, D, B = 8, 2, 64, 16
    sizes = [12, 3, 20, 7, 1, 16, 5]
    nmax = max(sizes)
    lens_all = rng.integers(800, 4000, size=nmax)
    nb = int(sum((n + 15) // 16 for n in lens_all)) + 4
    Q, K, V, T, L = _normal_case(23, nmax, nh, kvh, D, B, [int(x) for x in lens_all], nb)
    kt, kf = _round(K, "bf16")
    vt, vf = _round(V, "bf16")
    k, v = kt.cuda(), vt.cuda()
    q_all, t_all, l_all = torch.from_numpy(Q).cuda(), torch.from_numpy(T).cuda(), torch.from_numpy(L).cuda()
    out = torch.empty((nmax, nh, D), dtype=torch.float32, device="cuda")
    a = kvb.attention_args(q_all, k, v, t_all, l_all, out, nh, kvh, num_blocks=nb)
    ws = torch.zeros(kvb.workspace_bytes(a), dtype=torch.uint8, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for i, n in enumerate(sizes):
        sel = rng.permutation(nmax)[:n]
        q, t, l = q_all[sel].contiguous(), t_all[sel].contiguous(), l_all[sel].contiguous()
        o1 = torch.full((n, nh, D), float("nan"), dtype=torch.float32, device="cuda")
        o2 = torch.full_like(o1, float("nan"))
        a = kvb.attention_args(q, k, v, t, l, o1, nh, kvh, num_blocks=nb)
        assert kvb.workspace_bytes(a) <= ws.numel()
        a.workspace, a.workspace_bytes, a.flags = ws.data_ptr(), ws.numel(), kvb.KVP_ATTN_WORKSPACE_CLEAN
        assert kvb.lib().kvp_paged_attention(C.byref(a), stream) == 0
        kvb.paged_attention(q, k, v, t, l, nh, kvh, out=o2, num_blocks=nb)  # fresh zeroed workspace
        torch.cuda.synchronize()
        assert torch.equal(o1, o2), (i, n)
        if i % 3 == 0:
            ref = ora.reference_attention(nh, kvh, D, B, Q[sel], kf, vf, T[sel], L[sel])
            check_close(o1.cpu().numpy(), ref, what=f"batch of {n}")
    assert int(ws[:8192 * 4].view(torch.int32).abs().sum().item()) == 0


@pytest.mark.parametrize("q_misaligned", [False, True], ids=["q16", "q-unaligned"])
@pytest.mark.parametrize("shape", [(14, 2, 64), (32, 8, 128)], ids=["qwen", "llama"])
def test_early_start_back_to_back_bit_exact(kvb, cuda, shape, q_misaligned):
    """Eight layers launched back to back on one stream with early start (each kernel's prologue overlapping
    the previous kernel's tail) and early load (its first K/V tiles loaded before the previous kernel ends), with
    the fused append, give outputs and pools bit-identical to plain launches.  With queries off a 16-byte
    boundary the consumer warps read them with plain loads (no query slot), after waiting for the previous
    kernel themselves."""
    import torch
    nh, kvh, D = shape
    L, B, ns = 8, 16, 48
    rng = np.random.default_rng(5)
    lens = rng.integers(1, 900, size=ns)
    nblk = [(int(x) + B - 1) // B for x in lens]
    nb = sum(nblk) + 4
    perm = rng.permutation(nb)
    T = np.zeros((ns, max(nblk)), np.int32)
    o = 0
    for i, n in enumerate(nblk):
        T[i, :n] = perm[o:o + n]
        o += n
    g = torch.Generator(device="cuda").manual_seed(3)
    K = torch.randn((L, nb, B, kvh, D), generator=g, device="cuda").to(torch.bfloat16)
    V = torch.randn_like(K)
    q = torch.randn((L, ns, nh, D), generator=g, device="cuda").to(torch.bfloat16)
    if q_misaligned:  # each layer's rows one element past a 16-byte boundary
        qf = torch.empty((L, ns * nh * D + 1), dtype=torch.bfloat16, device="cuda")
        qf[:, 1:] = q.reshape(L, -1)
        q = qf[:, 1:].view(L, ns, nh, D)
        assert q[0].data_ptr() % 16 == 2
    kn = torch.randn((L, ns, kvh, D), generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn_like(kn)
    t = torch.from_numpy(T).cuda()
    ln = torch.from_numpy(lens.astype(np.int32)).cuda()
    res = []
    for mode in ("plain", "early_start", "early_load"):
        k2, v2 = K.clone(), V.clone()
        out = torch.empty_like(q)
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        for layer in range(L):
            kvb.paged_attention(q[layer], k2[layer], v2[layer], t, ln, nh, kvh, out=out[layer], status=st,
                                k_new=kn[layer], v_new=vn[layer], early_start=mode == "early_start",
                                early_load=mode == "early_load" and layer > 0)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        res.append((out, k2, v2))
    for other in res[1:]:
        for a, b in zip(res[0], other):
            assert torch.equal(a, b)


def test_reference_cuda_test_binary_on_drop_in(cuda):
    """The reference's own GPU test (cuda/test_paged_attention.cu: its case list -- block sizes 1..32, shared
    prefixes, Llama/Qwen head shapes, head_dim 32..256 -- checked against its own CPU reference_attention),
    built by oracle/Makefile with this library's launch_paged_attention in place of the reference kernel."""
    import os
    import subprocess
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "ref_cuda_test")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/ref_cuda_test not built (needs the reference sources at build time)")
    r = subprocess.run([exe, "--no-bench"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "ALL PASSED" in r.stdout
    assert r.stdout.count("| PASS |") >= 45
