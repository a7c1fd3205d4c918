"""The decode-step runtime (kvp_decoder_*) produces exactly what the individual entry points produce when
driven by hand (append batch -> copy-on-write -> append scatter -> attention per layer), with host buffers
and with device buffers, with and without graph replay, and its attention output matches the oracle on the
updated cache."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(kvb, seed, L=4, nb=192, B=16, kvh=2, D=64, nh=8):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((L, nb, B, kvh, D), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((L, nb, B, kvh, D), generator=g, device="cuda").to(torch.bfloat16)
    m = kvb.KVManager(nb, B)
    assert m.admit(0, 37) and m.fork(1, 0) and m.fork(2, 0) and m.admit(3, 300) and m.admit_with_prefix(4, 3, 160, 170)
    return k, v, m


def _manual_step(kvb, m, k, v, rids, q, kn, vn, split, max_blocks, nh, kvh):
    import torch
    done, slots, pairs = m.append_batch(rids)
    assert done == len(rids)
    if len(pairs):
        kvb.cow_copy(k, v, torch.from_numpy(np.ascontiguousarray(pairs)).cuda())
    kvb.append_scatter(kn, vn, k, v, torch.from_numpy(slots).cuda())
    tables, lens = m.dense_tables(rids, max_blocks)
    t, l = torch.from_numpy(tables).cuda(), torch.from_numpy(lens).cuda()
    out = torch.empty(q.shape, dtype=q.dtype, device="cuda")
    for layer in range(k.shape[0]):
        kvb.paged_attention(q[layer], k[layer], v[layer], t, l, nh, kvh, out=out[layer], split_tiles=split)
    return out


@pytest.mark.parametrize("graph", [True, False], ids=["graph", "launches"])
@pytest.mark.parametrize("split", [2, 0], ids=["split2", "balanced"])
@pytest.mark.parametrize("path", ["host", "device"])
def test_decoder_matches_manual_path(kvb, cuda, path, split, graph):
    """Eight steps, the batch size changing once (a graph is captured on the second step of a repeated key and
    replayed after it, then recaptured for the new size): outputs and pools equal the hand-driven two-launch
    path (append scatter, then attention) bit for bit."""
    import torch
    nh, kvh, D, L, MB = 8, 2, 64, 4, 40
    k1, v1, m1 = _setup(kvb, 1)
    k2, v2, m2 = k1.clone(), v1.clone(), None
    _, _, m2 = _setup(kvb, 1)
    dec = kvb.Decoder(m1, k1, v1, nh, max_seqs=8, max_blocks_per_seq=MB, split_tiles=split, graph=graph)
    rng = np.random.default_rng(3)
    bufs = {}
    side = torch.cuda.Stream()
    for step in range(8):
        rids = [0, 1, 2, 3, 4] if step < 5 else [0, 2, 4]
        order = [int(x) for x in rng.permutation(rids)]
        n = len(order)
        q = torch.randn((L, n, nh, D)).to(torch.bfloat16)
        kn = torch.randn((L, n, kvh, D)).to(torch.bfloat16)
        vn = torch.randn((L, n, kvh, D)).to(torch.bfloat16)
        if path == "host":
            if n not in bufs:  # the same pinned buffers every step of one batch size (the graph key repeats)
                bufs[n] = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, kn, vn, q)]
            hq, hk, hv, ho = bufs[n]
            hq.copy_(q), hk.copy_(kn), hv.copy_(vn)
            dec.step(order, hq, hk, hv, ho)
            out1 = ho.clone()
        else:
            if n not in bufs:  # the same device buffers every step of one batch size
                bufs[n] = [torch.empty(t.shape, dtype=t.dtype, device="cuda") for t in (q, kn, vn, q)]
            dq, dk, dv, do = bufs[n]
            dq.copy_(q), dk.copy_(kn), dv.copy_(vn)
            side.wait_stream(torch.cuda.current_stream())
            dec.step_device(order, dq, dk, dv, do, stream=side)  # a capturable (non-legacy) stream
            torch.cuda.synchronize()
            out1 = do.cpu()
        out2 = _manual_step(kvb, m2, k2, v2, order, q.cuda(), kn.cuda(), vn.cuda(), split, MB, nh, kvh)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2.cpu()), step
        assert torch.equal(k1, k2) and torch.equal(v1, v2), step
    assert dec.status() == 0
    assert m1.stats() == m2.stats() and m1.stats()["cow_copies"] == 2


def test_decoder_output_matches_oracle(kvb, ora, cuda):
    import torch
    nh, kvh, D, L, MB = 8, 2, 64, 4, 40
    k, v, m = _setup(kvb, 5)
    dec = kvb.Decoder(m, k, v, nh, max_seqs=8, max_blocks_per_seq=MB, out_dtype=torch.float32)
    rids = [4, 3, 2, 1, 0]
    q = torch.randn((L, 5, nh, D)).to(torch.bfloat16)
    kn = torch.randn((L, 5, kvh, D)).to(torch.bfloat16)
    vn = torch.randn((L, 5, kvh, D)).to(torch.bfloat16)
    out = torch.empty((L, 5, nh, D), dtype=torch.float32).pin_memory()
    dec.step(rids, q.pin_memory(), kn.pin_memory(), vn.pin_memory(), out)
    tables, lens = m.dense_tables(rids, MB)
    for layer in (0, 3):
        ref = ora.reference_attention(nh, kvh, D, 16, q[layer].float().numpy(), k[layer].float().cpu().numpy(),
                                      v[layer].float().cpu().numpy(), tables, lens)
        got = out[layer].numpy()
        assert np.isfinite(got).all()
        assert (np.abs(got - ref) <= 2e-3 + 2e-3 * np.abs(ref)).all()


def test_decoder_reports_exhaustion(kvb, cuda):
    import torch
    L, nb, B, kvh, D, nh = 2, 4, 16, 2, 64, 4
    k = torch.zeros((L, nb, B, kvh, D), dtype=torch.bfloat16, device="cuda")
    v = torch.zeros_like(k)
    m = kvb.KVManager(nb, B)
    assert m.admit(0, 32) and m.admit(1, 16)
    dec = kvb.Decoder(m, k, v, nh, max_seqs=2, max_blocks_per_seq=4)
    z = torch.zeros((L, 2, nh, D), dtype=torch.bfloat16).pin_memory()
    zk = torch.zeros((L, 2, kvh, D), dtype=torch.bfloat16).pin_memory()
    with pytest.raises(kvb.KVPError) as e:
        dec.step([0, 1], z, zk, zk, z.clone())  # both need a new block; only one is free
    assert e.value.code == kvb.KVP_ENOSPACE
    assert m.num_tokens(0) == 33 and m.num_tokens(1) == 16  # the first append happened, the second did not
    # The failed step had already started its first layer's copy (and set that layer's input-ready flag): the
    # next step must still wait for its own inputs.  Its fused append and attention must match a direct launch.
    m.free(1)
    g = torch.Generator().manual_seed(4)
    q = torch.randn((L, 1, nh, D), generator=g).to(torch.bfloat16).pin_memory()
    kn = torch.randn((L, 1, kvh, D), generator=g).to(torch.bfloat16).pin_memory()
    vn = torch.randn((L, 1, kvh, D), generator=g).to(torch.bfloat16).pin_memory()
    out = torch.empty((L, 1, nh, D), dtype=torch.bfloat16).pin_memory()
    dec.step([0], q, kn, vn, out)
    assert dec.status() == 0
    tables, lens = m.dense_tables([0], 4)
    t, ln = torch.from_numpy(tables).cuda(), torch.from_numpy(lens).cuda()
    for layer in range(L):
        want = kvb.paged_attention(q[layer].cuda(), k[layer], v[layer], t, ln, nh, kvh)
        assert torch.equal(out[layer], want.cpu()), layer


@pytest.mark.parametrize("path", ["host", "device"])
def test_decoder_staging_follows_external_table_changes(kvb, cuda, path):
    """The same batch in the same order step after step (the decoder then rewrites only the table entries its own
    appends changed), with the tables changed behind its back between steps: a request freed and re-admitted
    under the same id with another length, and an append made through the manager directly.  Every step must
    still equal the hand-driven path bit for bit."""
    import torch
    nh, kvh, D, L, MB = 8, 2, 64, 4, 40
    k1, v1, m1 = _setup(kvb, 7)
    k2, v2 = k1.clone(), v1.clone()
    _, _, m2 = _setup(kvb, 7)
    dec = kvb.Decoder(m1, k1, v1, nh, max_seqs=8, max_blocks_per_seq=MB)
    order = [3, 0, 4, 1, 2]
    n = len(order)
    side = torch.cuda.Stream()
    hbufs = [torch.empty(s, dtype=torch.bfloat16).pin_memory() for s in ((L, n, nh, D), (L, n, kvh, D), (L, n, kvh, D),
                                                                        (L, n, nh, D))]
    dbufs = [b.cuda() for b in hbufs]
    for step in range(9):
        if step == 3:  # request 1 freed and re-admitted under its id with a different length, on both managers
            for m in (m1, m2):
                m.free(1)
                assert m.admit(1, 90)
        if step == 6:  # an append made outside the decoder
            for m in (m1, m2):
                assert m.append_token(4)
        q = torch.randn((L, n, nh, D)).to(torch.bfloat16)
        kn = torch.randn((L, n, kvh, D)).to(torch.bfloat16)
        vn = torch.randn((L, n, kvh, D)).to(torch.bfloat16)
        if path == "host":
            hq, hk, hv, ho = hbufs
            hq.copy_(q), hk.copy_(kn), hv.copy_(vn)
            dec.step(order, hq, hk, hv, ho)
            out1 = ho.clone()
        else:
            dq, dk, dv, do = dbufs
            dq.copy_(q), dk.copy_(kn), dv.copy_(vn)
            side.wait_stream(torch.cuda.current_stream())
            dec.step_device(np.asarray(order, dtype=np.int64), dq, dk, dv, do, stream=side)
            torch.cuda.synchronize()
            out1 = do.cpu()
        out2 = _manual_step(kvb, m2, k2, v2, order, q.cuda(), kn.cuda(), vn.cuda(), 0, MB, nh, kvh)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2.cpu()), step
        assert torch.equal(k1, k2) and torch.equal(v1, v2), step
    assert dec.status() == 0


@pytest.mark.parametrize("path", ["host", "packed", "device"])
def test_decoder_pipelined_steps_match_manual_path(kvb, cuda, path):
    """Pipelined steps: each step is submitted (host buffers) or enqueued (device buffers), the NEXT step's
    bookkeeping is planned while it runs, and only then is it waited for.  Nine steps with the batch changing
    once (the plan is made for the next step's batch) and, between one plan and its submit, an append made
    through the manager directly (the planned tables are then re-read).  Outputs and pools equal the
    hand-driven path bit for bit at every step."""
    import torch
    nh, kvh, D, L, MB = 8, 2, 64, 4, 40
    k1, v1, m1 = _setup(kvb, 9)
    k2, v2 = k1.clone(), v1.clone()
    _, _, m2 = _setup(kvb, 9)
    dec = kvb.Decoder(m1, k1, v1, nh, max_seqs=8, max_blocks_per_seq=MB)
    rng = np.random.default_rng(4)
    orders = [[int(x) for x in rng.permutation([0, 1, 2, 3, 4] if s < 5 else [0, 2, 4])] for s in range(9)]
    side = torch.cuda.Stream()
    bufs = {}
    dec.plan(orders[0])
    for step, order in enumerate(orders):
        n = len(order)
        if step == 6:  # an append made outside the decoder, between the plan of this step and its submit
            for m in (m1, m2):
                assert m.append_token(order[0])
        q = torch.randn((L, n, nh, D)).to(torch.bfloat16)
        kn = torch.randn((L, n, kvh, D)).to(torch.bfloat16)
        vn = torch.randn((L, n, kvh, D)).to(torch.bfloat16)
        if n not in bufs:
            bufs[n] = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, kn, vn, q)]
            bufs[n] += [t.cuda() for t in bufs[n]]
        hq, hk, hv, ho, dq, dk, dv, do = bufs[n]
        if path == "host":
            hq.copy_(q), hk.copy_(kn), hv.copy_(vn)
            dec.submit(order, hq, hk, hv, ho)
        elif path == "packed":  # the decoder's own pinned input buffers (one copy per group of layers)
            pq, pk, pv = dec.host_inputs(n)
            pq.copy_(q), pk.copy_(kn), pv.copy_(vn)
            dec.submit(order, pq, pk, pv, ho)
        else:
            dq.copy_(q), dk.copy_(kn), dv.copy_(vn)
            side.wait_stream(torch.cuda.current_stream())
            dec.step_device(order, dq, dk, dv, do, stream=side)
        if step + 1 < len(orders):
            dec.plan(orders[step + 1])
        if path in ("host", "packed"):
            dec.wait()
            out1 = ho.clone()
        else:
            torch.cuda.synchronize()
            out1 = do.cpu()
        out2 = _manual_step(kvb, m2, k2, v2, order, q.cuda(), kn.cuda(), vn.cuda(), 0, MB, nh, kvh)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2.cpu()), step
        assert torch.equal(k1, k2) and torch.equal(v1, v2), step
    assert dec.status() == 0
    assert m1.stats() == m2.stats()


def test_decoder_plan_misuse(kvb, cuda):
    """A second plan before the planned step is an error (KVP_ESTATE); a step over another batch than the
    planned one is rejected (ValueError) and leaves the planned appends in the manager; a plan over an empty
    batch is a no-op."""
    import torch
    nh, kvh, D, L, MB = 8, 2, 64, 4, 40
    k, v, m = _setup(kvb, 11)
    dec = kvb.Decoder(m, k, v, nh, max_seqs=8, max_blocks_per_seq=MB)
    before = [m.num_tokens(r) for r in range(5)]
    dec.plan([])
    dec.plan([0, 1])
    assert [m.num_tokens(r) for r in range(5)] == [before[0] + 1, before[1] + 1] + before[2:]
    with pytest.raises(kvb.KVPError) as e:
        dec.plan([0, 1])
    assert e.value.code == kvb.KVP_ESTATE
    z = torch.zeros((L, 2, nh, D), dtype=torch.bfloat16).pin_memory()
    zk = torch.zeros((L, 2, kvh, D), dtype=torch.bfloat16).pin_memory()
    with pytest.raises(ValueError, match="planned batch"):
        dec.submit([1, 0], z, zk, zk, z.clone())
    assert [m.num_tokens(r) for r in range(5)] == [before[0] + 1, before[1] + 1] + before[2:]
    dec.step([1, 0], z, zk, zk, z.clone())  # no plan pending: a normal step
    assert [m.num_tokens(r) for r in range(5)] == [before[0] + 2, before[1] + 2] + before[2:]
    assert dec.status() == 0


def test_decoder_packed_inputs_for_another_n_rejected(kvb, cuda):
    """The packed input views of host_inputs(n) lay layers out for that n only.  The Python wrapper rejects
    them for another batch size by shape; the C ABI, given their raw pointers with another n, rejects the step
    (KVP_EINVAL) before any bookkeeping, and the manager is unchanged."""
    import torch
    nh, kvh, D, L, MB = 8, 2, 64, 4, 40
    k, v, m = _setup(kvb, 12)
    dec = kvb.Decoder(m, k, v, nh, max_seqs=8, max_blocks_per_seq=MB)
    before = [m.num_tokens(r) for r in range(5)]
    pq, pk, pv = dec.host_inputs(3)
    out = torch.zeros((L, 2, nh, D), dtype=torch.bfloat16).pin_memory()
    with pytest.raises(ValueError, match="expected"):
        dec.submit([0, 1], pq, pk, pv, out)
    r = np.array([0, 1], dtype=np.int64)
    lib = kvb.lib()
    for fn in (lib.kvp_decoder_submit, lib.kvp_decoder_step):
        rc = fn(dec._h, r.ctypes.data, 2, pq.data_ptr(), pk.data_ptr(), pv.data_ptr(), out.data_ptr())
        assert rc == kvb.KVP_EINVAL and "packed buffer" in kvb.last_error()
    assert [m.num_tokens(r) for r in range(5)] == before
    pq, pk, pv = dec.host_inputs(2)
    pq.zero_(), pk.zero_(), pv.zero_()
    dec.step([0, 1], pq, pk, pv, out)
    assert [m.num_tokens(r) for r in range(5)] == [before[0] + 1, before[1] + 1] + before[2:]
    assert dec.status() == 0
