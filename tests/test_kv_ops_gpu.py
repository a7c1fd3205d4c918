"""KV-cache mutations on the GPU (append scatter, copy-on-write, swap) are bit-exact against the data-plane
model of the reference's Python harness (python/paged_model.py:54-55, 92-95, 113-117, 145-146), with the
block decisions of the reference KVManager (where its library is built) or of the product KVManager, whose
decisions are proven identical to the reference's by the CPU tests."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _mgr(kvb, nb, B):
    import oracle
    return oracle.RefKVManager(nb, B) if oracle.have_ref() else kvb.KVManager(nb, B)


def _pools(L, nb, B, kvh, D, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((L, nb, B, kvh, D), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((L, nb, B, kvh, D), generator=g, device="cuda").to(torch.bfloat16)
    return k, v


def _bits(t):
    import torch
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


class Harness:
    """Drives the product KVManager (device ops) and the reference manager + numpy model in lockstep."""

    def __init__(self, kvb, L, nb, B, kvh, D, seed=0):
        import oracle
        self.kvb = kvb
        self.k, self.v = _pools(L, nb, B, kvh, D, seed)
        self.model = oracle.DataPlane(_bits(self.k), _bits(self.v))
        self.prod = kvb.KVManager(nb, B)
        self.ref = _mgr(kvb, nb, B)
        self.L, self.nb, self.B, self.kvh, self.D = L, nb, B, kvh, D
        self.rng = np.random.default_rng(seed + 1)
        self.cows = 0

    def both(self, name, *args):
        a = getattr(self.prod, name)(*args)
        b = getattr(self.ref, name)(*args)
        assert a == b, (name, args)
        return a

    def step(self, rids):
        """One decode step: batched append (host) -> COW copy -> append scatter (device and model)."""
        import torch
        da, slots, pairs = self.prod.append_batch(rids)
        db, slots_r, pairs_r = self.ref.append_batch(rids)
        assert da == db == len(rids)
        np.testing.assert_array_equal(slots, slots_r)
        np.testing.assert_array_equal(pairs, pairs_r)
        knew = torch.randn((self.L, len(rids), self.kvh, self.D), device="cuda").to(torch.bfloat16)
        vnew = torch.randn((self.L, len(rids), self.kvh, self.D), device="cuda").to(torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        if len(pairs):
            self.kvb.cow_copy(self.k, self.v, torch.from_numpy(np.ascontiguousarray(pairs)).cuda(), status=status)
            self.model.cow(pairs_r)
            self.cows += len(pairs)
        self.kvb.append_scatter(knew, vnew, self.k, self.v, torch.from_numpy(slots).cuda(), status=status)
        self.model.scatter(slots_r, _bits(knew), _bits(vnew))
        torch.cuda.synchronize()
        assert int(status.item()) == 0

    def check(self):
        np.testing.assert_array_equal(_bits(self.k), self.model.k)
        np.testing.assert_array_equal(_bits(self.v), self.model.v)
        live = [r for r in range(10000) if self.prod.contains(r)]
        for r in live:
            assert self.prod.block_table(r) == self.ref.block_table(r)
        assert self.prod.stats() == self.ref.stats()


def test_append_scatter_and_cow_bit_exact(kvb, cuda):
    h = Harness(kvb, L=3, nb=96, B=4, kvh=2, D=64, seed=3)
    assert h.both("admit", 0, 6)
    assert h.both("fork", 1, 0) and h.both("fork", 2, 0)
    assert h.both("admit", 3, 8)
    assert h.both("admit_with_prefix", 4, 3, 8, 9)
    rids = [0, 1, 2, 3, 4]
    for step in range(9):
        h.step(list(h.rng.permutation(rids)))
        h.check()
    assert h.cows == 2  # the two forks' first appends into the shared partial block


def test_swap_round_trip_bit_exact(kvb, cuda):
    """Swap-out copies a request's blocks to a pinned host pool and frees it; swap-in re-admits it (fresh ids,
    src/simulator.cpp:193, 231-241) and copies the data back: the context bytes are unchanged."""
    import torch
    L, nb, B, kvh, D = 4, 64, 16, 8, 128
    h = Harness(kvb, L, nb, B, kvh, D, seed=9)
    assert h.both("admit", 0, 40) and h.both("admit", 1, 70) and h.both("admit", 2, 16)
    for _ in range(3):
        h.step([0, 1, 2])
    h.check()
    victim = 1
    blocks = h.prod.block_table(victim)
    tokens = h.prod.num_tokens(victim)
    slot_bytes = kvb.host_slot_bytes(L, B, kvh, D)
    pool = torch.empty(slot_bytes * len(blocks), dtype=torch.uint8).pin_memory()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    kvb.swap_out(h.k, h.v, blocks, list(range(len(blocks))), pool, stream=side)
    side.synchronize()
    saved = h.model.swap_out(blocks)
    h.both("free", victim)
    # another request takes some of the freed blocks and writes into them
    assert h.both("admit", 3, 33)
    h.step([3, 0])
    new_id = 7
    assert h.both("admit", new_id, tokens)
    fresh = h.prod.block_table(new_id)
    assert fresh != blocks  # fresh ids, never shared
    kvb.swap_in(h.k, h.v, fresh, list(range(len(fresh))), pool, stream=side)
    side.synchronize()
    h.model.swap_in(fresh, saved)
    h.check()
    kb = _bits(h.k)
    for b_old, b_new, (ks, _) in zip(blocks, fresh, saved):
        np.testing.assert_array_equal(kb[:, b_new], ks)


def test_kv_op_mix_shared_prefix_samples(kvb, cuda):
    """The KV-op mix workload at reduced scale: a shared 2048-token prefix admitted with admit_with_prefix, each
    request forked into 8 samples (the original + 7 forks), appends whose first one copies the shared partial
    block, and every 4 steps 10% of the requests swapped out and back in (re-admitted with fresh ids).
    8 kv heads, D=128, bf16, B=16 as in that workload; 8 layers instead of 32 to keep the host model small.
    KVManager state and pool bytes are compared bit-exact after every step."""
    import torch
    L, B, kvh, D = 8, 16, 8, 128
    n_req, samples, prefix, suffix = 3, 8, 2048, 37
    nb = 1024
    h = Harness(kvb, L, nb, B, kvh, D, seed=21)
    assert h.both("admit", 1000, prefix + 5)  # the prefix owner
    rids = []
    for r in range(n_req):
        base = r * samples
        assert h.both("admit_with_prefix", base, 1000, prefix, prefix + suffix)
        rids.append(base)
        for s in range(1, samples):
            assert h.both("fork", base + s, base)
            rids.append(base + s)
    h.check()
    slot_bytes = kvb.host_slot_bytes(L, B, kvh, D)
    pool = torch.empty(slot_bytes * 256, dtype=torch.uint8).pin_memory()
    side = torch.cuda.Stream()
    next_id = 5000
    for step in range(10):
        h.step(list(h.rng.permutation(rids)))
        h.check()
        if step % 4 == 3:
            k = max(1, len(rids) // 10)
            victims = [int(x) for x in h.rng.choice(rids, size=k, replace=False)]
            for vic in victims:
                blocks = h.prod.block_table(vic)
                tokens = h.prod.num_tokens(vic)
                side.wait_stream(torch.cuda.current_stream())
                kvb.swap_out(h.k, h.v, blocks, list(range(len(blocks))), pool, stream=side)
                side.synchronize()
                saved = h.model.swap_out(blocks)
                h.both("free", vic)
                assert h.both("admit", next_id, tokens)
                fresh = h.prod.block_table(next_id)
                kvb.swap_in(h.k, h.v, fresh, list(range(len(fresh))), pool, stream=side)
                side.synchronize()
                h.model.swap_in(fresh, saved)
                rids[rids.index(vic)] = next_id
                next_id += 1
            h.check()
    # the first 7 of the 8 holders of the shared partial block copy it; the last one keeps the original
    assert h.cows == n_req * (samples - 1)


def test_cow_copy_full_block_property_large(kvb, cuda):
    """Size-independent property at a large size: 4096 copy-on-write pairs of 2 MiB blocks (32 layers x K/V,
    the KV-op mix workload's block size, 17 GB of pools) leave every destination bit-equal to its source and the sources
    untouched."""
    import torch
    L, B, kvh, D = 32, 16, 8, 128
    nb = 8192 + 64
    k, v = _pools(L, nb, B, kvh, D, seed=4)
    pairs = np.stack([np.arange(0, 4096), np.arange(4096, 8192)], axis=1).astype(np.int32)
    rng = np.random.default_rng(0)
    pairs[:, 1] = rng.permutation(pairs[:, 1])
    src = torch.from_numpy(pairs[:, 0].astype(np.int64)).cuda()
    dst = torch.from_numpy(pairs[:, 1].astype(np.int64)).cuda()

    def fingerprint(t, idx):
        out = []
        for c in range(0, idx.numel(), 512):
            out.append(t[:, idx[c:c + 512]].view(torch.int16).float().sum(dim=(0, 2, 3, 4)))
        return torch.cat(out)

    before = fingerprint(k, src), fingerprint(v, src)
    kvb.cow_copy(k, v, torch.from_numpy(pairs).cuda())
    torch.cuda.synchronize()
    for t in (k, v):
        for c in range(0, 4096, 512):
            assert torch.equal(t[:, src[c:c + 512]], t[:, dst[c:c + 512]])
    assert torch.equal(before[0], fingerprint(k, src)) and torch.equal(before[1], fingerprint(v, src))


def test_bad_slot_and_pair_flagged(kvb, cuda):
    import torch
    L, nb, B, kvh, D = 2, 8, 4, 2, 64
    k, v = _pools(L, nb, B, kvh, D, seed=1)
    k0, v0 = k.clone(), v.clone()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    knew = torch.zeros((L, 2, kvh, D), dtype=torch.bfloat16, device="cuda")
    kvb.append_scatter(knew, knew, k, v, torch.tensor([-1, nb * B + 3], dtype=torch.int32, device="cuda"),
                       status=status)
    kvb.cow_copy(k, v, torch.tensor([[0, 99]], dtype=torch.int32, device="cuda"), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & kvb.KVP_STATUS_BAD_BLOCK
    assert torch.equal(k, k0) and torch.equal(v, v0)
