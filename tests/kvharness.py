"""A GPU shard under test: device K/V pools, the product KVManager driven in lockstep with the reference's own
KVManager (where its library is built; decisions compared on every call), and the logical K/V history of
every live request -- the rows attention must see through the request's table, whatever sharing, copy-on-write,
prefix caching, eviction, swapping or migration did to the physical blocks.  check() gathers every live
request's context from the device through its table and compares it bit for bit with that history."""
import numpy as np


def bits(t):
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class Shard:
    def __init__(self, kvb, L, nb, B, kvh, D, nh, seed, device="cuda"):
        import torch
        import oracle
        self.kvb, self.L, self.nb, self.B, self.kvh, self.D, self.nh = kvb, L, nb, B, kvh, D, nh
        self.dev = torch.device(device)
        g = torch.Generator(device=self.dev).manual_seed(seed)
        self.k = torch.randn((L, nb, B, kvh, D), generator=g, device=self.dev).to(torch.bfloat16)
        self.v = torch.randn((L, nb, B, kvh, D), generator=g, device=self.dev).to(torch.bfloat16)
        self.mgr = kvb.KVManager(nb, B)
        self.ref = oracle.RefKVManager(nb, B) if oracle.have_ref() else None
        self.hist = {}    # rid -> (K rows [L][n][kvh][D] uint16, V rows)
        self.cached = {}  # prefix-cache key -> (K rows, V rows) of the cached tokens
        self.rng = np.random.default_rng(seed + 1)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.cows = 0

    # ---------------------------------------------------------------- helpers
    def both(self, name, *args):
        a = getattr(self.mgr, name)(*args)
        if self.ref is not None:
            b = getattr(self.ref, name)(*args)
            assert a == b, (name, args, a, b)
        return a

    def _empty(self):
        z = np.zeros((self.L, 0, self.kvh, self.D), np.uint16)
        return z, z.copy()

    def rows(self, n):
        """n new token rows for every layer, bf16 (host tensors)."""
        import torch
        k = torch.from_numpy(self.rng.standard_normal((self.L, n, self.kvh, self.D), dtype=np.float32))
        v = torch.from_numpy(self.rng.standard_normal((self.L, n, self.kvh, self.D), dtype=np.float32))
        return k.to(torch.bfloat16), v.to(torch.bfloat16)

    def _extend(self, rid, k, v):
        hk, hv = self.hist[rid]
        self.hist[rid] = (np.concatenate([hk, bits(k)], axis=1), np.concatenate([hv, bits(v)], axis=1))

    def _write(self, rid, start, n):
        """Prompt rows for positions [start, start + n) of rid, scattered into their slots."""
        import torch
        if n <= 0:
            return
        tbl = self.mgr.block_table(rid)
        B = self.B
        slots = torch.tensor([tbl[p // B] * B + p % B for p in range(start, start + n)], dtype=torch.int32,
                             device=self.dev)
        k, v = self.rows(n)
        self.kvb.append_scatter(k.to(self.dev), v.to(self.dev), self.k, self.v, slots, status=self.status)
        self._extend(rid, k, v)

    def _sync_cache(self):
        for key in list(self.cached):
            if not self.mgr.has_cached_prefix(key):
                del self.cached[key]

    # ---------------------------------------------------------------- KVManager operations with data
    def admit(self, rid, prompt):
        ok = self.both("admit", rid, prompt)
        if ok:
            self.hist[rid] = self._empty()
            self._write(rid, 0, prompt)
        self._sync_cache()
        return ok

    def admit_prefix(self, rid, parent, shared, prompt):
        nsh = min(shared, self.mgr.num_tokens(parent), prompt) // self.B * self.B
        ok = self.both("admit_with_prefix", rid, parent, shared, prompt)
        if ok:
            hk, hv = self.hist[parent]
            self.hist[rid] = (hk[:, :nsh].copy(), hv[:, :nsh].copy())
            self._write(rid, nsh, prompt - nsh)
        self._sync_cache()
        return ok

    def admit_cached(self, rid, key, shared, prompt):
        nsh = self.mgr.shared_blocks_with_cached(key, shared, prompt) * self.B
        base = self.cached.get(key)
        ok = self.both("admit_with_cached_prefix", rid, key, shared, prompt)
        if ok:
            hk, hv = base if nsh else self._empty()
            self.hist[rid] = (hk[:, :nsh].copy(), hv[:, :nsh].copy())
            self._write(rid, nsh, prompt - nsh)
        self._sync_cache()
        return ok, nsh

    def cache_prefix(self, key, owner, tokens):
        ok = self.both("cache_prefix", key, owner, tokens)
        if ok:
            n = self.mgr.cached_prefix_tokens(key)
            hk, hv = self.hist[owner]
            self.cached[key] = (hk[:, :n].copy(), hv[:, :n].copy())
        return ok

    def fork(self, child, parent):
        assert self.both("fork", child, parent)
        hk, hv = self.hist[parent]
        self.hist[child] = (hk.copy(), hv.copy())

    def free(self, rid):
        self.both("free", rid)
        del self.hist[rid]

    def clear_cache(self):
        self.both("clear_cache")
        self.cached = {}

    def step(self, rids, fused=True):
        """One decode step: batched appends (decisions compared with the reference), copy-on-write copies, each
        request's new token (written by the attention kernel itself, or by a scatter first) and attention for
        every layer.  Returns (q, out, tables, lens) with q/out [L][n][nh][D]."""
        import torch
        done, slots, pairs = self.mgr.append_batch(rids)
        if self.ref is not None:
            d2, s2, p2 = self.ref.append_batch(rids)
            assert done == d2
            np.testing.assert_array_equal(slots, s2)
            np.testing.assert_array_equal(np.asarray(pairs).reshape(-1, 2), p2)
        assert done == len(rids)
        self._sync_cache()
        if len(pairs):
            self.kvb.cow_copy(self.k, self.v, torch.from_numpy(np.ascontiguousarray(pairs)).to(self.dev),
                              status=self.status)
            self.cows += len(pairs)
        n = len(rids)
        k, v = self.rows(n)
        dk, dv = k.to(self.dev), v.to(self.dev)
        mb = max(len(self.mgr.block_table(r)) for r in rids)
        tables, lens = self.mgr.dense_tables(rids, mb)
        t, ln = torch.from_numpy(tables).to(self.dev), torch.from_numpy(lens).to(self.dev)
        q = torch.randn((self.L, n, self.nh, self.D)).to(torch.bfloat16).to(self.dev)
        out = torch.empty((self.L, n, self.nh, self.D), dtype=torch.float32, device=self.dev)
        if not fused:
            self.kvb.append_scatter(dk, dv, self.k, self.v, torch.from_numpy(slots).to(self.dev), status=self.status)
        for layer in range(self.L):
            kn, vn = (dk[layer], dv[layer]) if fused else (None, None)
            self.kvb.paged_attention(q[layer], self.k[layer], self.v[layer], t, ln, self.nh, self.kvh, out=out[layer],
                                     status=self.status, k_new=kn, v_new=vn)
        for i, r in enumerate(rids):
            self._extend(r, k[:, i:i + 1], v[:, i:i + 1])
        return q, out, tables, lens

    # ---------------------------------------------------------------- checks
    def check(self):
        import torch
        torch.cuda.synchronize(self.dev)
        assert int(self.status.item()) == 0
        for rid, (hk, hv) in self.hist.items():
            n = self.mgr.num_tokens(rid)
            assert n == hk.shape[1], rid
            idx = torch.tensor(self.mgr.block_table(rid), dtype=torch.long, device=self.dev)
            gk = self.k[:, idx].reshape(self.L, -1, self.kvh, self.D)[:, :n]
            gv = self.v[:, idx].reshape(self.L, -1, self.kvh, self.D)[:, :n]
            np.testing.assert_array_equal(bits(gk), hk, err_msg=f"K of request {rid}")
            np.testing.assert_array_equal(bits(gv), hv, err_msg=f"V of request {rid}")
            if self.ref is not None:
                assert self.mgr.block_table(rid) == self.ref.block_table(rid)
        assert self.mgr.validate() == ""
        if self.ref is not None:
            assert self.mgr.stats() == self.ref.stats()
            assert self.ref.validate() == ""

    def attention_vs_oracle(self, ora, rids, q, out):
        """The step's outputs against the fp64 reference attention over each request's logical history (laid
        out contiguously, identity tables)."""
        import torch
        B = self.B
        nblk = [(self.hist[r][0].shape[1] + B - 1) // B for r in rids]
        tot = sum(nblk)
        tables = np.zeros((len(rids), max(nblk)), np.int32)
        lens = np.zeros(len(rids), np.int32)
        for layer in range(self.L):
            K = np.zeros((tot, B, self.kvh, self.D), np.uint16)
            V = np.zeros_like(K)
            b0 = 0
            for i, r in enumerate(rids):
                hk, hv = self.hist[r]
                n = hk.shape[1]
                K.reshape(-1, self.kvh, self.D)[b0 * B:b0 * B + n] = hk[layer]
                V.reshape(-1, self.kvh, self.D)[b0 * B:b0 * B + n] = hv[layer]
                tables[i, :nblk[i]] = np.arange(b0, b0 + nblk[i])
                lens[i] = n
                b0 += nblk[i]
            kf = torch.from_numpy(K.view(np.int16)).view(torch.bfloat16).float().numpy()
            vf = torch.from_numpy(V.view(np.int16)).view(torch.bfloat16).float().numpy()
            ref = ora.reference_attention(self.nh, self.kvh, self.D, B, q[layer].float().cpu().numpy(), kf, vf,
                                          tables, lens)
            got = out[layer].cpu().numpy()
            assert (np.abs(got - ref) <= 2e-3 + 2e-3 * np.abs(ref)).all(), layer

    # ---------------------------------------------------------------- swap (reference semantics: copy + free,
    # re-admission with fresh ids + copy back; src/simulator.cpp:117-133, 193, 231-241)
    def swap_out(self, rid, pool, slot0, stream):
        blocks = self.mgr.block_table(rid)
        stream.wait_stream(__import__("torch").cuda.current_stream(self.dev))
        self.kvb.swap_out(self.k, self.v, blocks, list(range(slot0, slot0 + len(blocks))), pool, stream=stream)
        stream.synchronize()
        saved = (self.mgr.num_tokens(rid), self.hist[rid], len(blocks))
        self.free(rid)
        return saved

    def swap_in(self, rid, saved, pool, slot0, stream):
        tokens, h, nblk = saved
        if not self.both("admit", rid, tokens):
            return False
        fresh = self.mgr.block_table(rid)
        assert len(fresh) == nblk
        stream.wait_stream(__import__("torch").cuda.current_stream(self.dev))
        self.kvb.swap_in(self.k, self.v, fresh, list(range(slot0, slot0 + nblk)), pool, stream=stream)
        stream.synchronize()
        self.hist[rid] = h
        self._sync_cache()
        return True


def migrate(kvb, src: Shard, dst: Shard, rid: int, dst_rid: int) -> bool:
    """Moves a request between shards through the product helper (kvb.migrate_request: admit on the
    destination, block copy, free on the source), mirrored on the reference managers."""
    import torch
    tokens = src.mgr.num_tokens(rid)
    h = src.hist[rid]
    ok = kvb.migrate_request(src.mgr, src.k, src.v, dst.mgr, dst.k, dst.v, rid, dst_rid, status=dst.status)
    if dst.ref is not None:
        assert dst.ref.admit(dst_rid, tokens) == ok
        if ok:
            src.ref.free(rid)
    if ok:
        dst.hist[dst_rid] = h
        del src.hist[rid]
    src._sync_cache()
    dst._sync_cache()
    torch.cuda.synchronize(dst.dev)
    return ok
