"""KV data plane of one GPU shard, driven by a scheduler's decision stream.

The reference's scheduler simulation (src/simulator.cpp:80-289, run_paged) decides every step which running
requests append a token, which finish, which are preempted -- into a CPU swap pool (:117-133) or dropped for
recomputation -- and which waiting requests are admitted (sharing a running parent's prefix blocks or a cached
prefix, :171-232), swapped back in (:231-241) or forked (:245-251).  It moves no data.  `DataPlane.run` replays
such a decision stream on a GPU shard and issues the device traffic each decision implies, in the order the
decisions were made:

  admission (new or recomputed)   the rows [shared, prompt) written into the new blocks (kvp_append_scatter)
  admission of a swapped request  swap-in: the host slots copied into the fresh blocks (kvp_swap_in)
  append_token                    a copy-on-write block copy when the token lands in a shared partial block
                                  (kvp_cow_copy), then the token's K/V -- written by the attention kernel
                                  itself (fused append) or scattered first
  free of a preempted request     swap-out into host slots (kvp_swap_out) before the blocks are released, or
                                  nothing (recomputed at re-admission)
  end of step                     paged decode attention, every layer, of every request that generated a token
                                  this step (kvp_paged_attention)

A request that generated this step and is then freed (finished or preempted) gets its attention launched
before the free, together with every other request that has generated so far in the step, because its blocks
may be handed to the next allocation.  Every KVManager decision is re-made by this package's KVManager and
compared with the recorded result, and each end-of-step marker is checked against the manager's statistics.

Decision streams are rows of seven int64 values (op, a, b, c, d, result, flag):

  TRACE_STEP          a..d = the recording manager's requests, allocated_blocks, cow_copies, cache_evictions
  TRACE_ADMIT_PREFIX  admit_with_prefix(a, parent=b, shared_tokens=c, prompt_tokens=d); flag 1 = swap-in
  TRACE_ADMIT_CACHED  admit_with_cached_prefix(a, key=b, shared_tokens=c, prompt_tokens=d)
  TRACE_CACHE_PREFIX  cache_prefix(key=a, owner=b, tokens=c)
  TRACE_FORK          fork(child=a, parent=b)
  TRACE_APPEND        append_token(a)
  TRACE_FREE          free(a); b = its tokens; flag FREE_FINISHED / FREE_SWAPPED / FREE_DROPPED
  TRACE_CLEAR_CACHE   clear_cache()
"""
from __future__ import annotations

import importlib
from typing import Callable, Optional

import numpy as np

TRACE_STEP, TRACE_ADMIT_PREFIX, TRACE_ADMIT_CACHED, TRACE_CACHE_PREFIX, TRACE_FORK, TRACE_APPEND, TRACE_FREE, \
    TRACE_CLEAR_CACHE = range(8)
FREE_FINISHED, FREE_SWAPPED, FREE_DROPPED = 0, 1, 2
NO_REQUEST = -1

_kvb = importlib.import_module(__package__) if __package__ else None


def _lib():
    global _kvb
    if _kvb is None:
        _kvb = importlib.import_module("paged-kv-cache-manager_b200")
    return _kvb


class TraceMismatch(RuntimeError):
    """The manager's decision differs from the recorded one."""


def _expect(got, want, row, what):
    if got != want:
        raise TraceMismatch(f"{what}: got {got}, recorded {want} (row {list(map(int, row))})")


class DecisionCounters:
    """What a replay did: the data-plane volumes and the scheduler-level totals they must agree with."""

    def __init__(self):
        self.steps = 0
        self.tokens_generated = 0     # successful appends
        self.prefill_tokens = 0       # rows written at admissions that are not swap-ins
        self.cache_hits = 0           # cached-prefix admissions that shared at least one block
        self.cow_copies = 0           # copy-on-write block copies
        self.swap_out_blocks = 0
        self.swap_in_blocks = 0
        self.attention_launches = 0   # per-layer kernel launches
        self.attention_rows = 0       # (request, step) pairs attended

    def as_dict(self) -> dict:
        return dict(vars(self))


def _admission_shared_tokens(mgr, row) -> int:
    """Tokens an admission will share (full blocks only), queried before the admission."""
    op, r, b, c, d = (int(x) for x in row[:5])
    B = mgr.block_size()
    if op == TRACE_ADMIT_PREFIX:
        return (-(-d // B) - mgr.blocks_needed_to_admit(b, c, d)) * B
    return mgr.shared_blocks_with_cached(b, c, d) * B


def _check_step(mgr, row):
    s = mgr.stats()
    got = (s["requests"], s["allocated_blocks"], s["cow_copies"], s["cache_evictions"])
    _expect(got, tuple(int(x) for x in row[1:5]), row, "end-of-step statistics")


def replay_decisions(mgr, trace) -> DecisionCounters:
    """Host-only replay: re-makes every recorded decision with `mgr` (a KVManager) and checks each result and
    each end-of-step statistics marker.  Moves no data."""
    n = DecisionCounters()
    for row in np.asarray(trace):
        op = int(row[0])
        res = int(row[5])
        if op == TRACE_STEP:
            _check_step(mgr, row)
            n.steps += 1
        elif op in (TRACE_ADMIT_PREFIX, TRACE_ADMIT_CACHED):
            shared = _admission_shared_tokens(mgr, row)
            fn = mgr.admit_with_prefix if op == TRACE_ADMIT_PREFIX else mgr.admit_with_cached_prefix
            _expect(int(fn(int(row[1]), int(row[2]), int(row[3]), int(row[4]))), res, row, "admission")
            if res and int(row[6]) == 0:
                n.prefill_tokens += int(row[4]) - shared
                n.cache_hits += int(op == TRACE_ADMIT_CACHED and shared > 0)
        elif op == TRACE_CACHE_PREFIX:
            _expect(int(mgr.cache_prefix(int(row[1]), int(row[2]), int(row[3]))), res, row, "cache_prefix")
        elif op == TRACE_FORK:
            _expect(int(mgr.fork(int(row[1]), int(row[2]))), res, row, "fork")
        elif op == TRACE_APPEND:
            done, _, pairs = mgr.append_batch([int(row[1])])
            _expect(done, res, row, "append_token")
            n.tokens_generated += done
            n.cow_copies += len(pairs)
        elif op == TRACE_FREE:
            _expect(mgr.num_tokens(int(row[1])), int(row[2]), row, "tokens at free")
            if int(row[6]) == FREE_SWAPPED:
                blocks = len(mgr.block_table(int(row[1])))
                n.swap_out_blocks += blocks
            mgr.free(int(row[1]))
        elif op == TRACE_CLEAR_CACHE:
            mgr.clear_cache()
        else:
            raise ValueError(f"unknown trace op {op}")
    n.swap_in_blocks = n.swap_out_blocks
    return n


class DataPlane:
    """One shard: K/V pools [layers][num_blocks][block_size][kv_heads][head_dim] on `device`, a pinned host
    swap pool of `swap_slots` block slots (all layers, K and V), this package's KVManager, a compute stream and
    a swap stream.

    `source(rids, positions) -> (k, v)` supplies K/V rows -- row i is position positions[i] of request rids[i]
    -- as [layers][n][kv_heads][head_dim] device tensors in the pool dtype (what a model's prefill / decode
    step would produce); `queries(rids) -> q` the queries of an attention batch, [layers][n][num_heads]
    [head_dim].  `on_attention(rids, q, out, tables, lens)` (optional) sees every attention batch after its
    launches.  The host never waits for the device: metadata goes up through pinned staging copies, and
    every launch, copy and allocation is ordered on the shard's compute stream -- except the swaps, which run
    on the swap stream: a swap-out starts after everything queued before it and the compute stream waits for
    it before its next write (the freed blocks may be handed out again at once); a swap-in (into fresh
    blocks) overlaps all work that does not touch its request, and the compute stream waits for it only
    before writing that request's new token, attending it, sharing its blocks (fork, prefix, prefix cache) or
    freeing it."""

    def __init__(self, num_blocks: int, block_size: int, *, layers: int, num_heads: int, kv_heads: int,
                 head_dim: int, source: Callable, queries: Callable, dtype=None, device="cuda",
                 swap_slots: int = 0, fused_append: bool = True, on_attention: Optional[Callable] = None,
                 out_dtype=None, early_start: bool = True):
        import torch
        kvb = _lib()
        self.kvb = kvb
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise ValueError("the data plane runs on a CUDA device")
        dtype = dtype or torch.bfloat16
        self.L, self.nb, self.B, self.kvh, self.D, self.nh = layers, num_blocks, block_size, kv_heads, head_dim, \
            num_heads
        self.mgr = kvb.KVManager(num_blocks, block_size)
        shape = (layers, num_blocks, block_size, kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=self.dev)
        self.v = torch.zeros(shape, dtype=dtype, device=self.dev)
        slot_bytes = kvb.host_slot_bytes(layers, block_size, kv_heads, head_dim, self.k.element_size())
        self.pool = torch.empty(max(swap_slots, 1) * slot_bytes, dtype=torch.uint8).pin_memory()
        self.free_slots = list(range(swap_slots - 1, -1, -1))
        self.swapped = {}          # rid -> (host slots, tokens)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.stream = torch.cuda.Stream(self.dev)
        self.side = torch.cuda.Stream(self.dev)  # swaps
        self.swapins = {}          # rid -> event after its swap-in (not yet waited for by the compute stream)
        self.swapout_ev = None     # event after the latest swap-out (not yet waited for)
        self.workspace = torch.zeros(0, dtype=torch.uint8, device=self.dev)
        self.source, self.queries, self.on_attention = source, queries, on_attention
        self.fused, self.early = fused_append, early_start
        self.out_dtype = out_dtype or torch.float32
        self.pending = {}          # rid -> position of the token it appended this step (attention not run yet)
        self.pending_cow = []      # (old, new) block pairs not yet copied
        self.pending_tokens = []   # (rid, slot, pos): non-fused token rows not yet scattered
        self.tokens = {}           # rid -> tokens, for every request holding blocks
        self.n = DecisionCounters()
        self.events = []           # (start, end, algorithmic bytes) of each attention batch

    # ------------------------------------------------------------------ device traffic
    def _to_dev(self, a):
        """Host array -> device through a pinned staging copy, asynchronous on the current stream."""
        import torch
        return torch.from_numpy(np.ascontiguousarray(a)).pin_memory().to(self.dev, non_blocking=True)

    def _wait_swapouts(self):
        """Before a compute-stream write: blocks freed by a swap-out may have been handed out again."""
        if self.swapout_ev is not None:
            self.stream.wait_event(self.swapout_ev)
            self.swapout_ev = None

    def _wait_swapin(self, rid: int):
        ev = self.swapins.pop(rid, None)
        if ev is not None:
            self.stream.wait_event(ev)

    def _side_after_compute(self):
        """The swap stream starts after everything queued on the compute stream so far."""
        import torch
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self.side.wait_event(ev)

    def _write_rows(self, rid: int, positions: np.ndarray):
        """K/V rows of `positions` of rid into their slots through its table."""
        if len(positions) == 0:
            return
        self._wait_swapouts()
        tbl = np.asarray(self.mgr.block_table(rid), dtype=np.int64)
        slots = (tbl[positions // self.B] * self.B + positions % self.B).astype(np.int32)
        k, v = self.source(np.full(len(positions), rid, dtype=np.int64), positions)
        self.kvb.append_scatter(k, v, self.k, self.v, self._to_dev(slots), status=self.status,
                                stream=self.stream)

    def _flush_copies(self):
        if self.pending_cow or self.pending_tokens:
            self._wait_swapouts()
        for r, _, _ in self.pending_tokens:  # a token lands in its request's (maybe just swapped-in) last block
            self._wait_swapin(r)
        if self.pending_cow:
            self.kvb.cow_copy(self.k, self.v, self._to_dev(np.asarray(self.pending_cow, dtype=np.int32)),
                              status=self.status, stream=self.stream)
            self.pending_cow = []
        if self.pending_tokens:
            r, slots, pos = (np.asarray(x, dtype=np.int64) for x in zip(*self.pending_tokens))
            k, v = self.source(r, pos)
            self.kvb.append_scatter(k, v, self.k, self.v, self._to_dev(slots.astype(np.int32)),
                                    status=self.status, stream=self.stream)
            self.pending_tokens = []

    def _flush_attention(self):
        self._flush_copies()
        if not self.pending:
            return
        import torch
        kvb = self.kvb
        rids = list(self.pending)
        self._wait_swapouts()  # the fused append writes
        for r in rids:
            self._wait_swapin(r)
        tables, lens = self.mgr.dense_tables(rids, max(self.pending.values()) // self.B + 1)
        t, ln = self._to_dev(tables), self._to_dev(lens)
        q = self.queries(rids)
        out = torch.empty((self.L, len(rids), self.nh, self.D), dtype=self.out_dtype, device=self.dev)
        kn = vn = None
        if self.fused:
            r = np.asarray(rids, dtype=np.int64)
            kn, vn = self.source(r, np.asarray([self.pending[x] for x in rids], dtype=np.int64))
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        a = kvb.attention_args(q[0], self.k[0], self.v[0], t, ln, out[0], self.nh, self.kvh, status=self.status,
                               k_new=None if kn is None else kn[0], v_new=None if vn is None else vn[0])
        need = kvb.workspace_bytes(a)  # the same for every layer of the batch
        if need > self.workspace.numel():
            self.workspace = torch.zeros(need + need // 4, dtype=torch.uint8, device=self.dev)
        if need:
            a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
            a.flags |= kvb.KVP_ATTN_WORKSPACE_CLEAN  # counters return to zero after every launch
        fn = kvb.lib().kvp_paged_attention
        # per-layer byte strides (each layer's slice is contiguous, which attention_args checked for layer 0)
        layer_k, layer_q, layer_o = (t.stride(0) * t.element_size() for t in (self.k, q, out))
        layer_n = 0 if kn is None else kn.stride(0) * kn.element_size()
        if kn is not None and vn.stride(0) != kn.stride(0):
            raise ValueError("k_new and v_new rows must share a layout")
        ev0.record(self.stream)
        for layer in range(self.L):
            if layer:  # the same arguments, moved to the next layer's buffers
                a.q += layer_q
                a.k_cache += layer_k
                a.v_cache += layer_k
                a.out += layer_o
                if kn is not None:
                    a.k_new += layer_n
                    a.v_new += layer_n
                if self.early:  # the previous kernel is layer-1's: it writes neither these pools nor the
                    a.flags |= kvb.KVP_ATTN_EARLY_LOAD  # tables and lengths
            kvb._launch(self.dev, fn, a, self.stream)
        ev1.record(self.stream)
        ctx_tokens = int(lens.sum())
        self.events.append((ev0, ev1, ctx_tokens * self.L * self.kvh * self.D * 2 * self.k.element_size()))
        self.n.attention_launches += self.L
        self.n.attention_rows += len(rids)
        self.pending = {}
        if self.on_attention is not None:
            self.on_attention(rids, q, out, tables, lens)

    # ------------------------------------------------------------------ decisions
    def apply(self, row):
        """Re-makes one recorded decision and issues its device traffic (on the shard's stream, which is also
        the current stream for every allocation the traffic makes)."""
        import torch
        with torch.cuda.stream(self.stream):
            self._apply(row)

    def _appends(self, rows):
        """A run of consecutive append decisions: one batched manager call (which stops at the first failure,
        changing nothing for it, as the recorded run does)."""
        rids = [int(x) for x in rows[:, 1]]
        want = rows[:, 5]
        fail = np.nonzero(want == 0)[0]
        upto = int(fail[0]) + 1 if len(fail) else len(rids)
        done, slots, pairs = self.mgr.append_batch(rids[:upto])
        _expect(done, upto - (1 if len(fail) else 0), rows[min(done, len(rows) - 1)], "append_token run")
        if upto < len(rids):
            raise TraceMismatch("append decisions recorded after a failed append in the same run")
        if not done:
            return
        if len(pairs):
            self.pending_cow.extend(map(tuple, pairs.tolist()))
            self.n.cow_copies += len(pairs)
        for i in range(done):
            r = rids[i]
            pos = self.tokens[r]
            self.tokens[r] = pos + 1
            if not self.fused:
                self.pending_tokens.append((r, int(slots[i]), pos))
            self.pending[r] = pos
        self.n.tokens_generated += done

    def _apply(self, row):
        op, res, flag = int(row[0]), int(row[5]), int(row[6])
        mgr = self.mgr
        if op == TRACE_APPEND:
            self._appends(np.asarray(row).reshape(1, -1))
            return
        self._flush_copies()
        if op == TRACE_STEP:
            self._flush_attention()
            _check_step(mgr, row)
            self.n.steps += 1
        elif op in (TRACE_ADMIT_PREFIX, TRACE_ADMIT_CACHED):
            r, prompt = int(row[1]), int(row[4])
            if op == TRACE_ADMIT_PREFIX and int(row[2]) != NO_REQUEST:
                self._wait_swapin(int(row[2]))  # its blocks are about to be shared
            shared = _admission_shared_tokens(mgr, row)
            fn = mgr.admit_with_prefix if op == TRACE_ADMIT_PREFIX else mgr.admit_with_cached_prefix
            _expect(int(fn(r, int(row[2]), int(row[3]), prompt)), res, row, "admission")
            if not res:
                return
            self.tokens[r] = prompt
            if flag == 1:  # swap-in: fresh blocks, no sharing
                import torch
                slots, tokens = self.swapped.pop(r)
                _expect(prompt, tokens, row, "swapped-in tokens")
                blocks = mgr.block_table(r)
                self._side_after_compute()  # the fresh blocks' previous readers are queued there
                self.kvb.swap_in(self.k, self.v, blocks, slots, self.pool, stream=self.side)
                ev = torch.cuda.Event()
                ev.record(self.side)
                self.swapins[r] = ev
                self.free_slots.extend(reversed(slots))
                self.n.swap_in_blocks += len(blocks)
            else:
                self._write_rows(r, np.arange(shared, prompt, dtype=np.int64))
                self.n.prefill_tokens += prompt - shared
                self.n.cache_hits += int(op == TRACE_ADMIT_CACHED and shared > 0)
        elif op == TRACE_CACHE_PREFIX:
            if int(row[2]) in self.pending:  # the owner's newest row must be in place before blocks are shared
                self._flush_attention()
            self._wait_swapin(int(row[2]))
            _expect(int(mgr.cache_prefix(int(row[1]), int(row[2]), int(row[3]))), res, row, "cache_prefix")
        elif op == TRACE_FORK:
            if int(row[2]) in self.pending:
                self._flush_attention()
            self._wait_swapin(int(row[2]))
            _expect(int(mgr.fork(int(row[1]), int(row[2]))), res, row, "fork")
            if res:
                self.tokens[int(row[1])] = self.tokens[int(row[2])]
        elif op == TRACE_FREE:
            r = int(row[1])
            _expect(self.tokens.get(r), int(row[2]), row, "tokens at free")
            if r in self.pending:  # it generated this step: attend before its blocks can be reused
                self._flush_attention()
            if flag == FREE_SWAPPED:
                import torch
                blocks = mgr.block_table(r)
                if len(self.free_slots) < len(blocks):
                    raise RuntimeError("host swap pool exhausted")
                slots = [self.free_slots.pop() for _ in blocks]
                self._side_after_compute()  # its rows, and a swap-in of it still in flight, come first
                self.kvb.swap_out(self.k, self.v, blocks, slots, self.pool, stream=self.side)
                ev = torch.cuda.Event()
                ev.record(self.side)
                self.swapout_ev = ev  # the swap stream is serial: this covers every earlier swap
                self.swapins.pop(r, None)
                self.swapped[r] = (slots, int(row[2]))
                self.n.swap_out_blocks += len(blocks)
            else:
                self._wait_swapin(r)  # its blocks may be handed out again
            mgr.free(r)
            del self.tokens[r]
        elif op == TRACE_CLEAR_CACHE:
            mgr.clear_cache()
        else:
            raise ValueError(f"unknown trace op {op}")

    def run(self, trace, *, on_step: Optional[Callable] = None) -> DecisionCounters:
        """Replays a decision stream; `on_step(step_index)` runs after each end-of-step marker.  Runs of
        consecutive appends go to the manager as one batch."""
        import torch
        t = np.asarray(trace)
        op = t[:, 0]
        # boundaries of runs of consecutive APPEND rows
        is_app = op == TRACE_APPEND
        with torch.cuda.stream(self.stream):
            i, n = 0, len(t)
            while i < n:
                if is_app[i]:
                    j = i
                    while j < n and is_app[j] and (j == i or t[j - 1, 5] == 1):
                        j += 1
                    self._appends(t[i:j])
                    i = j
                    continue
                self._apply(t[i])
                if on_step is not None and op[i] == TRACE_STEP:
                    on_step(self.n.steps - 1)
                i += 1
            self._flush_attention()
        return self.n

    def attention_time(self):
        """(seconds, algorithmic bytes) summed over the attention batches so far (synchronises)."""
        import torch
        torch.cuda.synchronize(self.dev)
        secs = sum(a.elapsed_time(b) for a, b, _ in self.events) / 1e3
        return secs, sum(x for _, _, x in self.events)

    def status_word(self) -> int:
        import torch
        torch.cuda.synchronize(self.dev)
        return int(self.status.item())


class SyntheticContent:
    """Deterministic synthetic K/V and queries for a workload's requests (the reference's Request fields):
    position p of request r holds the rows of its *origin* -- the fork leader's position while p is below the
    leader's prompt length, the prefix group's position while p is below the group's prefix length, else r's
    own -- so rows shared through prefix blocks, forks, the prefix cache or recomputation agree with a fresh
    computation.  Values are uniform in [-1, 1) from an integer hash of (origin, position, element), computed
    on the device."""

    P = 2147483647  # 2^31 - 1

    def __init__(self, requests, *, layers: int, kv_heads: int, head_dim: int, num_heads: int, dtype=None,
                 device="cuda", seed: int = 1):
        import torch
        self.L, self.kvh, self.D, self.nh = layers, kv_heads, head_dim, num_heads
        self.dtype = dtype or torch.bfloat16
        self.dev = torch.device(device)
        req = np.asarray(requests, dtype=np.int64).reshape(-1, 8)
        self.index = {int(r[0]): i for i, r in enumerate(req)}
        self.prompt, self.group, self.plen = req[:, 2], req[:, 4], req[:, 5]
        self.leader = np.asarray([self.index.get(int(f), -1) if f != NO_REQUEST else -1 for f in req[:, 6]])
        self.ids = req[:, 0]
        self.seed = seed
        self.gen = torch.Generator(device=self.dev).manual_seed(seed)
        e = layers * kv_heads * head_dim
        self.elem = torch.arange(2 * e, dtype=torch.int64, device=self.dev)

    def origins(self, rids, positions) -> np.ndarray:
        """Origin key of each row (a request id, or 2^40 + group for prefix-group positions)."""
        rids = np.asarray(rids, dtype=np.int64)
        positions = np.asarray(positions, dtype=np.int64)
        ix = np.fromiter((self.index[int(r)] for r in rids), dtype=np.int64, count=len(rids))
        lead = self.leader[ix]
        forked = (lead >= 0) & (positions < self.prompt[np.maximum(lead, 0)])
        ix = np.where(forked, lead, ix)  # below the fork point a sample is its leader
        out = self.ids[ix].copy()
        grp = (self.group[ix] >= 0) & (positions < self.plen[ix])
        out[grp] = (1 << 40) + self.group[ix][grp]
        return out

    def _hash(self, x):
        for _ in range(3):
            x = (x * 48271) % self.P
        return x

    def __call__(self, rids, positions):
        import torch
        positions = np.asarray(positions, dtype=np.int64)
        keys = (self.origins(rids, positions) % self.P) * 1000003 + positions + self.seed * 7919
        row = self._hash(torch.from_numpy(keys % self.P).pin_memory().to(self.dev, non_blocking=True))
        x = self._hash((row[:, None] * 65599 + self.elem[None, :] + 1) % self.P)
        vals = ((x >> 7) % 2048).to(torch.float32) / 1024.0 - 1.0
        n = len(positions)
        kv = vals.view(n, 2, self.L, self.kvh, self.D).permute(1, 2, 0, 3, 4).to(self.dtype).contiguous()
        return kv[0], kv[1]

    def queries(self, rids):
        import torch
        return torch.randn((self.L, len(rids), self.nh, self.D), generator=self.gen, device=self.dev).to(self.dtype)
