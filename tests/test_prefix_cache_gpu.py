"""Prefix cache on the device: cache_prefix / admit_with_cached_prefix / LRU eviction
(src/kv_manager.cpp:37-151 of the reference) with real K/V bytes.  Block ids change hands under eviction and
the cached rows are shared without a copy, so after every operation each live request's context, gathered
from the pools through its table, must equal its logical history bit for bit (tests/kvharness.py), the
manager decisions must equal the reference's, and attention over the tables must match the fp64 oracle over
the histories.  The scenarios follow the reference's tests/test_features.cpp:32-127, with data."""
import numpy as np
import pytest

from kvharness import Shard

pytestmark = pytest.mark.gpu

L, KVH, D, NH, B = 2, 2, 64, 8, 16


def _shard(kvb, nb, seed):
    return Shard(kvb, L, nb, B, KVH, D, NH, seed)


def test_cached_prefix_outlives_its_owner(kvb, ora, cuda):
    s = _shard(kvb, 10, 1)
    assert s.admit(1, 40)
    s.step([1])
    assert s.cache_prefix(7, 1, 40) and s.mgr.cached_prefix_tokens(7) == 32
    assert not s.cache_prefix(7, 1, 40)
    owner_rows = s.cached[7]
    s.free(1)
    assert s.mgr.free_blocks() == 8 and s.mgr.stats()["cached_blocks"] == 2
    assert s.admit(3, 20)  # another request writes its own rows into free blocks
    s.check()
    ok, nsh = s.admit_cached(2, 7, 32, 50)
    assert ok and nsh == 32 and s.mgr.free_blocks() == 4
    np.testing.assert_array_equal(s.hist[2][0][:, :32], owner_rows[0])  # no copy: the owner's bytes
    s.check()
    for _ in range(3):
        q, out, _, _ = s.step([2, 3])
        s.check()
    s.attention_vs_oracle(ora, [2, 3], q, out)
    s.free(2), s.free(3)
    s.clear_cache()
    assert s.mgr.free_blocks() == 10
    s.check()


def test_eviction_hands_cached_blocks_to_a_new_request(kvb, ora, cuda):
    """cache_is_reclaimed_when_admission_needs_memory with data: the evicted entry's blocks are reused and
    overwritten by the admitted request; nothing reads the old rows."""
    s = _shard(kvb, 4, 2)
    assert s.admit(1, 32)
    cached_blocks = s.mgr.block_table(1)
    assert s.cache_prefix(0, 1, 32)
    s.free(1)
    assert s.admit(2, 64)
    assert not s.mgr.has_cached_prefix(0) and 0 not in s.cached
    assert s.mgr.stats()["cache_evictions"] == 1
    assert set(cached_blocks) <= set(s.mgr.block_table(2))
    s.check()


def test_append_reclaims_the_cache(kvb, ora, cuda):
    """cache_is_reclaimed_when_append_needs_a_block with data, through a fused decode step."""
    s = _shard(kvb, 3, 3)
    assert s.admit(1, 32)
    assert s.cache_prefix(0, 1, 32)
    s.free(1)
    assert s.admit(2, 16)
    q, out, _, _ = s.step([2])  # needs a new block: evicts the entry and writes the token into a freed block
    assert s.mgr.stats()["cache_evictions"] == 1 and len(s.mgr.block_table(2)) == 2
    s.check()
    s.attention_vs_oracle(ora, [2], q, out)


def test_shared_entry_survives_and_partial_block_copies_on_write(kvb, ora, cuda):
    """cache_does_not_evict_the_entry_being_shared with data, then a fork whose partial block is copied."""
    s = _shard(kvb, 5, 4)
    assert s.admit(1, 32)
    assert s.cache_prefix(0, 1, 32)
    s.free(1)
    ok, nsh = s.admit_cached(2, 0, 32, 40)
    assert ok and nsh == 32 and s.mgr.has_cached_prefix(0)
    s.fork(3, 2)
    q, out, _, _ = s.step([3, 2])  # 3 appends first: copies the shared partial block
    assert s.cows == 1
    s.check()
    s.attention_vs_oracle(ora, [3, 2], q, out)
    assert s.mgr.stats()["cache_evictions"] == 0
    # not enough memory: nothing changes, the entry and its bytes stay
    ok, _ = s.admit_cached(4, 0, 32, 100)
    assert not ok and not s.mgr.contains(4) and s.mgr.has_cached_prefix(0)
    s.check()


def test_lru_order_with_data(kvb, ora, cuda):
    s = _shard(kvb, 6, 5)
    assert s.admit(1, 16) and s.admit(2, 16)
    assert s.cache_prefix(1, 1, 16) and s.cache_prefix(2, 2, 16)
    s.free(1), s.free(2)
    ok, _ = s.admit_cached(3, 1, 16, 16)  # touches entry 1
    assert ok
    s.free(3)
    assert s.admit(4, 64)
    assert s.mgr.stats()["cache_evictions"] == 0
    assert s.admit(5, 16)  # evicts the least recently used entry (2)
    assert not s.mgr.has_cached_prefix(2) and s.mgr.has_cached_prefix(1)
    ok, nsh = s.admit_cached(6, 1, 16, 20)  # entry 1's bytes are still the first request's
    assert not ok or nsh == 16
    s.check()


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "scatter"])
def test_random_trace_with_cache_swap_and_forks(kvb, ora, cuda, fused):
    """300 random operations on a 48-block pool (admissions with and without a cached or parent prefix,
    prefix caching, forks, decode steps, frees, swaps out and back in, cache clears): after every operation
    the device contexts equal the logical histories and the manager equals the reference."""
    import torch
    s = _shard(kvb, 48, 11 + fused)
    rng = np.random.default_rng(7)
    pool = torch.empty(kvb.host_slot_bytes(L, B, KVH, D) * 64, dtype=torch.uint8).pin_memory()
    side = torch.cuda.Stream()
    swapped = {}
    next_id, next_slot, steps, evictions = 0, 0, 0, 0
    for op in range(300):
        live = sorted(s.hist)
        kind = rng.choice(["admit", "cached", "prefix", "cache", "fork", "step", "free", "swap", "unswap", "clear"],
                          p=[.1, .1, .06, .08, .06, .35, .1, .06, .07, .02])
        if kind == "admit":
            s.admit(next_id, int(rng.integers(1, 70)))
            next_id += 1
        elif kind == "cached" and s.cached:
            key = int(rng.choice(sorted(s.cached)))
            s.admit_cached(next_id, key, int(rng.integers(0, 80)), int(rng.integers(1, 90)))
            next_id += 1
        elif kind == "prefix" and live:
            par = int(rng.choice(live))
            s.admit_prefix(next_id, par, int(rng.integers(0, 80)), int(rng.integers(1, 90)))
            next_id += 1
        elif kind == "cache" and live:
            own = int(rng.choice(live))
            s.cache_prefix(int(rng.integers(0, 6)), own, int(rng.integers(1, 80)))
        elif kind == "fork" and live:
            s.fork(next_id, int(rng.choice(live)))
            next_id += 1
        elif kind == "step" and live:
            if s.mgr.available_blocks() == 0:  # the pool is exhausted: preempt a request first
                s.free(int(rng.choice(live)))
                live = sorted(s.hist)
            # each append takes at most one block (a new one or a copy)
            k = min(int(rng.integers(1, len(live) + 1)), s.mgr.available_blocks())
            rids = [int(r) for r in rng.permutation(live)[:k]]
            if rids:
                q, out, _, _ = s.step(rids, fused=fused)
                steps += 1
                if steps % 10 == 0:
                    s.check()
                    s.attention_vs_oracle(ora, rids, q, out)
        elif kind == "free" and live:
            s.free(int(rng.choice(live)))
        elif kind == "swap" and live and next_slot + 8 <= 64:
            r = int(rng.choice(live))
            if len(s.mgr.block_table(r)) <= 8:
                swapped[r] = (s.swap_out(r, pool, next_slot, side), next_slot)
                next_slot += 8
        elif kind == "unswap" and swapped:
            r = sorted(swapped)[0]
            saved, slot0 = swapped[r]
            if s.swap_in(r, saved, pool, slot0, side):
                del swapped[r]
        elif kind == "clear":
            evictions += s.mgr.stats()["cache_evictions"]  # clear_cache resets the counter
            s.clear_cache()
        s.check()
    evictions += s.mgr.stats()["cache_evictions"]
    assert steps > 60 and evictions > 0 and s.cows > 0  # the trace did reach eviction and copy-on-write
