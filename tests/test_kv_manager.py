"""Host control plane: the reference's known-answer tests for the KVManager and allocator, run against the
product (and against the reference library itself where it was built here, to show the expectations are
the reference's).  Expectations follow tests/test_kv_manager.cpp:6-95, tests/test_prefix_cow.cpp:6-107,
tests/test_allocator.cpp:8-69 (through the manager) and tests/test_features.cpp:32-127."""
import pytest

NO = -1


def _impls():
    out = ["product"]
    import oracle
    if oracle.have_ref():
        out.append("reference")
    return out


@pytest.fixture(params=_impls())
def make(request, kvb):
    if request.param == "product":
        def f(nb, B):
            m = kvb.KVManager(nb, B)
            m.set_check_each_op(True)
            return m
    else:
        import oracle

        def f(nb, B):
            m = oracle.RefKVManager(nb, B)
            m.set_check_each_op(True)
            return m
    return f


def ceil_div(a, b):
    return (a + b - 1) // b


# ------------------------------------------------------------------ test_kv_manager.cpp
def test_block_counts_at_boundaries(make):
    B = 4
    for tokens in range(0, 3 * B + 2):
        kv = make(16, B)
        assert kv.admit(1, tokens)
        assert len(kv.block_table(1)) == ceil_div(tokens, B)
        assert kv.num_tokens(1) == tokens
        assert kv.free_blocks() == 16 - ceil_div(tokens, B)
        assert kv.validate() == ""


def test_append_allocates_only_at_boundary(make):
    B = 4
    kv = make(8, B)
    assert kv.admit(1, 0)
    for t in range(1, 3 * B + 1):
        before = kv.free_blocks()
        assert kv.append_token(1)
        assert before - kv.free_blocks() == (1 if (t - 1) % B == 0 else 0)
        assert len(kv.block_table(1)) == ceil_div(t, B)


def test_only_last_block_partial(make):
    kv = make(8, 4)
    assert kv.admit(1, 9)
    s = kv.stats()
    assert (s["used_tokens"], s["allocated_slots"], s["internal_waste"]) == (9, 12, 3)


def test_free_returns_everything(make):
    kv = make(10, 4)
    assert kv.admit(1, 7) and kv.admit(2, 12)
    for _ in range(5):
        assert kv.append_token(1)
    kv.free(1)
    kv.free(2)
    assert kv.free_blocks() == 10 and kv.stats()["requests"] == 0 and kv.validate() == ""


def test_admit_fails_cleanly(make):
    kv = make(3, 4)
    assert kv.admit(1, 8)
    assert not kv.can_admit(8)
    assert not kv.admit(2, 8)
    assert not kv.contains(2) and kv.free_blocks() == 1
    assert kv.can_admit(4) and kv.admit(2, 4) and kv.free_blocks() == 0


def test_append_fails_cleanly(make):
    kv = make(2, 4)
    assert kv.admit(1, 8)
    assert not kv.append_token(1)
    assert kv.num_tokens(1) == 8 and kv.free_blocks() == 0
    kv.free(1)
    assert kv.admit(2, 3)
    assert kv.append_token(2) and kv.append_token(2)
    assert kv.validate() == ""


def test_unknown_and_duplicate_requests_raise(make, kvb):
    kv = make(4, 4)
    for f in (lambda: kv.append_token(7), lambda: kv.free(7), lambda: kv.block_table(7)):
        with pytest.raises(RuntimeError):
            f()
    assert kv.admit(1, 4)
    with pytest.raises(RuntimeError):
        kv.admit(1, 4)
    with pytest.raises(ValueError):
        make(4, 0)
    with pytest.raises(ValueError):
        kv.admit(9, -1)


# ------------------------------------------------------------------ test_allocator.cpp through the manager
def test_lowest_ids_first_and_reuse(make):
    kv = make(4, 1)
    for r in range(4):
        assert kv.admit(r, 1)
        assert kv.block_table(r) == [r]
    assert not kv.admit(9, 1)
    kv.free(2)
    assert kv.admit(10, 1) and kv.block_table(10) == [2]  # the released block is reused first


def test_release_order_is_lifo(make):
    kv = make(8, 2)
    assert kv.admit(1, 6)  # blocks 0 1 2
    kv.free(1)             # releases 0, 1, 2 in table order -> 2 is on top
    assert kv.admit(2, 2) and kv.block_table(2) == [2]
    assert kv.admit(3, 2) and kv.block_table(3) == [1]


# ------------------------------------------------------------------ test_prefix_cow.cpp
def test_prefix_shares_only_full_blocks(make):
    B = 16
    kv = make(20, B)
    assert kv.admit(1, 40)
    assert kv.blocks_needed_to_admit(1, 40, 60) == ceil_div(60, B) - 2
    assert kv.admit_with_prefix(2, 1, 40, 60)
    p, c = kv.block_table(1), kv.block_table(2)
    assert c[:2] == p[:2] and c[2] != p[2]
    assert kv.refcount(p[0]) == 2 and kv.refcount(p[2]) == 1
    assert kv.total_blocks() - kv.free_blocks() == 5
    s = kv.stats()
    assert s["blocks_saved"] == 2 and s["logical_blocks"] == 7
    assert kv.validate() == ""


def test_prefix_clamped(make):
    kv = make(20, 4)
    assert kv.admit(1, 10)
    assert kv.admit_with_prefix(2, 1, 100, 6)
    assert kv.block_table(2)[0] == kv.block_table(1)[0]
    assert kv.block_table(2)[1] != kv.block_table(1)[1]


def test_prefix_failure_has_no_side_effects(make):
    kv = make(4, 4)
    assert kv.admit(1, 12)
    assert not kv.admit_with_prefix(2, 1, 12, 24)
    assert not kv.contains(2)
    assert kv.refcount(kv.block_table(1)[0]) == 1 and kv.free_blocks() == 1


def test_cow_on_append_into_shared_partial_block(make):
    kv = make(10, 4)
    assert kv.admit(1, 6) and kv.fork(2, 1)
    shared = kv.block_table(1)[1]
    assert kv.refcount(shared) == 2
    free_before = kv.free_blocks()
    assert kv.append_token(2)
    assert kv.stats()["cow_copies"] == 1
    assert kv.block_table(2)[1] != shared and kv.block_table(1)[1] == shared
    assert kv.refcount(shared) == 1 and kv.free_blocks() == free_before - 1
    assert kv.append_token(2) and kv.append_token(1)
    assert kv.stats()["cow_copies"] == 1 and kv.validate() == ""


def test_no_cow_when_last_block_full(make):
    kv = make(10, 4)
    assert kv.admit(1, 8) and kv.fork(2, 1)
    assert kv.append_token(2)
    assert kv.stats()["cow_copies"] == 0
    assert len(kv.block_table(2)) == 3 and kv.block_table(2)[:2] == kv.block_table(1)[:2]


def test_cow_fails_cleanly(make):
    kv = make(2, 4)
    assert kv.admit(1, 6) and kv.fork(2, 1)
    assert not kv.append_token(2)
    assert kv.stats()["cow_copies"] == 0 and kv.num_tokens(2) == 6
    assert kv.refcount(kv.block_table(1)[1]) == 2 and kv.validate() == ""


def test_freeing_parent_keeps_shared_alive(make):
    kv = make(10, 4)
    assert kv.admit(1, 8) and kv.admit_with_prefix(2, 1, 8, 10)
    b0 = kv.block_table(1)[0]
    kv.free(1)
    assert kv.refcount(b0) == 1 and kv.validate() == ""
    kv.free(2)
    assert kv.free_blocks() == 10


def test_many_children_share_one_copy(make):
    kv = make(64, 8)
    assert kv.admit(0, 32)
    for i in range(1, 11):
        assert kv.admit_with_prefix(i, 0, 32, 40)
    assert kv.total_blocks() - kv.free_blocks() == 14
    assert kv.refcount(kv.block_table(0)[0]) == 11
    assert kv.stats()["blocks_saved"] == 40
    for i in range(11):
        kv.free(i)
    assert kv.free_blocks() == 64


# ------------------------------------------------------------------ test_features.cpp (prefix cache)
def test_cache_prefix_outlives_owner(make):
    kv = make(10, 16)
    assert kv.admit(1, 40) and kv.cache_prefix(7, 1, 40)
    assert kv.cached_prefix_tokens(7) == 32 and not kv.cache_prefix(7, 1, 40)
    kv.free(1)
    assert kv.free_blocks() == 8 and kv.stats()["cached_blocks"] == 2 and kv.evictable_blocks() == 2
    assert kv.blocks_needed_to_admit_cached(7, 32, 50) == 2
    assert kv.admit_with_cached_prefix(2, 7, 32, 50)
    assert kv.free_blocks() == 6 and len(kv.block_table(2)) == 4 and kv.evictable_blocks() == 0
    kv.free(2)
    kv.clear_cache()
    assert kv.free_blocks() == 10 and kv.validate() == ""


def test_cache_reclaimed_on_admission_and_append(make):
    kv = make(4, 16)
    assert kv.admit(1, 32) and kv.cache_prefix(0, 1, 32)
    kv.free(1)
    assert kv.can_admit(64) and kv.admit(2, 64)
    assert not kv.has_cached_prefix(0) and kv.stats()["cache_evictions"] == 1 and kv.free_blocks() == 0
    kv2 = make(3, 16)
    assert kv2.admit(1, 32) and kv2.cache_prefix(0, 1, 32)
    kv2.free(1)
    assert kv2.admit(2, 16) and kv2.free_blocks() == 0
    assert kv2.append_token(2)
    assert kv2.stats()["cache_evictions"] == 1 and len(kv2.block_table(2)) == 2 and kv2.validate() == ""


def test_cache_entry_being_shared_is_kept(make):
    kv = make(3, 16)
    assert kv.admit(1, 32) and kv.cache_prefix(0, 1, 32)
    kv.free(1)
    assert kv.admit_with_cached_prefix(2, 0, 32, 48)
    assert kv.has_cached_prefix(0) and kv.stats()["cache_evictions"] == 0
    small = make(3, 16)
    assert small.admit(1, 32) and small.cache_prefix(0, 1, 32)
    small.free(1)
    assert not small.admit_with_cached_prefix(2, 0, 32, 80)
    assert not small.contains(2) and small.has_cached_prefix(0) and small.refcount(0) == 1
    assert small.free_blocks() == 1 and small.validate() == ""


def test_cache_lru_order(make):
    kv = make(6, 16)
    assert kv.admit(1, 16) and kv.admit(2, 16)
    assert kv.cache_prefix(1, 1, 16) and kv.cache_prefix(2, 2, 16)
    kv.free(1)
    kv.free(2)
    assert kv.admit_with_cached_prefix(3, 1, 16, 16)
    kv.free(3)
    assert kv.admit(4, 64) and kv.stats()["cache_evictions"] == 0
    assert kv.admit(5, 16)
    assert not kv.has_cached_prefix(2) and kv.has_cached_prefix(1) and kv.validate() == ""


def test_too_short_prefix_not_cached(make):
    kv = make(4, 16)
    assert kv.admit(1, 15)
    assert not kv.cache_prefix(1, 1, 15) and not kv.has_cached_prefix(1)


def test_stats_agree_with_recompute(kvb):
    """validate() cross-checks the O(1) statistics against a from-scratch recount
    (kv_manager.cpp:261-300 of the reference); both agree after fork + copy-on-write."""
    kv = kvb.KVManager(16, 4)
    assert kv.admit(1, 9) and kv.fork(2, 1) and kv.append_token(2)
    assert kv.validate() == ""
    s, r = kv.stats(), kv.recompute_stats()
    for f in ("used_tokens", "logical_blocks", "blocks_saved", "internal_waste", "cached_blocks"):
        assert s[f] == r[f]
