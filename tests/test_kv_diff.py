"""Product KVManager vs the reference KVManager on random operation sequences: identical return values,
tables, refcounts and statistics after every operation (the property of tests/test_random.cpp:30-145,
strengthened from a shadow model to the reference itself).  The golden traces recorded from the reference
run everywhere; the live comparison runs where the reference library was built."""
import json
import os

import numpy as np
import pytest

from cases import Lcg

TRACES = os.path.join(os.path.dirname(__file__), "golden", "kv_traces.json")


def _apply(kv, op):
    name = op[0]
    if name == "admit":
        return int(kv.admit(op[1], op[2]))
    if name == "admit_with_prefix":
        return int(kv.admit_with_prefix(op[1], op[2], op[3], op[4]))
    if name == "fork":
        return int(kv.fork(op[1], op[2]))
    if name == "cache_prefix":
        return int(kv.cache_prefix(op[1], op[2], op[3]))
    if name == "admit_with_cached_prefix":
        return int(kv.admit_with_cached_prefix(op[1], op[2], op[3], op[4]))
    if name == "append_token":
        return int(kv.append_token(op[1]))
    if name == "clear_cache":
        kv.clear_cache()
        return None
    if name == "free":
        kv.free(op[1])
        return None
    raise AssertionError(name)


def test_golden_traces_replay_bit_exact(kvb):
    traces = json.load(open(TRACES))
    assert len(traces) >= 100
    n_ops = 0
    for tr in traces:
        kv = kvb.KVManager(tr["total"], tr["B"])
        kv.set_check_each_op(True)
        for op in tr["ops"]:
            got = _apply(kv, op)
            if got is not None:
                assert got == op[-1], (tr["seed"], op)
            n_ops += 1
        fin = tr["final"]
        for r, t in fin["tables"].items():
            assert kv.block_table(int(r)) == t
            assert kv.num_tokens(int(r)) == fin["tokens"][r]
        assert [kv.refcount(b) for b in range(tr["total"])] == fin["refcounts"]
        assert kv.stats() == fin["stats"]
        assert kv.free_blocks() == fin["free_blocks"]
        assert kv.validate() == ""
    assert n_ops > 10000


def _state(kv, live, total):
    return ([kv.block_table(r) for r in live], [kv.num_tokens(r) for r in live],
            [kv.refcount(b) for b in range(total)], kv.stats(), kv.free_blocks(), kv.available_blocks())


@pytest.mark.parametrize("seed", range(1, 41))
def test_live_differential_against_reference(kvb, seed):
    import oracle
    if not oracle.have_ref():
        pytest.skip("reference library not built on this machine")
    rng = Lcg(seed * 7919 + 11)
    B = rng.range(1, 8)
    total = rng.range(4, 48)
    a, b = kvb.KVManager(total, B), oracle.RefKVManager(total, B)
    a.set_check_each_op(True)
    b.set_check_each_op(True)
    live, nid = [], 0
    for step in range(300):
        c = rng.range(0, 99)
        pick = (lambda: live[rng.range(0, len(live) - 1)]) if live else (lambda: None)
        if c < 18:
            p = rng.range(0, 5 * B)
            ra, rb = a.admit(nid, p), b.admit(nid, p)
            if ra:
                live.append(nid)
            nid += 1
        elif c < 32:
            par = pick()
            if par is None:
                continue
            sh, pr = rng.range(0, a.num_tokens(par) + B), rng.range(0, 6 * B)
            ra, rb = a.admit_with_prefix(nid, par, sh, pr), b.admit_with_prefix(nid, par, sh, pr)
            if ra:
                live.append(nid)
            nid += 1
        elif c < 38:
            par = pick()
            if par is None:
                continue
            ra, rb = a.fork(nid, par), b.fork(nid, par)
            live.append(nid)
            nid += 1
        elif c < 44:
            par = pick()
            if par is None:
                continue
            k, t = rng.range(0, 3), rng.range(0, 4 * B)
            ra, rb = a.cache_prefix(k, par, t), b.cache_prefix(k, par, t)
        elif c < 52:
            k, sh, pr = rng.range(0, 3), rng.range(0, 4 * B), rng.range(0, 6 * B)
            assert a.evictable_blocks(k, sh // B) == b.evictable_blocks(k, sh // B)
            assert a.blocks_needed_to_admit_cached(k, sh, pr) == b.blocks_needed_to_admit_cached(k, sh, pr)
            ra, rb = a.admit_with_cached_prefix(nid, k, sh, pr), b.admit_with_cached_prefix(nid, k, sh, pr)
            if ra:
                live.append(nid)
            nid += 1
        elif c < 86:
            r = pick()
            if r is None:
                continue
            ra, rb = a.append_token(r), b.append_token(r)
        else:
            r = pick()
            if r is None:
                continue
            if rng.range(0, 25) == 0:
                a.clear_cache(), b.clear_cache()
                ra = rb = None
            else:
                a.free(r), b.free(r)
                live.remove(r)
                ra = rb = None
        live.sort()
        assert ra == rb, (seed, step)
        assert _state(a, live, total) == _state(b, live, total), (seed, step)
    for r in list(live):
        a.free(r), b.free(r)
    a.clear_cache(), b.clear_cache()
    assert a.free_blocks() == total == b.free_blocks()


def test_append_batch_matches_reference_harness(kvb):
    """The native batched decode bookkeeping (slots + copy-on-write pairs) equals the reference harness's
    per-request logic (python/paged_model.py:105-118) driven through the reference-compatible manager."""
    import oracle
    mk = oracle.RefKVManager if oracle.have_ref() else kvb.KVManager
    rng = np.random.default_rng(5)
    B = 4
    a, b = kvb.KVManager(64, B), mk(64, B)
    for m in (a, b):
        assert m.admit(0, 6) and m.fork(1, 0) and m.fork(2, 0) and m.admit(3, 8) and m.admit_with_prefix(4, 3, 8, 9)
    for _ in range(12):
        rids = [int(x) for x in rng.permutation(5)]
        da, sa, pa = a.append_batch(rids)
        db, sb, pb = b.append_batch(rids)
        assert da == db == 5
        np.testing.assert_array_equal(sa, sb)
        np.testing.assert_array_equal(pa, pb)
    assert a.stats()["cow_copies"] == 2
