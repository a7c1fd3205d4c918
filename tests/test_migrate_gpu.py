"""Cross-shard request migration (kvp_migrate_blocks + migrate_request): a request's blocks are copied into
another shard's pools -- a second pool on the same GPU, or a peer GPU's pool read over NVLink -- under fresh
block ids, then freed at the source.  The migrated request's context, gathered through its new table, equals
its history bit for bit; both shards keep the reference's manager decisions; attention on the destination
matches the fp64 oracle (tests/kvharness.py)."""
import numpy as np
import pytest

from kvharness import Shard, migrate

pytestmark = pytest.mark.gpu

L, KVH, D, NH, B = 2, 8, 128, 32, 16


def _trace(kvb, ora, a, b, ops, seed):
    rng = np.random.default_rng(seed)
    shards = [a, b]
    next_id = 0
    moved = 0
    for op in range(ops):
        s = shards[int(rng.integers(2))]
        other = shards[1] if s is shards[0] else shards[0]
        live = sorted(s.hist)
        kind = rng.choice(["admit", "prefix", "fork", "step", "free", "migrate", "migrate"])
        if kind == "admit":
            s.admit(next_id, int(rng.integers(1, 300)))
            next_id += 1
        elif kind == "prefix" and live:
            s.admit_prefix(next_id, int(rng.choice(live)), int(rng.integers(0, 200)), int(rng.integers(1, 300)))
            next_id += 1
        elif kind == "fork" and live:
            s.fork(next_id, int(rng.choice(live)))
            next_id += 1
        elif kind == "step" and live:
            rids = [int(r) for r in rng.permutation(live)[: int(rng.integers(1, len(live) + 1))]]
            if len(rids) <= s.mgr.available_blocks():
                q, out, _, _ = s.step(rids)
                if op % 5 == 0:
                    s.check()
                    s.attention_vs_oracle(ora, rids, q, out)
        elif kind == "free" and live:
            s.free(int(rng.choice(live)))
        elif kind == "migrate" and live:
            r = int(rng.choice(live))
            if migrate(kvb, s, other, r, next_id):
                moved += 1
                rids = [next_id]
                next_id += 1
                q, out, _, _ = other.step(rids)  # the migrated request keeps decoding on its new shard
                other.check()
                other.attention_vs_oracle(ora, rids, q, out)
        a.check()
        b.check()
    return moved


def test_migrate_between_pools_on_one_gpu(kvb, ora, cuda):
    a = Shard(kvb, L, 96, B, KVH, D, NH, seed=1)
    b = Shard(kvb, L, 64, B, KVH, D, NH, seed=2)
    assert _trace(kvb, ora, a, b, 120, seed=3) > 10


def test_migrate_between_gpus_over_nvlink(kvb, ora, cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    a = Shard(kvb, L, 96, B, KVH, D, NH, seed=4, device="cuda:0")
    b = Shard(kvb, L, 64, B, KVH, D, NH, seed=5, device="cuda:1")
    assert _trace(kvb, ora, a, b, 120, seed=6) > 10


def test_migrate_rejects_bad_launch(kvb, cuda):
    """The copy must run on the destination pools' device; bad block ids are skipped and flagged."""
    import torch
    a = torch.zeros((1, 4, B, KVH, D), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros_like(a)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    pairs = torch.tensor([[0, 1], [3, 9], [-1, 2]], dtype=torch.int32, device="cuda")
    a[:, 0] = 1.0
    kvb.migrate_blocks(a, a, b, b, pairs, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & kvb.KVP_STATUS_BAD_BLOCK
    assert torch.equal(b[:, 1], a[:, 0]) and int(b[:, 2].abs().sum()) == 0
    with pytest.raises(ValueError):
        kvb.migrate_blocks(a, a, b[:, :, :8], b[:, :, :8], pairs)
