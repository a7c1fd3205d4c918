"""Request sharding across ranks (one process per GPU, no collective on the data path), exercised with
world_size-2 gloo process groups on CPU: every request lands on exactly one rank, sharing groups stay
together, per-rank KVManager shards are independent, and timings are combined as the max over ranks."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_assign_balances_and_keeps_groups(kvb):
    import importlib
    sh = importlib.import_module("paged-kv-cache-manager_b200.sharding")
    rng = np.random.default_rng(0)
    lens = np.clip(np.round(rng.lognormal(np.log(4096), 0.35, 2048)), 1, 32768).astype(int).tolist()
    for world in (1, 2, 4, 8):
        r = sh.assign_requests(lens, world)
        assert sorted(set(r)) == list(range(world))
        assert sh.imbalance(lens, r, world) < 1.01
    groups = [i // 8 for i in range(len(lens))]  # 8 samples forked from one leader
    r = sh.assign_requests(lens, 4, groups)
    for g in range(len(lens) // 8):
        assert len({r[i] for i in range(g * 8, g * 8 + 8)}) == 1
    assert sh.assign_requests(lens, 4) == sh.assign_requests(lens, 4)


def _worker(rank, world, port, q):
    import importlib
    import sys
    import torch.distributed as dist
    import torch
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        kvb = importlib.import_module("paged-kv-cache-manager_b200")
        sh = importlib.import_module("paged-kv-cache-manager_b200.sharding")
        rng = np.random.default_rng(42)
        lens = rng.integers(1, 3000, size=97).tolist()
        rank_of = sh.assign_requests(lens, world)
        mine = sh.shard_of(rank_of, rank)
        B = 16
        need = sum((lens[i] + 40 + B - 1) // B for i in mine) + 8
        mgr = kvb.KVManager(need, B)
        for i in mine:
            assert mgr.admit(i, lens[i])
        for _ in range(20):
            done, slots, pairs = mgr.append_batch(mine)
            assert done == len(mine) and len(pairs) == 0
        tokens = sum(mgr.num_tokens(i) for i in mine)
        t = torch.tensor([float(tokens), float(len(mine)), float(tokens)], dtype=torch.float64)
        s = t.clone()
        dist.all_reduce(s[:2], op=dist.ReduceOp.SUM)
        m = t[2:].clone()
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        q.put((rank, int(s[0]), int(s[1]), float(m[0]), mgr.validate()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, "error", repr(e)))


def test_two_rank_shards_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] != "error" for r in res), res
    rng = np.random.default_rng(42)
    lens = rng.integers(1, 3000, size=97)
    total = int(lens.sum()) + 20 * 97
    for rank, tok_sum, n_sum, tok_max, err in res:
        assert tok_sum == total and n_sum == 97 and err == ""
        assert tok_max >= total / 2
