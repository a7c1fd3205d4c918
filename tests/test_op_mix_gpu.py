"""The KV-management op mix (bench.OpMix, the workload of `bench.py --op mix`) at one eighth of its stated scale:
64 requests x 8 samples on a 2048-token shared prefix, Llama-3-8B-shaped blocks (32 layers, 8 kv heads x 128,
bf16, block 16), copy-on-write on the first append, a swap round every 16 steps (10% of the allocated blocks out
to pinned host memory, back in after one step with fresh ids).

Every KVManager call the mix makes is replayed on the reference's own KVManager (src/kv_manager.cpp:155-251)
and must return the same result -- slots and copy-on-write pairs included; tables, refcounts and statistics are
compared after every swap round and at the end; and every live sample's context, gathered from the device through
its table, must equal the content model bit for bit (python/paged_model.py:54-55, 92-95, 113-117 semantics).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_op_mix_eighth_scale_in_lockstep_with_the_reference(kvb, ora, cuda):
    import torch
    import bench
    if not ora.have_ref():
        pytest.skip("the reference KVManager library (oracle/_ref) is not built")
    cfg = dict(bench.CONFIGS["llama3-8b"])
    steps = 48
    mix = bench.OpMix(kvb, cfg, torch.device("cuda:0"), requests=64, steps=steps, seed=3)
    ref = ora.RefKVManager(mix.nb, mix.B)
    calls = []

    def shadow(name, args, res):
        r = getattr(ref, name)(*args)
        calls.append(name)
        if name == "append_batch":
            assert res[0] == r[0]
            np.testing.assert_array_equal(res[1], r[1])
            np.testing.assert_array_equal(res[2], r[2])
        else:
            assert res == r, (name, args, res, r)

    mix.on_op = shadow

    def compare_state():
        assert mix.mgr.stats() == ref.stats()
        for ident in mix.live:
            assert mix.mgr.block_table(mix.mid[ident]) == ref.block_table(mix.mid[ident])
        for b in range(mix.nb):
            assert mix.mgr.refcount(b) == ref.refcount(b), b
        assert mix.mgr.validate() == "" and ref.validate() == ""

    mix.setup()
    compare_state()
    assert mix.check() > 0
    for s in range(steps):
        mix.step()
        if s == 0:
            # every sample but the last of each request copied its request's shared partial block
            assert mix.mgr.stats()["cow_copies"] == 64 * 7
        if (s + 1) % 16 == 0 or s == steps - 1:
            assert mix.settle() == 0
            compare_state()
            mix.check()
    c = mix.counters
    assert c["swap_rounds"] == steps // 16 and c["swap_out_blocks"] > 0 and c["swap_in_blocks"] > 0
    assert c["cow_pairs"] == 64 * 7
    assert calls.count("append_batch") == steps
