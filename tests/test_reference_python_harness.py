"""The reference's own Python model harness, python/paged_model.py (PagedEngine: block tables from the C++
KVManager through the `kvpage_py` binding, K/V in CPU tensors), run unchanged with this library's `kvpage_py`
module (paged-kv-cache-manager_b200/kvpage_py.py) in place of its pybind11 build, on a random-initialised Qwen2
model (no checkpoint here).  The checks are the reference's own model properties (python/model_check.py):
bit-identical logits whatever the block size and physical placement (:304-330), and fork + divergent decode
with exactly one copy-on-write (:134-158).  Runs where the reference sources are present; skipped elsewhere."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "paged-kv-cache-manager_b200")
REF_MODEL = "/root/reference/python/paged_model.py"

pytestmark = pytest.mark.skipif(not os.path.exists(REF_MODEL), reason="reference sources not present")


@pytest.fixture(scope="module")
def harness(kvb):
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM
    if PKG_DIR not in sys.path:
        sys.path.insert(0, PKG_DIR)  # provides `import kvpage_py`
    spec = importlib.util.spec_from_file_location("reference_paged_model", REF_MODEL)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.kvpage_py.KVManager is kvb.KVManager  # the reference engine runs on this library's KVManager
    cfg = Qwen2Config(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, max_position_embeddings=512, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).eval()
    tokens = np.random.default_rng(3).integers(0, 300, size=80).tolist()
    return mod.PagedEngine, model, tokens


def _run(engine, prompt, follow):
    out = [engine.prefill(1, prompt)]
    for t in follow:
        out.append(engine.decode(1, t))
    return out


def test_reference_engine_layout_invariance_on_this_kvmanager(harness):
    import torch
    Engine, model, tokens = harness
    prompt, follow = tokens[:21], tokens[21:27]
    ref = _run(Engine(model, num_blocks=2, block_size=256), prompt, follow)
    for B in (1, 4, 16):
        e = Engine(model, num_blocks=400, block_size=B)
        junk = list(range(100, 140))
        for r in junk:  # fragment the free list
            assert e.kv.admit(r, B)
        for r in junk[::2] + junk[1::2]:
            e.kv.free(r)
        got = _run(e, prompt, follow)
        assert all(torch.equal(a, b) for a, b in zip(ref, got)), B
        assert e.kv.validate() == ""


def test_reference_engine_fork_copies_on_write_once(harness):
    Engine, model, tokens = harness
    e = Engine(model, num_blocks=32, block_size=4)
    e.prefill(1, tokens[:10])  # 10 tokens: the last block holds 2
    e.fork(2, 1)
    e.decode(2, tokens[10])     # the child's first append copies the shared partial block
    e.decode(1, tokens[11])
    st = e.kv.stats()
    assert st.cow_copies == 1 and st["cow_copies"] == 1 and e.cow_data_copies == 1
    assert e.kv.block_table(1)[:2] == e.kv.block_table(2)[:2] and e.kv.block_table(1)[2] != e.kv.block_table(2)[2]
    assert e.kv.validate() == ""
