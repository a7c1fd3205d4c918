"""End-to-end: a decoder-only model (Qwen2 architecture, random weights -- no checkpoint is needed) running
with its KV cache in paged blocks on the GPU through this library (paged-kv-cache-manager_b200/model.py),
checked the way the reference's python/model_check.py checks its CPU harness:
  * layout invariance: block size and physical placement do not change a single bit of the logits
    (model_check.py:304-330);
  * copy-on-write: a fork at a partial block and divergent continuations give exactly what independent
    requests give (model_check.py:134-158);
  * prefix sharing and batched decode match unshared / one-at-a-time decoding (model_check.py:105-131, 247-289);
  * the paged engine tracks the stock HF contiguous-cache model up to bf16 noise (model_check.py:68-102).
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(kvb, cuda):
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=1000, hidden_size=256, intermediate_size=704, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=2048,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    mod = importlib.import_module("paged-kv-cache-manager_b200.model")
    base = np.random.default_rng(1).integers(0, 1000, size=160).tolist()
    return model, mod.PagedEngine, base


def _scatter_pool(eng, n, seed):
    """Fragments the free list (allocate n one-block requests, free them in shuffled order)."""
    rids = list(range(100000, 100000 + n))
    for r in rids:
        assert eng.kv.admit(r, 1)
    np.random.default_rng(seed).shuffle(rids)
    for r in rids:
        eng.kv.free(r)


def _greedy(eng, rid, prompt, n_new, forced=None, first=None):
    """Prefill + greedy decode (or along `forced` tokens); returns (logits list, tokens)."""
    lg = eng.prefill(rid, prompt)
    logits = [lg]
    toks = [int(lg.argmax()) if first is None else first]
    for step in range(n_new - 1):
        nxt = toks[-1] if forced is None else forced[step]
        lg = eng.decode(rid, nxt)
        logits.append(lg)
        toks.append(int(lg.argmax()))
    return logits, toks


def test_layout_invariance_bit_exact(setup):
    """Block size 256 (one block per request) against B = 1, 3, 16 on fragmented pools with interleaved
    decoding of three requests: torch.equal on every logit."""
    import torch
    model, Engine, base = setup
    prompts = {1: base[:37], 2: base[:64], 3: base[20:75]}
    n_new = 10
    ref = {}
    for r, p in prompts.items():
        ref[r] = _greedy(Engine(model, num_blocks=2, block_size=256), 1, p, n_new)
    for B in (1, 3, 16):
        eng = Engine(model, num_blocks=400 if B == 1 else 200, block_size=B)
        _scatter_pool(eng, 120 if B == 1 else 60, seed=B)
        got = {r: [eng.prefill(r, prompts[r])] for r in prompts}
        for step in range(n_new - 1):
            for r in prompts:
                got[r].append(eng.decode(r, ref[r][1][step]))
        for r in prompts:
            for a, b in zip(ref[r][0], got[r]):
                assert torch.equal(a, b), (B, r)
        tables = [eng.kv.block_table(r) for r in prompts]
        assert any(t != sorted(t) for t in tables)  # the blocks really are scattered
        assert eng.kv.validate() == "" and int(eng.status.item()) == 0


def test_fork_copy_on_write_bit_exact(setup):
    """Fork at a partial block (37 tokens, B = 16); the child decodes first and copies the shared partial
    block; parent and child then follow different tokens.  Each equals an independent request bit for bit."""
    import torch
    model, Engine, base = setup
    prompt = base[:37]
    eng = Engine(model, num_blocks=32, block_size=16)
    lg = eng.prefill(1, prompt)
    top2 = [int(t) for t in lg.float().topk(2).indices]
    eng.fork(2, 1)
    assert eng.kv.refcount(eng.kv.block_table(1)[-1]) == 2
    p_log, c_log = [lg], [lg]
    p_toks, c_toks = [top2[0]], [top2[1]]
    for _ in range(12):
        lc = eng.decode(2, c_toks[-1]); c_log.append(lc); c_toks.append(int(lc.argmax()))  # child first: COW
        lp = eng.decode(1, p_toks[-1]); p_log.append(lp); p_toks.append(int(lp.argmax()))
    assert eng.kv.stats()["cow_copies"] == 1 and eng.cow_data_copies == 1
    for toks, logs in ((p_toks, p_log), (c_toks, c_log)):
        ind = Engine(model, num_blocks=32, block_size=16)
        il, _ = _greedy(ind, 7, prompt, len(toks), forced=toks, first=toks[0])
        for a, b in zip(il, logs):
            assert torch.equal(a, b)
    eng.free(1)
    eng.free(2)
    assert eng.kv.free_blocks() == 32 and eng.kv.validate() == ""


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def test_prefix_sharing_matches_unshared(setup):
    """A child admitted with 2 shared full prefix blocks (prefill skips them) decodes like an unshared one."""
    model, Engine, base = setup
    parent, child = base[:40], base[:32] + base[60:80]
    eng = Engine(model, num_blocks=64, block_size=16)
    eng.prefill(1, parent)
    lg = eng.prefill(2, child, parent=1, shared_tokens=32)
    assert eng.kv.block_table(1)[:2] == eng.kv.block_table(2)[:2] and eng.kv.stats()["blocks_saved"] == 2
    assert eng.prefill_tokens_computed == len(parent) + len(child) - 32
    got = [lg]
    toks = [int(lg.argmax())]
    for _ in range(9):
        got.append(eng.decode(2, toks[-1]))
        toks.append(int(got[-1].argmax()))
    ind = Engine(model, num_blocks=64, block_size=16)
    ref, _ = _greedy(ind, 1, child, 10, forced=toks, first=toks[0])
    assert max(_rel(a, b) for a, b in zip(got, ref)) < 0.05


def test_batched_decode_matches_one_at_a_time(setup):
    """Six requests (mixed lengths, a shared-prefix child, a fork that copies on write) in one batched forward
    per step, against decoding each request alone."""
    model, Engine, base = setup
    prompts = {1: base[:21], 2: base[:48], 3: base[:33], 4: base[5:70], 5: base[:32] + base[90:100]}

    def start(eng):
        first = {}
        for r in (1, 2, 3, 4):
            first[r] = int(eng.prefill(r, prompts[r]).argmax())
        first[5] = int(eng.prefill(5, prompts[5], parent=2, shared_tokens=32).argmax())
        eng.fork(6, 3)
        first[6] = first[3]
        return first

    a = Engine(model, num_blocks=96, block_size=16)
    b = Engine(model, num_blocks=96, block_size=16)
    ta, tb = start(a), start(b)
    rids = [1, 2, 3, 4, 5, 6]
    last = [ta[r] for r in rids]
    worst = 0.0
    for _ in range(8):
        batched = a.decode_batch(rids, last)
        single = [b.decode(r, t) for r, t in zip(rids, last)]
        worst = max(worst, max(_rel(x, y) for x, y in zip(batched, single)))
        last = [int(x.argmax()) for x in batched]
    assert worst < 0.05
    assert a.kv.stats()["cow_copies"] == 1 and a.cow_data_copies == 1
    assert a.kv.stats() == b.kv.stats() and a.kv.validate() == ""


def test_tracks_hf_contiguous_cache(setup):
    """Teacher-forced along the stock HF model's greedy tokens (contiguous cache, same bf16 weights): the
    logits agree up to bf16 rounding noise."""
    import torch
    model, Engine, base = setup
    prompt = base[:45]
    with torch.no_grad():
        out = model(torch.tensor([prompt], device="cuda"), use_cache=True)
        pkv, hf = out.past_key_values, [out.logits[0, -1]]
        toks = [int(hf[0].argmax())]
        for _ in range(11):
            out = model(torch.tensor([[toks[-1]]], device="cuda"), past_key_values=pkv, use_cache=True)
            hf.append(out.logits[0, -1])
            toks.append(int(hf[-1].argmax()))
    eng = Engine(model, num_blocks=16, block_size=16)
    got, _ = _greedy(eng, 1, prompt, 12, forced=toks, first=toks[0])
    cos = min(float(torch.nn.functional.cosine_similarity(a.float(), b.float(), dim=0)) for a, b in zip(got, hf))
    agree = sum(int(a.argmax()) == int(b.argmax()) for a, b in zip(got, hf)) / len(hf)
    assert cos > 0.99 and agree >= 0.75, (cos, agree)
