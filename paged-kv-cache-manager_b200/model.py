"""A decoder-only HF model (Qwen2 / Llama architecture) running with its KV cache in paged blocks on the GPU.

The device form of the reference's Python harness (python/paged_model.py:14-158 of
prathameshpranjale/paged-kv-cache-manager), with the same request API -- prefill / fork / decode /
decode_batch / free -- and the same block bookkeeping (this library's KVManager).  What moves from torch to
this library's kernels:
  * writing each new token's K/V into its slot  -> kvp_append_scatter for prompts (paged_model.py:54-55), fused
                                                   into kvp_paged_attention for decode steps (paged_model.py:145-146)
  * the copy-on-write copy after a fork          -> kvp_cow_copy         (paged_model.py:92-95, 113-117)
  * attention over the context                   -> kvp_paged_attention  (paged_model.py:56-63, 147-151)
Prefill attention uses the same decode kernel: prompt position p is a one-query sequence of length p + 1
over the request's block table, which is exactly causal attention.  Norms, projections, rotary embedding and
the MLP stay the model's own torch modules.
"""
from __future__ import annotations

import importlib
from typing import List, Optional, Sequence

import torch

_kvb = importlib.import_module(__package__) if __package__ else None


def _lib():
    global _kvb
    if _kvb is None:
        _kvb = importlib.import_module("paged-kv-cache-manager_b200")
    return _kvb


class PagedEngine:
    """Paged-KV inference for one model on one GPU.  K/V pools are [layers][num_blocks][B][kv_heads][head_dim]
    in the model's dtype (fp16 or bf16)."""

    def __init__(self, model, num_blocks: int, block_size: int):
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb  # same for Qwen2 and Llama

        kvb = _lib()
        self._rope = apply_rotary_pos_emb
        self.m = model.eval()
        c = model.config
        self.L = c.num_hidden_layers
        self.nh = c.num_attention_heads
        self.kvh = c.num_key_value_heads
        self.hd = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
        self.B = block_size
        self.num_blocks = num_blocks
        self.dev = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        if self.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("the paged cache holds fp16 or bf16 K/V: load the model in one of them")
        self.kv = kvb.KVManager(num_blocks, block_size)
        self.K = torch.zeros(self.L, num_blocks, block_size, self.kvh, self.hd, dtype=self.dtype, device=self.dev)
        self.V = torch.zeros_like(self.K)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.prefill_tokens_computed = 0
        self.cow_data_copies = 0

    # ------------------------------------------------------------------ internals
    def _slots(self, table: Sequence[int], positions: Sequence[int]) -> torch.Tensor:
        B = self.B
        return torch.tensor([table[p // B] * B + p % B for p in positions], dtype=torch.int32, device=self.dev)

    @torch.no_grad()
    def _layers(self, h, positions: torch.Tensor, slots: Optional[torch.Tensor], tables: torch.Tensor,
                lens: torch.Tensor):
        """Runs every layer for n query tokens (h: [1, n, H]); token i is at positions[i], writes its K/V to
        slots[i] and attends over its context: tables[i] / lens[i].  With slots None (a decode step: every
        token is the newest of its own request) the attention kernel writes the K/V itself (fused append);
        otherwise (several prompt positions of one request read each other's slots) a scatter runs first."""
        kvb = _lib()
        mdl = self.m.model
        n = h.shape[1]
        cos, sin = mdl.rotary_emb(h, positions[None])
        for li, layer in enumerate(mdl.layers):
            a = layer.self_attn
            x = layer.input_layernorm(h)
            q = a.q_proj(x).view(1, n, self.nh, self.hd).transpose(1, 2)
            k = a.k_proj(x).view(1, n, self.kvh, self.hd).transpose(1, 2)
            v = a.v_proj(x).view(1, n, self.kvh, self.hd).transpose(1, 2)
            q, k = self._rope(q, k, cos, sin)
            kn, vn = k[0].transpose(0, 1).contiguous(), v[0].transpose(0, 1).contiguous()
            if slots is not None:
                kvb.append_scatter(kn[None], vn[None], self.K[li:li + 1], self.V[li:li + 1], slots, status=self.status)
                kn = vn = None
            o = kvb.paged_attention(q[0].transpose(0, 1).contiguous(), self.K[li], self.V[li], tables, lens, self.nh,
                                    self.kvh, out_dtype=self.dtype, status=self.status, num_blocks=self.num_blocks,
                                    k_new=kn, v_new=vn)
            h = h + a.o_proj(o.reshape(1, n, self.nh * self.hd))
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        return mdl.norm(h)

    def _table_rows(self, rows: List[List[int]]) -> torch.Tensor:
        mb = max(1, max(len(r) for r in rows))
        t = torch.zeros((len(rows), mb), dtype=torch.int32)
        for i, r in enumerate(rows):
            if r:
                t[i, : len(r)] = torch.tensor(r, dtype=torch.int32)
        return t.to(self.dev)

    @torch.no_grad()
    def _forward(self, rid: int, tokens: Sequence[int], start: int, fused: bool = False):
        """Tokens placed at positions start .. start+n-1 of request rid (the manager already holds them)."""
        n = len(tokens)
        total = start + n
        table = self.kv.block_table(rid)
        assert self.kv.num_tokens(rid) >= total
        positions = list(range(start, total))
        ctx = table[: (total + self.B - 1) // self.B]
        tables = self._table_rows([ctx] * n)
        lens = torch.tensor([p + 1 for p in positions], dtype=torch.int32, device=self.dev)
        h = self.m.model.embed_tokens(torch.tensor(tokens, device=self.dev))[None]
        slots = None if fused else self._slots(table, positions)
        h = self._layers(h, torch.tensor(positions, device=self.dev), slots, tables, lens)
        return self.m.lm_head(h[:, -1])[0]

    def _cow(self, pairs):
        if len(pairs):
            _lib().cow_copy(self.K, self.V, torch.as_tensor(pairs, dtype=torch.int32).reshape(-1, 2).to(self.dev),
                            status=self.status)
            self.cow_data_copies += len(pairs)

    # ------------------------------------------------------------------ request lifecycle
    def prefill(self, rid: int, seq: Sequence[int], parent: Optional[int] = None, shared_tokens: int = 0):
        """Admit rid with context seq; returns the logits of the next token, or None if out of blocks.  Shared
        full prefix blocks of `parent` are reused, not recomputed."""
        if parent is None:
            ok = self.kv.admit(rid, len(seq))
            start = 0
        else:
            start = min(shared_tokens, self.kv.num_tokens(parent), len(seq)) // self.B * self.B
            ok = self.kv.admit_with_prefix(rid, parent, shared_tokens, len(seq))
        if not ok:
            return None
        self.prefill_tokens_computed += len(seq) - start
        return self._forward(rid, list(seq[start:]), start)

    def fork(self, rid: int, parent: int):
        self.kv.fork(rid, parent)

    def decode(self, rid: int, last_token: int):
        """Appends last_token; returns the next-token logits, or None if no block is available."""
        before = self.kv.num_tokens(rid)
        done, _, pairs = self.kv.append_batch([rid])
        if done != 1:
            return None
        self._cow(pairs)  # before the new token is written into the copied block
        return self._forward(rid, [last_token], before, fused=True)

    @torch.no_grad()
    def decode_batch(self, rids: Sequence[int], last_tokens: Sequence[int]):
        """One decode step for several requests in one batched forward: logits [len(rids)][vocab]."""
        before = [self.kv.num_tokens(r) for r in rids]
        done, _, pairs = self.kv.append_batch(list(rids))
        if done != len(rids):
            raise RuntimeError("out of blocks in decode_batch")
        self._cow(pairs)
        tables = self._table_rows([self.kv.block_table(r)[: (p + self.B) // self.B] for r, p in zip(rids, before)])
        lens = torch.tensor([p + 1 for p in before], dtype=torch.int32, device=self.dev)
        h = self.m.model.embed_tokens(torch.tensor(list(last_tokens), device=self.dev))[None]
        h = self._layers(h, torch.tensor(before, device=self.dev), None, tables, lens)  # fused append
        return self.m.lm_head(h[0])

    def free(self, rid: int):
        self.kv.free(rid)

    def kv_bytes_per_token(self) -> int:
        return 2 * self.L * self.kvh * self.hd * self.K.element_size()
