"""ORACLE -- test infrastructure, not product code.

CPU checkers for the paged KV-cache data plane.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg (and its reference arm) load this package; the product never does.

  * c_oracle(): oracle/kvp_oracle.c, a plain-C restatement of the reference's attention
    (src/paged_attention.cpp:25-114 of prathameshpranjale/paged-kv-cache-manager).
  * ref(): oracle/_ref/libkvpage_ref.so, the reference's own C++ sources compiled here (oracle/Makefile)
    with a C shim (ref_shim.cpp): the real KVManager and the real attention functions.
  * ref_gpu_attention(): oracle/_ref/libref_gpu_attention.so, the reference's own GPU kernel
    (cuda/paged_attention.cu) compiled here for sm_100a -- the implementation the drop-in replaces.
  * RefKVManager: the reference KVManager with the same Python interface as the product's KVManager.
  * DataPlane: a numpy model of the bytes the reference's Python harness moves
    (python/paged_model.py:54-55 scatter, :92-95 / :113-117 copy-on-write) plus swap as a host copy.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
C_LIB = os.path.join(HERE, "_build", "libkvp_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libkvpage_ref.so")
REF_GPU_LIB = os.path.join(HERE, "_ref", "libref_gpu_attention.so")

_pf, _pi32 = C.POINTER(C.c_float), C.POINTER(C.c_int32)
_ATTN = [C.c_int] * 6 + [_pf, _pf, _pf, _pi32, _pi32, _pf]


def build(reference: str = "/root/reference") -> None:
    """Builds the C oracle, and the reference library when the reference sources are present."""
    subprocess.run(["make", "-s", "-C", HERE, "all", f"REFERENCE={reference}"], check=True)


_c = None
_r = None


def c_oracle() -> C.CDLL:
    global _c
    if _c is None:
        if not os.path.exists(C_LIB):
            subprocess.run(["make", "-s", "-C", HERE, "c"], check=True)
        L = C.CDLL(C_LIB)
        L.ora_reference_attention.argtypes = _ATTN
        L.ora_reference_attention.restype = C.c_int
        L.ora_paged_attention_cpu.argtypes = _ATTN + [C.c_int]
        L.ora_paged_attention_cpu.restype = C.c_int
        L.ora_paged_attention_cpu_mt.argtypes = _ATTN + [C.c_int, C.c_int]
        L.ora_paged_attention_cpu_mt.restype = C.c_int
        L.ora_f32_to_bf16.argtypes = [_pf, C.POINTER(C.c_uint16), C.c_size_t]
        L.ora_bf16_to_f32.argtypes = [C.POINTER(C.c_uint16), _pf, C.c_size_t]
        _c = L
    return _c


def have_ref() -> bool:
    return os.path.exists(REF_LIB)


def ref() -> C.CDLL:
    """The reference library (raises if it was not built: it needs the reference sources)."""
    global _r
    if _r is None:
        if not os.path.exists(REF_LIB):
            raise RuntimeError(f"{REF_LIB} missing: run `make -C oracle ref` where the reference sources exist")
        L = C.CDLL(REF_LIB)
        i32, i64, vp = C.c_int32, C.c_int64, C.c_void_p
        sig = {
            "ref_last_error": (C.c_char_p, []),
            "ref_mgr_new": (vp, [i32, i32]), "ref_mgr_delete": (None, [vp]),
            "ref_mgr_set_check_each_op": (None, [vp, i32]),
            "ref_mgr_admit": (C.c_int, [vp, i64, i32]),
            "ref_mgr_admit_with_prefix": (C.c_int, [vp, i64, i64, i32, i32]),
            "ref_mgr_fork": (C.c_int, [vp, i64, i64]), "ref_mgr_append_token": (C.c_int, [vp, i64]),
            "ref_mgr_free": (C.c_int, [vp, i64]), "ref_mgr_contains": (C.c_int, [vp, i64]),
            "ref_mgr_num_tokens": (C.c_int, [vp, i64]), "ref_mgr_table": (C.c_int, [vp, i64, _pi32, i32]),
            "ref_mgr_refcount": (C.c_int, [vp, i32]), "ref_mgr_free_blocks": (C.c_int, [vp]),
            "ref_mgr_total_blocks": (C.c_int, [vp]), "ref_mgr_available_blocks": (C.c_int, [vp]),
            "ref_mgr_can_admit": (C.c_int, [vp, i32]),
            "ref_mgr_blocks_needed_to_admit": (C.c_int, [vp, i64, i32, i32]),
            "ref_mgr_stats": (None, [vp, C.POINTER(C.c_int64)]),
            "ref_mgr_recompute_stats": (None, [vp, C.POINTER(C.c_int64)]),
            "ref_mgr_validate": (C.c_int, [vp, C.c_char_p, i32]),
            "ref_mgr_cache_prefix": (C.c_int, [vp, i32, i64, i32]),
            "ref_mgr_has_cached_prefix": (C.c_int, [vp, i32]),
            "ref_mgr_cached_prefix_tokens": (C.c_int, [vp, i32]),
            "ref_mgr_blocks_needed_to_admit_cached": (C.c_int, [vp, i32, i32, i32]),
            "ref_mgr_admit_with_cached_prefix": (C.c_int, [vp, i64, i32, i32, i32]),
            "ref_mgr_evictable_blocks": (C.c_int, [vp, i32, i32]),
            "ref_mgr_shared_blocks_with_cached": (C.c_int, [vp, i32, i32, i32]),
            "ref_mgr_clear_cache": (C.c_int, [vp]),
            "ref_reference_attention": (C.c_int, _ATTN),
            "ref_paged_attention_cpu": (C.c_int, _ATTN + [C.c_int]),
            "ref_paged_attention_cpu_mt": (C.c_int, _ATTN + [C.c_int, C.c_int]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _r = L
    return _r


_g = None


def have_ref_gpu() -> bool:
    return os.path.exists(REF_GPU_LIB)


def ref_gpu_attention(q, k_cache, v_cache, block_tables, seq_lens, out, num_seqs, num_heads, kv_heads, head_dim,
                      block_size, max_blocks, warps, stream=None) -> int:
    """The reference's launch_paged_attention (cuda/paged_attention.cuh:16-19) on device pointers (fp16 q, K/V
    and out; int32 tables and lengths); returns its cudaError_t."""
    global _g
    if _g is None:
        if not have_ref_gpu():
            raise RuntimeError(f"{REF_GPU_LIB} missing: run `make -C oracle ref` where the reference sources exist")
        L = C.CDLL(REF_GPU_LIB)
        L.ref_gpu_launch_paged_attention.restype = C.c_int
        L.ref_gpu_launch_paged_attention.argtypes = [C.c_void_p] * 6 + [C.c_int] * 7 + [C.c_void_p]
        _g = L
    return _g.ref_gpu_launch_paged_attention(q, k_cache, v_cache, block_tables, seq_lens, out, num_seqs, num_heads,
                                             kv_heads, head_dim, block_size, max_blocks, warps, stream)


# ----------------------------------------------------------------------------- attention
def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _call_attn(fn, nh, kvh, hd, bs, q, k, v, tables, lens, extra=()):
    q, k, v, tables, lens = _f32(q), _f32(k), _f32(v), _i32(tables), _i32(lens)
    ns = q.shape[0]
    out = np.empty((ns, nh, hd), dtype=np.float32)
    rc = fn(nh, kvh, hd, bs, ns, tables.shape[1], q.ctypes.data_as(_pf), k.ctypes.data_as(_pf),
            v.ctypes.data_as(_pf), tables.ctypes.data_as(_pi32), lens.ctypes.data_as(_pi32),
            out.ctypes.data_as(_pf), *extra)
    if rc != 0:
        raise ValueError(f"oracle rejected the input (status {rc})")
    return out


def reference_attention(nh, kvh, hd, bs, q, k, v, tables, lens, impl: str = "c"):
    """Double-precision reference (src/paged_attention.cpp:25-66). impl: "c" (restatement) or "ref"."""
    fn = c_oracle().ora_reference_attention if impl == "c" else ref().ref_reference_attention
    return _call_attn(fn, nh, kvh, hd, bs, q, k, v, tables, lens)


def paged_attention_cpu(nh, kvh, hd, bs, q, k, v, tables, lens, partitions=1, nthreads=1, impl: str = "c"):
    """fp32 partitioned online softmax (src/paged_attention.cpp:68-114)."""
    fn = c_oracle().ora_paged_attention_cpu_mt if impl == "c" else ref().ref_paged_attention_cpu_mt
    return _call_attn(fn, nh, kvh, hd, bs, q, k, v, tables, lens, (partitions, nthreads))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    y = np.empty(x.shape, dtype=np.uint16)
    c_oracle().ora_f32_to_bf16(x.ctypes.data_as(_pf), y.ctypes.data_as(C.POINTER(C.c_uint16)), x.size)
    return y


def bf16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, dtype=np.float32)
    c_oracle().ora_bf16_to_f32(x.ctypes.data_as(C.POINTER(C.c_uint16)), y.ctypes.data_as(_pf), x.size)
    return y


# ----------------------------------------------------------------------------- KV manager (reference)
STATS_FIELDS = ("requests", "used_tokens", "allocated_blocks", "allocated_slots", "internal_waste",
                "logical_blocks", "blocks_saved", "cow_copies", "cached_blocks", "cache_evictions")


class RefKVManager:
    """The reference's kvp::KVManager (compiled from its sources) behind the product's Python interface."""

    def __init__(self, num_blocks: int, block_size: int):
        self._L = ref()
        h = self._L.ref_mgr_new(num_blocks, block_size)
        if not h:
            raise ValueError(self._L.ref_last_error().decode())
        self._h = C.c_void_p(h)
        self._B = block_size

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                self._L.ref_mgr_delete(self._h)
                self._h = None
        except Exception:
            pass

    def _b(self, rc):
        if rc == -2:
            raise ValueError(self._L.ref_last_error().decode())
        if rc < 0:
            raise RuntimeError(self._L.ref_last_error().decode())
        return bool(rc)

    def _v(self, rc):
        if rc < 0:
            self._b(rc)
        return rc

    def set_check_each_op(self, on):
        self._L.ref_mgr_set_check_each_op(self._h, 1 if on else 0)

    def block_size(self):
        return self._B

    def admit(self, r, prompt):
        return self._b(self._L.ref_mgr_admit(self._h, r, prompt))

    def admit_with_prefix(self, r, parent, shared, prompt):
        return self._b(self._L.ref_mgr_admit_with_prefix(self._h, r, parent, shared, prompt))

    def fork(self, r, parent):
        return self._b(self._L.ref_mgr_fork(self._h, r, parent))

    def append_token(self, r):
        return self._b(self._L.ref_mgr_append_token(self._h, r))

    def free(self, r):
        self._b(self._L.ref_mgr_free(self._h, r))

    def contains(self, r):
        return bool(self._L.ref_mgr_contains(self._h, r))

    def num_tokens(self, r):
        return self._v(self._L.ref_mgr_num_tokens(self._h, r))

    def block_table(self, r):
        n = self._v(self._L.ref_mgr_table(self._h, r, None, 0))
        buf = (C.c_int32 * max(n, 1))()
        self._L.ref_mgr_table(self._h, r, buf, n)
        return list(buf[:n])

    def refcount(self, b):
        return self._v(self._L.ref_mgr_refcount(self._h, b))

    def free_blocks(self):
        return self._L.ref_mgr_free_blocks(self._h)

    def total_blocks(self):
        return self._L.ref_mgr_total_blocks(self._h)

    def available_blocks(self):
        return self._L.ref_mgr_available_blocks(self._h)

    def can_admit(self, prompt):
        return self._b(self._L.ref_mgr_can_admit(self._h, prompt))

    def blocks_needed_to_admit(self, parent, shared, prompt):
        return self._L.ref_mgr_blocks_needed_to_admit(self._h, parent, shared, prompt)

    def stats(self):
        buf = (C.c_int64 * 10)()
        self._L.ref_mgr_stats(self._h, buf)
        return dict(zip(STATS_FIELDS, list(buf)))

    def recompute_stats(self):
        buf = (C.c_int64 * 10)()
        self._L.ref_mgr_recompute_stats(self._h, buf)
        return dict(zip(STATS_FIELDS, list(buf)))

    def validate(self):
        buf = C.create_string_buffer(1024)
        self._L.ref_mgr_validate(self._h, buf, 1024)
        return buf.value.decode()

    def cache_prefix(self, key, owner, tokens):
        return self._b(self._L.ref_mgr_cache_prefix(self._h, key, owner, tokens))

    def has_cached_prefix(self, key):
        return bool(self._L.ref_mgr_has_cached_prefix(self._h, key))

    def cached_prefix_tokens(self, key):
        return self._L.ref_mgr_cached_prefix_tokens(self._h, key)

    def blocks_needed_to_admit_cached(self, key, shared, prompt):
        return self._L.ref_mgr_blocks_needed_to_admit_cached(self._h, key, shared, prompt)

    def admit_with_cached_prefix(self, r, key, shared, prompt):
        return self._b(self._L.ref_mgr_admit_with_cached_prefix(self._h, r, key, shared, prompt))

    def evictable_blocks(self, key=-1, shared_blocks=0):
        return self._L.ref_mgr_evictable_blocks(self._h, key, shared_blocks)

    def shared_blocks_with_cached(self, key, shared, prompt):
        return self._L.ref_mgr_shared_blocks_with_cached(self._h, key, shared, prompt)

    def clear_cache(self):
        self._b(self._L.ref_mgr_clear_cache(self._h))

    def append_batch(self, rids):
        """The reference harness's per-request decode bookkeeping (python/paged_model.py:105-118):
        returns (done, slots, cow pairs) with the same conventions as the product's append_batch."""
        B = self._B
        slots = np.full(len(rids), -1, dtype=np.int32)
        pairs = []
        done = 0
        for i, r in enumerate(rids):
            pos = self.num_tokens(r)
            tbl = self.block_table(r)
            old_last = tbl[-1] if tbl else -1
            if not self.append_token(r):
                break
            tbl2 = self.block_table(r)
            if pos % B != 0 and tbl2[-1] != old_last:
                pairs.append((old_last, tbl2[-1]))
            slots[i] = tbl2[pos // B] * B + pos % B
            done += 1
        return done, slots, np.asarray(pairs, dtype=np.int32).reshape(-1, 2)


# ----------------------------------------------------------------------------- data plane model
class DataPlane:
    """Bytes of the K/V pools as numpy uint16 arrays [L][num_blocks][B][kvh][D] (bit patterns), mutated
    exactly as the reference's Python harness does."""

    def __init__(self, k: np.ndarray, v: np.ndarray):
        self.k = np.array(k, dtype=np.uint16, copy=True)
        self.v = np.array(v, dtype=np.uint16, copy=True)
        self.L, self.nb, self.B = self.k.shape[:3]

    def scatter(self, slots, k_new, v_new):
        """python/paged_model.py:145-146: K[l, blk, off] = k_new[l, i] for every layer, slot >= 0."""
        for i, s in enumerate(np.asarray(slots)):
            if s < 0:
                continue
            blk, off = divmod(int(s), self.B)
            self.k[:, blk, off] = k_new[:, i]
            self.v[:, blk, off] = v_new[:, i]

    def cow(self, pairs):
        """python/paged_model.py:92-95 / 113-117: whole-block copy of every layer, K and V."""
        for src, dst in np.asarray(pairs).reshape(-1, 2):
            self.k[:, dst] = self.k[:, src]
            self.v[:, dst] = self.v[:, src]

    def swap_out(self, blocks):
        """Host copies of the blocks (all layers, K and V), in order."""
        return [(self.k[:, b].copy(), self.v[:, b].copy()) for b in blocks]

    def swap_in(self, blocks, saved):
        for b, (kk, vv) in zip(blocks, saved):
            self.k[:, b] = kk
            self.v[:, b] = vv
