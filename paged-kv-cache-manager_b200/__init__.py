"""kvpage-b200: B200-native paged KV cache data plane.

Python mirror of the library's C ABI (include/kvp_b200.h), loaded with ctypes from the in-tree
libkvpage_b200.so.  It mirrors the reference's Python binding (python/kvpage_py.cpp:12-66 of
prathameshpranjale/paged-kv-cache-manager: KVManager with block_table / num_tokens / refcount / stats /
validate) and adds the device entry points: paged_attention, append_scatter, cow_copy, swap_out/in.
Device buffers are torch CUDA tensors (torch supplies device memory and streams); every computation runs
in this library's CUDA kernels.  There is no CPU fallback: without the shared library, or for CPU
tensors, the device calls raise.

The directory name contains dashes, so import it with importlib:
    kvb = importlib.import_module("paged-kv-cache-manager_b200")
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkvpage_b200.so")

KVP_OK, KVP_EINVAL, KVP_ECUDA, KVP_EBOUNDS, KVP_ENOSPACE, KVP_ESTATE = 0, 1, 2, 3, 4, 5
KVP_STATUS_BAD_BLOCK, KVP_STATUS_BAD_LEN, KVP_STATUS_TIMEOUT = 1, 2, 4
KVP_ATTN_WORKSPACE_CLEAN = 1
KVP_ATTN_EARLY_START = 2
KVP_ATTN_EARLY_LOAD = 4
KVP_NOALLOC_SCRATCH_BYTES = 32 << 20  # the no-allocation entry point's fixed scratch array
F32, F16, BF16 = 0, 1, 2
NO_REQUEST = -1
STATS_FIELDS = ("requests", "used_tokens", "allocated_blocks", "allocated_slots", "internal_waste",
                "logical_blocks", "blocks_saved", "cow_copies", "cached_blocks", "cache_evictions")

class KVStats(dict):
    """KVManager statistics (kvpage::KVStats): a dict of STATS_FIELDS that also reads as attributes
    (`stats().cow_copies`), as the reference's Python binding exposes them (python/kvpage_py.cpp:14-20)."""

    def __getattr__(self, name):
        try:
            return self[name]
        except KeyError:
            raise AttributeError(name) from None


_i32, _i64, _vp, _f32, _sz = C.c_int32, C.c_int64, C.c_void_p, C.c_float, C.c_size_t
_pi32, _pi64 = C.POINTER(C.c_int32), C.POINTER(C.c_int64)


class AttnArgs(C.Structure):
    _fields_ = [("q", _vp), ("q_dtype", _i32), ("k_cache", _vp), ("v_cache", _vp), ("kv_dtype", _i32),
                ("num_blocks", _i64), ("block_tables", _vp), ("seq_lens", _vp), ("out", _vp), ("out_dtype", _i32),
                ("num_seqs", _i32), ("num_heads", _i32), ("kv_heads", _i32), ("head_dim", _i32),
                ("block_size", _i32), ("max_blocks", _i32), ("scale", _f32), ("split_tiles", _i32),
                ("kv_heads_per_cta", _i32), ("stages", _i32), ("workspace", _vp), ("workspace_bytes", _sz),
                ("status", _vp), ("warps_per_kv_head", _i32), ("flags", _i32), ("k_new", _vp), ("v_new", _vp),
                ("seq_start_tiles", _i32), ("inputs_ready", _vp), ("inputs_epoch", _vp)]


class AppendArgs(C.Structure):
    _fields_ = [("k_new", _vp), ("v_new", _vp), ("k_cache", _vp), ("v_cache", _vp), ("layer_stride", _i64),
                ("slots", _vp), ("kv_dtype", _i32), ("num_layers", _i32), ("num_seqs", _i32), ("kv_heads", _i32),
                ("head_dim", _i32), ("block_size", _i32), ("num_blocks", _i64), ("status", _vp)]


class CowArgs(C.Structure):
    _fields_ = [("k_cache", _vp), ("v_cache", _vp), ("layer_stride", _i64), ("pairs", _vp), ("n_pairs", _i32),
                ("kv_dtype", _i32), ("num_layers", _i32), ("kv_heads", _i32), ("head_dim", _i32),
                ("block_size", _i32), ("num_blocks", _i64), ("status", _vp)]


class MigrateArgs(C.Structure):
    _fields_ = [("src_k_cache", _vp), ("src_v_cache", _vp), ("src_layer_stride", _i64), ("src_num_blocks", _i64),
                ("dst_k_cache", _vp), ("dst_v_cache", _vp), ("dst_layer_stride", _i64), ("dst_num_blocks", _i64),
                ("pairs", _vp), ("n_pairs", _i32), ("kv_dtype", _i32), ("num_layers", _i32), ("kv_heads", _i32),
                ("head_dim", _i32), ("block_size", _i32), ("status", _vp)]


class SwapArgs(C.Structure):
    _fields_ = [("k_cache", _vp), ("v_cache", _vp), ("layer_stride", _i64), ("kv_dtype", _i32),
                ("num_layers", _i32), ("kv_heads", _i32), ("head_dim", _i32), ("block_size", _i32),
                ("num_blocks", _i64), ("blocks", _pi32), ("host_slots", _pi64), ("n", _i32), ("host_pool", _vp),
                ("host_pool_slots", _i64)]


class DecoderConfig(C.Structure):
    _fields_ = [("num_layers", _i32), ("num_heads", _i32), ("kv_heads", _i32), ("head_dim", _i32),
                ("block_size", _i32), ("kv_dtype", _i32), ("q_dtype", _i32), ("out_dtype", _i32),
                ("num_blocks", _i64), ("layer_stride", _i64), ("max_seqs", _i32), ("max_blocks_per_seq", _i32),
                ("split_tiles", _i32), ("k_cache", _vp), ("v_cache", _vp), ("workspace", _vp),
                ("workspace_bytes", _sz), ("graph", _i32)]


# (name, restype, argtypes) of every C-ABI entry point in include/kvp_b200.h.
_SIGNATURES = [
    ("kvp_last_error", C.c_char_p, []),
    ("kvp_version", C.c_char_p, []),
    ("kvp_attention_workspace_size", _sz, [C.POINTER(AttnArgs)]),
    ("kvp_paged_attention", C.c_int, [C.POINTER(AttnArgs), _vp]),
    ("kvp_paged_attention_noalloc", C.c_int, [C.POINTER(AttnArgs), _vp]),
    ("kvp_attention_wait_test", C.c_int, [C.POINTER(AttnArgs), _vp, _i64, _i32]),
    ("kvp_paged_attention_host", C.c_int, [_i32] * 6 + [_vp] * 6 + [_i32]),
    ("kvp_append_scatter", C.c_int, [C.POINTER(AppendArgs), _vp]),
    ("kvp_cow_copy", C.c_int, [C.POINTER(CowArgs), _vp]),
    ("kvp_migrate_blocks", C.c_int, [C.POINTER(MigrateArgs), _vp]),
    ("kvp_enable_peer_access", C.c_int, [_i32]),
    ("kvp_swap_out", C.c_int, [C.POINTER(SwapArgs), _vp]),
    ("kvp_swap_in", C.c_int, [C.POINTER(SwapArgs), _vp]),
    ("kvp_mgr_create", _vp, [_i32, _i32]),
    ("kvp_mgr_destroy", None, [_vp]),
    ("kvp_mgr_set_check_each_op", None, [_vp, _i32]),
    ("kvp_mgr_admit", C.c_int, [_vp, _i64, _i32]),
    ("kvp_mgr_admit_with_prefix", C.c_int, [_vp, _i64, _i64, _i32, _i32]),
    ("kvp_mgr_fork", C.c_int, [_vp, _i64, _i64]),
    ("kvp_mgr_append_token", C.c_int, [_vp, _i64]),
    ("kvp_mgr_free", C.c_int, [_vp, _i64]),
    ("kvp_mgr_contains", C.c_int, [_vp, _i64]),
    ("kvp_mgr_num_tokens", C.c_int, [_vp, _i64]),
    ("kvp_mgr_table", C.c_int, [_vp, _i64, _pi32, _i32]),
    ("kvp_mgr_refcount", C.c_int, [_vp, _i32]),
    ("kvp_mgr_free_blocks", C.c_int, [_vp]),
    ("kvp_mgr_total_blocks", C.c_int, [_vp]),
    ("kvp_mgr_available_blocks", C.c_int, [_vp]),
    ("kvp_mgr_can_admit", C.c_int, [_vp, _i32]),
    ("kvp_mgr_blocks_needed_to_admit", C.c_int, [_vp, _i64, _i32, _i32]),
    ("kvp_mgr_stats", None, [_vp, _pi64]),
    ("kvp_mgr_recompute_stats", None, [_vp, _pi64]),
    ("kvp_mgr_validate", C.c_int, [_vp, C.c_char_p, _i32]),
    ("kvp_mgr_cache_prefix", C.c_int, [_vp, _i32, _i64, _i32]),
    ("kvp_mgr_has_cached_prefix", C.c_int, [_vp, _i32]),
    ("kvp_mgr_cached_prefix_tokens", C.c_int, [_vp, _i32]),
    ("kvp_mgr_blocks_needed_to_admit_cached", C.c_int, [_vp, _i32, _i32, _i32]),
    ("kvp_mgr_admit_with_cached_prefix", C.c_int, [_vp, _i64, _i32, _i32, _i32]),
    ("kvp_mgr_evictable_blocks", C.c_int, [_vp, _i32, _i32]),
    ("kvp_mgr_shared_blocks_with_cached", C.c_int, [_vp, _i32, _i32, _i32]),
    ("kvp_mgr_clear_cache", C.c_int, [_vp]),
    ("kvp_mgr_append_batch", C.c_int, [_vp, _pi64, _i32, _pi32, _pi32, _pi32]),
    ("kvp_mgr_dense_tables", C.c_int, [_vp, _pi64, _i32, _i32, _i32, _pi32, _pi32]),
    ("kvp_decoder_workspace_size", _sz, [C.POINTER(DecoderConfig)]),
    ("kvp_decoder_create", _vp, [C.POINTER(DecoderConfig), _vp]),
    ("kvp_decoder_destroy", None, [_vp]),
    # request ids go in as the address of an int64 array (c_void_p: no ctypes pointer object per step)
    ("kvp_decoder_step", C.c_int, [_vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    ("kvp_decoder_step_device", C.c_int, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    ("kvp_decoder_submit", C.c_int, [_vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    ("kvp_decoder_host_inputs", C.c_int, [_vp, _i32, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_sz)]),
    ("kvp_decoder_plan", C.c_int, [_vp, _vp, _i32]),
    ("kvp_decoder_wait", C.c_int, [_vp]),
    ("kvp_decoder_status", C.c_int, [_vp]),
]

_lib = None


def lib() -> C.CDLL:
    """The loaded libkvpage_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing; build it with build_lib.py (no CPU fallback exists)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in _SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list:
    return [n for n, _, _ in _SIGNATURES]


def last_error() -> str:
    return lib().kvp_last_error().decode()


class KVPError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"kvp error {code}: {msg}")
        self.code = code


def _check(rc: int) -> int:
    if rc != KVP_OK:
        msg = last_error()
        if rc in (KVP_EINVAL,):
            raise ValueError(msg)
        raise KVPError(rc, msg)
    return rc


def _bool(rc: int) -> bool:
    """Maps a bool-returning C entry point: 1/0, or -code when the C++ side threw."""
    if rc < 0:
        code = -rc
        msg = last_error()
        if code == KVP_EINVAL:
            raise ValueError(msg)
        raise RuntimeError(msg)  # std::logic_error in the reference
    return bool(rc)


# ============================================================================ host control plane
class KVManager:
    """kvp::KVManager through the C ABI; method names follow the reference's Python binding."""

    def __init__(self, num_blocks: int, block_size: int):
        self._L = lib()
        h = self._L.kvp_mgr_create(num_blocks, block_size)
        if not h:
            raise ValueError(last_error())
        self._h = C.c_void_p(h)
        self._B = block_size

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                self._L.kvp_mgr_destroy(self._h)
                self._h = None
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def set_check_each_op(self, on: bool):
        self._L.kvp_mgr_set_check_each_op(self._h, 1 if on else 0)

    def block_size(self) -> int:
        return self._B

    def admit(self, r: int, prompt: int) -> bool:
        return _bool(self._L.kvp_mgr_admit(self._h, r, prompt))

    def admit_with_prefix(self, r: int, parent: int, shared: int, prompt: int) -> bool:
        return _bool(self._L.kvp_mgr_admit_with_prefix(self._h, r, parent, shared, prompt))

    def fork(self, r: int, parent: int) -> bool:
        return _bool(self._L.kvp_mgr_fork(self._h, r, parent))

    def append_token(self, r: int) -> bool:
        return _bool(self._L.kvp_mgr_append_token(self._h, r))

    def free(self, r: int):
        _bool(self._L.kvp_mgr_free(self._h, r))

    def contains(self, r: int) -> bool:
        return bool(self._L.kvp_mgr_contains(self._h, r))

    def num_tokens(self, r: int) -> int:
        v = self._L.kvp_mgr_num_tokens(self._h, r)
        if v < 0:
            _bool(v)
        return v

    def block_table(self, r: int) -> list:
        n = self._L.kvp_mgr_table(self._h, r, None, 0)
        if n < 0:
            _bool(n)
        buf = (C.c_int32 * max(n, 1))()
        self._L.kvp_mgr_table(self._h, r, buf, n)
        return list(buf[:n])

    def refcount(self, b: int) -> int:
        v = self._L.kvp_mgr_refcount(self._h, b)
        if v < 0:
            _bool(v)
        return v

    def free_blocks(self) -> int:
        return self._L.kvp_mgr_free_blocks(self._h)

    def total_blocks(self) -> int:
        return self._L.kvp_mgr_total_blocks(self._h)

    def available_blocks(self) -> int:
        return self._L.kvp_mgr_available_blocks(self._h)

    def can_admit(self, prompt: int) -> bool:
        return _bool(self._L.kvp_mgr_can_admit(self._h, prompt))

    def blocks_needed_to_admit(self, parent: int, shared_tokens: int, prompt_tokens: int) -> int:
        v = self._L.kvp_mgr_blocks_needed_to_admit(self._h, parent, shared_tokens, prompt_tokens)
        if v < 0 and last_error():
            _bool(v)
        return v

    def stats(self) -> KVStats:
        buf = (C.c_int64 * 10)()
        self._L.kvp_mgr_stats(self._h, buf)
        return KVStats(zip(STATS_FIELDS, list(buf)))

    def recompute_stats(self) -> KVStats:
        buf = (C.c_int64 * 10)()
        self._L.kvp_mgr_recompute_stats(self._h, buf)
        return KVStats(zip(STATS_FIELDS, list(buf)))

    def validate(self) -> str:
        buf = C.create_string_buffer(1024)
        self._L.kvp_mgr_validate(self._h, buf, 1024)
        return buf.value.decode()

    def cache_prefix(self, key: int, owner: int, tokens: int) -> bool:
        return _bool(self._L.kvp_mgr_cache_prefix(self._h, key, owner, tokens))

    def has_cached_prefix(self, key: int) -> bool:
        return bool(self._L.kvp_mgr_has_cached_prefix(self._h, key))

    def cached_prefix_tokens(self, key: int) -> int:
        return self._L.kvp_mgr_cached_prefix_tokens(self._h, key)

    def blocks_needed_to_admit_cached(self, key: int, shared: int, prompt: int) -> int:
        return self._L.kvp_mgr_blocks_needed_to_admit_cached(self._h, key, shared, prompt)

    def admit_with_cached_prefix(self, r: int, key: int, shared: int, prompt: int) -> bool:
        return _bool(self._L.kvp_mgr_admit_with_cached_prefix(self._h, r, key, shared, prompt))

    def evictable_blocks(self, key: int = -1, shared_blocks: int = 0) -> int:
        return self._L.kvp_mgr_evictable_blocks(self._h, key, shared_blocks)

    def shared_blocks_with_cached(self, key: int, shared: int, prompt: int) -> int:
        return self._L.kvp_mgr_shared_blocks_with_cached(self._h, key, shared, prompt)

    def clear_cache(self):
        _bool(self._L.kvp_mgr_clear_cache(self._h))

    # ---- decode-step helpers (native loops) ----
    def append_batch(self, rids: Sequence[int]):
        """append_token for each request in order; returns (done, slots[n], cow_pairs[k][2])."""
        import numpy as np
        n = len(rids)
        r = np.ascontiguousarray(np.asarray(rids, dtype=np.int64))
        slots = np.empty(max(n, 1), dtype=np.int32)
        pairs = np.empty(max(2 * n, 2), dtype=np.int32)
        ncow = C.c_int32(0)
        done = self._L.kvp_mgr_append_batch(self._h, r.ctypes.data_as(_pi64), n, slots.ctypes.data_as(_pi32),
                                            pairs.ctypes.data_as(_pi32), C.byref(ncow))
        if done < 0:
            _bool(done)
        return done, slots[:n], pairs[: 2 * ncow.value].reshape(-1, 2)

    def dense_tables(self, rids: Sequence[int], max_blocks: int, pad: int = 0):
        """Padded [n][max_blocks] int32 tables and int32 lengths of the given requests."""
        import numpy as np
        n = len(rids)
        r = np.ascontiguousarray(np.asarray(rids, dtype=np.int64))
        tables = np.empty((max(n, 1), max_blocks), dtype=np.int32)
        lens = np.empty(max(n, 1), dtype=np.int32)
        _check(self._L.kvp_mgr_dense_tables(self._h, r.ctypes.data_as(_pi64), n, max_blocks, pad,
                                            tables.ctypes.data_as(_pi32), lens.ctypes.data_as(_pi32)))
        return tables[:n], lens[:n]


# ============================================================================ device entry points
def _dtype_code(t) -> int:
    import torch
    m = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
    if t.dtype not in m:
        raise ValueError(f"unsupported dtype {t.dtype}")
    return m[t.dtype]


def _dev(t, name):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _same_device(*named):
    """All given tensors (None skipped) on one CUDA device; returns it.  Launches go to that device."""
    dev = None
    for name, t in named:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name} is on {t.device}, the other operands on {dev}")
    return dev


def _launch(device, fn, args, stream):
    """Calls a C-ABI launcher with `device` current (the library launches on the current device) on `stream`
    (default: that device's current stream)."""
    import torch
    with torch.cuda.device(device):
        _check(fn(C.byref(args), _stream_ptr(stream)))


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def attention_args(q, k_cache, v_cache, block_tables, seq_lens, out, num_heads, kv_heads, *, num_blocks=None,
                   workspace=None, split_tiles=0, kv_heads_per_cta=0, stages=0, status=None, scale=0.0,
                   warps_per_kv_head=0, k_new=None, v_new=None, seq_start_tiles=0, inputs_ready=None) -> AttnArgs:
    """AttnArgs for one layer; k_cache/v_cache are [num_blocks][B][kv_heads][D] (or views of them).  With
    k_new/v_new ([num_seqs][kv_heads][D], pool dtype) the kernel first writes each sequence's newest token.
    inputs_ready: an int32 device word the kernel waits for (non-zero) before it reads q / k_new / v_new."""
    nb, B, kvh, D = k_cache.shape[-4:]
    assert kvh == kv_heads
    a = AttnArgs()
    a.q, a.q_dtype = _dev(q, "q"), _dtype_code(q)
    a.k_cache, a.v_cache, a.kv_dtype = _dev(k_cache, "k_cache"), _dev(v_cache, "v_cache"), _dtype_code(k_cache)
    a.num_blocks = nb if num_blocks is None else num_blocks
    a.block_tables, a.seq_lens = _dev(block_tables, "block_tables"), _dev(seq_lens, "seq_lens")
    a.out, a.out_dtype = _dev(out, "out"), _dtype_code(out)
    a.num_seqs, a.num_heads, a.kv_heads, a.head_dim = q.shape[0], num_heads, kv_heads, D
    a.block_size, a.max_blocks = B, block_tables.shape[1]
    a.scale, a.split_tiles, a.kv_heads_per_cta, a.stages = scale, split_tiles, kv_heads_per_cta, stages
    a.warps_per_kv_head = warps_per_kv_head
    a.seq_start_tiles = seq_start_tiles
    if workspace is not None:
        a.workspace, a.workspace_bytes = _dev(workspace, "workspace"), workspace.numel() * workspace.element_size()
    a.status = _dev(status, "status") if status is not None else None
    if (k_new is None) != (v_new is None):
        raise ValueError("k_new and v_new go together")
    if k_new is not None:
        for t, name in ((k_new, "k_new"), (v_new, "v_new")):
            if tuple(t.shape) != (q.shape[0], kv_heads, D) or t.dtype != k_cache.dtype or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous [num_seqs][kv_heads][head_dim] tensor in the pool dtype")
        a.k_new, a.v_new = _dev(k_new, "k_new"), _dev(v_new, "v_new")
    if inputs_ready is not None:
        a.inputs_ready = _dev(inputs_ready, "inputs_ready")
    return a


def workspace_bytes(args: AttnArgs) -> int:
    return int(lib().kvp_attention_workspace_size(C.byref(args)))


def paged_attention(q, k_cache, v_cache, block_tables, seq_lens, num_heads: int, kv_heads: int, *, out=None,
                    out_dtype=None, workspace=None, split_tiles: int = 0, kv_heads_per_cta: int = 0, stages: int = 0,
                    status=None, stream=None, num_blocks: Optional[int] = None, warps_per_kv_head: int = 0,
                    k_new=None, v_new=None, early_start: bool = False, early_load: bool = False,
                    seq_start_tiles: int = 0):
    """Decode attention through the C ABI (kvp_paged_attention).  Allocates `out` (and a workspace when
    none is given and the context will be split) with torch if not provided.  k_new/v_new: fused append of
    each sequence's newest token (position seq_lens[s] - 1) before attending.  early_start: the kernel may start
    while the previous kernel on the stream still runs (it must not write seq_lens); early_load: it may also
    load K/V before that kernel ends (which must not write block_tables or these pools either)."""
    import torch
    dev = _same_device(("q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("block_tables", block_tables),
                       ("seq_lens", seq_lens), ("out", out), ("workspace", workspace), ("status", status),
                       ("k_new", k_new), ("v_new", v_new))
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype or q.dtype, device=q.device)
    a = attention_args(q, k_cache, v_cache, block_tables, seq_lens, out, num_heads, kv_heads, num_blocks=num_blocks,
                       workspace=workspace, split_tiles=split_tiles, kv_heads_per_cta=kv_heads_per_cta,
                       stages=stages, status=status, warps_per_kv_head=warps_per_kv_head, k_new=k_new, v_new=v_new,
                       seq_start_tiles=seq_start_tiles)
    if workspace is None and split_tiles >= 0:
        need = workspace_bytes(a)
        if need:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
            a.workspace, a.workspace_bytes = workspace.data_ptr(), need
            a.flags |= KVP_ATTN_WORKSPACE_CLEAN
    if early_start:
        a.flags |= KVP_ATTN_EARLY_START
    if early_load:
        a.flags |= KVP_ATTN_EARLY_LOAD
    _launch(dev, lib().kvp_paged_attention, a, stream)
    return out


def paged_attention_host(num_heads: int, kv_heads: int, head_dim: int, block_size: int, q, k_cache, v_cache,
                         block_tables, seq_lens, partitions: int = 1):
    """kvp_paged_attention_host: the reference's CPU attention signature (host arrays, fp32) on the device path
    of the current CUDA device -- copy in, the fp32 CUDA-core kernel, copy out.  q [ns][nh][D], k/v
    [num_blocks][B][kvh][D], tables [ns][max_blocks] int32, lens [ns] int32; returns out [ns][nh][D] (numpy,
    fp32).  The reference's argument checks raise ValueError, as its binding's std::invalid_argument does."""
    import numpy as np
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k_cache, dtype=np.float32)
    v = np.ascontiguousarray(v_cache, dtype=np.float32)
    t = np.ascontiguousarray(block_tables, dtype=np.int32)
    n = np.ascontiguousarray(seq_lens, dtype=np.int32)
    out = np.empty(q.shape, dtype=np.float32)
    rc = lib().kvp_paged_attention_host(num_heads, kv_heads, head_dim, block_size, q.shape[0],
                                        t.shape[1] if t.ndim == 2 else 0, q.ctypes.data, k.ctypes.data,
                                        v.ctypes.data, t.ctypes.data, n.ctypes.data, out.ctypes.data, partitions)
    if rc in (KVP_EINVAL, KVP_EBOUNDS):
        raise ValueError(last_error())
    _check(rc)
    return out


def append_scatter(k_new, v_new, k_cache, v_cache, slots, *, status=None, stream=None):
    """k_new/v_new: [L][num_seqs][kvh][D]; k_cache/v_cache: [L][num_blocks][B][kvh][D]; slots int32 [num_seqs]."""
    L, nb, B, kvh, D = k_cache.shape
    a = AppendArgs()
    a.k_new, a.v_new = _dev(k_new, "k_new"), _dev(v_new, "v_new")
    a.k_cache, a.v_cache = _dev(k_cache, "k_cache"), _dev(v_cache, "v_cache")
    a.layer_stride, a.slots = nb * B * kvh * D, _dev(slots, "slots")
    a.kv_dtype, a.num_layers, a.num_seqs = _dtype_code(k_cache), L, slots.shape[0]
    a.kv_heads, a.head_dim, a.block_size, a.num_blocks = kvh, D, B, nb
    a.status = _dev(status, "status") if status is not None else None
    dev = _same_device(("k_new", k_new), ("v_new", v_new), ("k_cache", k_cache), ("v_cache", v_cache),
                       ("slots", slots), ("status", status))
    _launch(dev, lib().kvp_append_scatter, a, stream)


def cow_copy(k_cache, v_cache, pairs, *, status=None, stream=None):
    """pairs: int32 [n][2] device tensor of (src, dst) blocks."""
    L, nb, B, kvh, D = k_cache.shape
    a = CowArgs()
    a.k_cache, a.v_cache = _dev(k_cache, "k_cache"), _dev(v_cache, "v_cache")
    a.layer_stride, a.pairs, a.n_pairs = nb * B * kvh * D, _dev(pairs, "pairs"), pairs.shape[0]
    a.kv_dtype, a.num_layers, a.kv_heads, a.head_dim, a.block_size, a.num_blocks = (
        _dtype_code(k_cache), L, kvh, D, B, nb)
    a.status = _dev(status, "status") if status is not None else None
    dev = _same_device(("k_cache", k_cache), ("v_cache", v_cache), ("pairs", pairs), ("status", status))
    _launch(dev, lib().kvp_cow_copy, a, stream)


def _swap(fn, k_cache, v_cache, blocks, host_slots, host_pool, stream):
    import numpy as np
    L, nb, B, kvh, D = k_cache.shape
    b = np.ascontiguousarray(np.asarray(blocks, dtype=np.int32))
    s = np.ascontiguousarray(np.asarray(host_slots, dtype=np.int64))
    a = SwapArgs()
    a.k_cache, a.v_cache = _dev(k_cache, "k_cache"), _dev(v_cache, "v_cache")
    a.layer_stride, a.kv_dtype, a.num_layers = nb * B * kvh * D, _dtype_code(k_cache), L
    a.kv_heads, a.head_dim, a.block_size, a.num_blocks = kvh, D, B, nb
    a.blocks, a.host_slots, a.n = b.ctypes.data_as(_pi32), s.ctypes.data_as(_pi64), len(b)
    if host_pool.is_cuda or not host_pool.is_pinned():
        raise ValueError("host_pool must be pinned host memory")
    a.host_pool = host_pool.data_ptr()
    a.host_pool_slots = host_pool.numel() * host_pool.element_size() // host_slot_bytes(L, B, kvh, D,
                                                                                         k_cache.element_size())
    _launch(_same_device(("k_cache", k_cache), ("v_cache", v_cache)), fn, a, stream)


def migrate_blocks(src_k, src_v, dst_k, dst_v, pairs, *, status=None, stream=None):
    """Whole-block copies from one shard's pools [L][nb][B][kvh][D] into another's (same or peer GPU), on a
    stream of the destination device.  pairs: int32 [n][2] (src block, dst block) on the destination device."""
    L, snb, B, kvh, D = src_k.shape
    dnb = dst_k.shape[1]
    if dst_k.shape[0] != L or tuple(dst_k.shape[2:]) != (B, kvh, D) or dst_k.dtype != src_k.dtype:
        raise ValueError("source and destination pools differ in shape or dtype")
    a = MigrateArgs()
    a.src_k_cache, a.src_v_cache = _dev(src_k, "src_k"), _dev(src_v, "src_v")
    a.dst_k_cache, a.dst_v_cache = _dev(dst_k, "dst_k"), _dev(dst_v, "dst_v")
    a.src_layer_stride, a.src_num_blocks = snb * B * kvh * D, snb
    a.dst_layer_stride, a.dst_num_blocks = dnb * B * kvh * D, dnb
    a.pairs, a.n_pairs = _dev(pairs, "pairs"), pairs.shape[0]
    a.kv_dtype, a.num_layers, a.kv_heads, a.head_dim, a.block_size = _dtype_code(src_k), L, kvh, D, B
    a.status = _dev(status, "status") if status is not None else None
    _same_device(("src_k", src_k), ("src_v", src_v))
    dev = _same_device(("dst_k", dst_k), ("dst_v", dst_v), ("pairs", pairs), ("status", status))
    _launch(dev, lib().kvp_migrate_blocks, a, stream)


def migrate_request(src_mgr: "KVManager", src_k, src_v, dst_mgr: "KVManager", dst_k, dst_v, rid: int,
                    dst_rid: Optional[int] = None, *, status=None, stream=None, src_stream=None) -> bool:
    """Moves request `rid` from one shard to another: admitted on the destination manager with fresh blocks
    (as `dst_rid`, default the same id), its blocks copied over (kvp_migrate_blocks on `stream`, a stream of
    the destination device), then freed on the source manager.  The source stream (default: the source
    device's current stream) waits for the copy, so later source-side writes into the freed blocks cannot
    overtake it.  Returns False, changing nothing, if the destination has no room."""
    import numpy as np
    import torch
    dst_rid = rid if dst_rid is None else dst_rid
    tokens = src_mgr.num_tokens(rid)
    if not dst_mgr.admit(dst_rid, tokens):
        return False
    src_tbl, dst_tbl = src_mgr.block_table(rid), dst_mgr.block_table(dst_rid)
    pairs = torch.from_numpy(np.asarray([src_tbl, dst_tbl], dtype=np.int32).T.copy()).to(dst_k.device)
    stream = stream or torch.cuda.current_stream(dst_k.device)
    migrate_blocks(src_k, src_v, dst_k, dst_v, pairs, status=status, stream=stream)
    ev = torch.cuda.Event()
    ev.record(stream)
    (src_stream or torch.cuda.current_stream(src_k.device)).wait_event(ev)
    src_mgr.free(rid)
    return True


def swap_out(k_cache, v_cache, blocks, host_slots, host_pool, *, stream=None):
    """Copies the given blocks (all layers, K and V) into host slots of a pinned pool."""
    _swap(lib().kvp_swap_out, k_cache, v_cache, blocks, host_slots, host_pool, stream)


def swap_in(k_cache, v_cache, blocks, host_slots, host_pool, *, stream=None):
    """Copies host slots back into the given (freshly admitted) blocks."""
    _swap(lib().kvp_swap_in, k_cache, v_cache, blocks, host_slots, host_pool, stream)


def host_slot_bytes(num_layers: int, block_size: int, kv_heads: int, head_dim: int, elem: int = 2) -> int:
    return 2 * num_layers * block_size * kv_heads * head_dim * elem


# ============================================================================ decode-step runtime
class Decoder:
    """kvp_decoder: one call per decode step for one GPU shard (appends through `mgr`, copy-on-write, and a
    fused append + attention launch for every layer).  k_cache / v_cache: [L][num_blocks][B][kv_heads][D]
    device pools.  The workspace is allocated here with torch unless one is passed.  graph: replay a step's
    launches as a CUDA graph while the batch size and buffers repeat."""

    def __init__(self, mgr: "KVManager", k_cache, v_cache, num_heads: int, max_seqs: int, max_blocks_per_seq: int,
                 q_dtype=None, out_dtype=None, split_tiles: int = 0, workspace=None, graph: bool = True):
        import torch
        L, nb, B, kvh, D = k_cache.shape
        c = DecoderConfig()
        c.num_layers, c.num_heads, c.kv_heads, c.head_dim, c.block_size = L, num_heads, kvh, D, B
        c.kv_dtype = _dtype_code(k_cache)
        tq = {None: c.kv_dtype, torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
        c.q_dtype, c.out_dtype = tq[q_dtype], tq[out_dtype]
        c.num_blocks, c.layer_stride = nb, nb * B * kvh * D
        c.max_seqs, c.max_blocks_per_seq, c.split_tiles = max_seqs, max_blocks_per_seq, split_tiles
        c.k_cache, c.v_cache = _dev(k_cache, "k_cache"), _dev(v_cache, "v_cache")
        c.graph = 1 if graph else 0
        self._L = lib()
        need = int(self._L.kvp_decoder_workspace_size(C.byref(c)))
        if need == 0:
            raise ValueError("invalid decoder configuration")
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=k_cache.device)
        c.workspace, c.workspace_bytes = _dev(workspace, "workspace"), workspace.numel() * workspace.element_size()
        self._ws, self._k, self._v, self._mgr, self.cfg = workspace, k_cache, v_cache, mgr, c
        self._last_args = None  # the previous host step's objects and validated C arguments
        with torch.cuda.device(k_cache.device):
            h = self._L.kvp_decoder_create(C.byref(c), mgr.handle)
        if not h:
            raise KVPError(KVP_EINVAL, last_error())
        self._h = C.c_void_p(h)

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                self._L.kvp_decoder_destroy(self._h)
                self._h = None
        except Exception:
            pass

    @staticmethod
    def _rids(rids):
        import numpy as np
        return np.ascontiguousarray(np.asarray(rids, dtype=np.int64))

    def step(self, rids, q, k_new, v_new, out):
        """Host tensors (pinned for overlap): q/out [L][n][nh][D], k_new/v_new [L][n][kvh][D].  Returns once
        `out` holds the step's attention outputs."""
        _check(self._L.kvp_decoder_step(*self._host_step_args(rids, q, k_new, v_new, out)))

    def _host_step_args(self, rids, q, k_new, v_new, out):
        """The C arguments of a host-buffer step, validated: shapes [L][n][heads][D] and dtypes of the config,
        host memory, contiguous (inputs may also be the host_inputs() views).  A serving loop passes the same
        objects every step (one int64 request-id array, the same tensors): that repeat reuses the validation
        and re-reads only the data pointers, so the call costs the host a few microseconds, not ~10."""
        c = self._last_args
        if c is not None and c[0] is rids and c[1] is q and c[2] is k_new and c[3] is v_new and c[4] is out:
            ptrs = (q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), out.data_ptr())
            if ptrs == c[5] and len(rids) == c[6][2]:
                return c[6]
        r = self._rids(rids)
        n = len(r)
        cfg = self.cfg
        for t, heads, code, name in ((q, cfg.num_heads, cfg.q_dtype, "q"), (k_new, cfg.kv_heads, cfg.kv_dtype, "k_new"),
                                     (v_new, cfg.kv_heads, cfg.kv_dtype, "v_new"),
                                     (out, cfg.num_heads, cfg.out_dtype, "out")):
            if t.is_cuda:
                raise ValueError(f"{name}: the decoder's host-buffer steps take host tensors")
            want = (cfg.num_layers, n, heads, cfg.head_dim)
            if tuple(t.shape) != want or _dtype_code(t) != code:
                raise ValueError(f"{name}: expected {want} of the config's dtype, got {tuple(t.shape)} {t.dtype}")
            if not (t.is_contiguous() or (name != "out" and self._is_host_view(t))):
                raise ValueError(f"{name}: host tensors must be contiguous (inputs may be the host_inputs() views)")
        ptrs = (q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), out.data_ptr())
        args = (self._h, r.ctypes.data, n) + ptrs
        # only an int64 array the caller owns is remembered: a list converted here could change in place
        self._last_args = (rids, q, k_new, v_new, out, ptrs, args) if r is rids else None
        return args

    def host_inputs(self, n: int):
        """The decoder's own pinned input buffers for a step of n requests (kvp_decoder_host_inputs): q, k_new,
        v_new as [L][n][heads][D] host tensors whose layers interleave in one allocation, so a step given them
        copies each group of layers up in one transfer.  Write a step's inputs into them and pass them to
        submit() / step()."""
        import numpy as np
        import torch
        c = self.cfg
        ptrs = [C.c_void_p() for _ in range(3)]
        stride = _sz()
        _check(self._L.kvp_decoder_host_inputs(self._h, n, C.byref(ptrs[0]), C.byref(ptrs[1]), C.byref(ptrs[2]),
                                                C.byref(stride)))
        dt = {F32: (np.float32, torch.float32), F16: (np.uint16, torch.float16), BF16: (np.uint16, torch.bfloat16)}
        total = c.num_layers * stride.value
        base = ptrs[0].value
        buf = np.ctypeslib.as_array((C.c_uint8 * total).from_address(base))
        out = []
        for p, heads, code in ((ptrs[0], c.num_heads, c.q_dtype), (ptrs[1], c.kv_heads, c.kv_dtype),
                               (ptrs[2], c.kv_heads, c.kv_dtype)):
            npt, tt = dt[code]
            item = np.dtype(npt).itemsize
            view = np.lib.stride_tricks.as_strided(
                buf[p.value - base:].view(npt), shape=(c.num_layers, n, heads, c.head_dim),
                strides=(stride.value, heads * c.head_dim * item, c.head_dim * item, item))
            out.append(torch.from_numpy(view).view(tt))
        self._host_in = (out, buf)  # keeps the views' memory referenced while they are in use
        return out

    def _is_host_view(self, t):
        views = getattr(self, "_host_in", None)
        return views is not None and any(t.data_ptr() == v.data_ptr() and t.shape == v.shape and
                                         t.stride() == v.stride() for v in views[0])

    def submit(self, rids, q, k_new, v_new, out):
        """step() without the wait: issues the step's copies and launches and returns; `out` is complete after
        wait()."""
        _check(self._L.kvp_decoder_submit(*self._host_step_args(rids, q, k_new, v_new, out)))

    def plan(self, rids):
        """The next step's bookkeeping now (its KVManager appends happen at once), overlapping a submitted step;
        the next submit / step / step_device must be for the same requests in the same order."""
        r = self._rids(rids)
        _check(self._L.kvp_decoder_plan(self._h, r.ctypes.data, len(r)))

    def wait(self):
        """Returns once the submitted step's outputs are in host memory."""
        _check(self._L.kvp_decoder_wait(self._h))

    def step_device(self, rids, q, k_new, v_new, out, stream=None):
        """Device tensors of the host step's shapes and dtypes, contiguous; asynchronous on `stream`."""
        r = self._rids(rids)
        n, cfg = len(r), self.cfg
        for t, heads, code, name in ((q, cfg.num_heads, cfg.q_dtype, "q"), (k_new, cfg.kv_heads, cfg.kv_dtype, "k_new"),
                                     (v_new, cfg.kv_heads, cfg.kv_dtype, "v_new"),
                                     (out, cfg.num_heads, cfg.out_dtype, "out")):
            want = (cfg.num_layers, n, heads, cfg.head_dim)
            if tuple(t.shape) != want or _dtype_code(t) != code:
                raise ValueError(f"{name}: expected {want} of the config's dtype, got {tuple(t.shape)} {t.dtype}")
        _check(self._L.kvp_decoder_step_device(self._h, r.ctypes.data, n, _dev(q, "q"), _dev(k_new, "k_new"),
                                                _dev(v_new, "v_new"), _dev(out, "out"), _stream_ptr(stream)))

    def status(self) -> int:
        return int(self._L.kvp_decoder_status(self._h))
