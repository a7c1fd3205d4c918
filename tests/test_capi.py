"""The C-ABI library loads without a GPU, exports every entry point include/kvp_b200.h declares plus the
C++ drop-in API, and rejects invalid arguments before touching the device."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "kvp_b200.h")).read()
    return sorted(set(re.findall(r"KVP_API\s+[\w\s\*]+?\b(kvp_\w+)\s*\(", src)))


def test_header_declarations_are_all_exported(kvb):
    names = _declared()
    assert len(names) >= 38
    L = kvb.lib()
    for n in names:
        assert hasattr(L, n), n
    assert sorted(kvb.exported_symbols()) == names


def test_cxx_drop_in_symbols_exported(kvb):
    out = subprocess.run(["nm", "-DC", "--defined-only", kvb.LIB_PATH], capture_output=True, text=True).stdout
    for sym in ("kvp::KVManager::append_token(long)", "kvp::KVManager::admit_with_prefix(long, long, int, int)",
                "kvp::KVManager::fork(long, long)", "kvp::KVManager::free(long)",
                "kvp::BlockAllocator::allocate()", "launch_paged_attention(",
                "kvp::paged_attention(kvp::AttnShape const&",
                # the reference's host-buffer attention signatures (include/kvpage/paged_attention.h:25-35)
                "kvp::reference_attention(kvp::AttnShape const&, int, int, float const*, float const*, float const*, "
                "int const*, int const*, float*)",
                "kvp::paged_attention_cpu(kvp::AttnShape const&, int, int, float const*, float const*, float const*, "
                "int const*, int const*, float*, int)"):
        assert sym in out, sym
    # nothing from the statically linked CUDA runtime leaks out of the library
    assert " cudaMalloc" not in out


def test_version_and_error_string(kvb):
    assert b"sm_100a" in kvb.lib().kvp_version()


def _args(kvb, **kw):
    a = kvb.AttnArgs()
    a.q_dtype, a.kv_dtype, a.out_dtype = kvb.F32, kvb.F16, kvb.F32
    a.num_seqs, a.num_heads, a.kv_heads, a.head_dim, a.block_size, a.max_blocks = 2, 8, 2, 64, 16, 4
    a.num_blocks = 16
    # fake, 256-byte aligned addresses: validation fails before any device access
    a.q = a.k_cache = a.v_cache = a.block_tables = a.seq_lens = a.out = 1 << 20
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("bad", [dict(head_dim=48), dict(kv_heads=3), dict(num_heads=40, kv_heads=2),
                                 dict(kv_dtype=9), dict(q_dtype=7), dict(block_size=0), dict(k_cache=(1 << 20) + 2),
                                 dict(kv_dtype=0, k_new=1 << 20, v_new=1 << 20), dict(kv_dtype=0, head_dim=48),
                                 dict(kv_dtype=0, k_cache=(1 << 20) + 2)])
def test_attention_rejects_invalid_arguments(kvb, bad):
    L = kvb.lib()
    rc = L.kvp_paged_attention(C.byref(_args(kvb, **bad)), None)
    assert rc == kvb.KVP_EINVAL
    assert kvb.last_error()


def test_workspace_needed_only_when_split(kvb):
    L = kvb.lib()
    a = _args(kvb, split_tiles=1, max_blocks=8)
    n = L.kvp_attention_workspace_size(C.byref(a))
    assert n == pytest.approx(2 * 8 * 8 * (8 + 64 * 4), rel=0.1)
    a.split_tiles = -1
    assert L.kvp_attention_workspace_size(C.byref(a)) == 0
    a = _args(kvb, split_tiles=1, max_blocks=8)
    assert L.kvp_paged_attention(C.byref(a), None) == kvb.KVP_ENOSPACE  # no workspace given


def test_kv_ops_reject_invalid_arguments(kvb):
    L = kvb.lib()
    a = kvb.AppendArgs()
    a.kv_dtype = kvb.F32
    assert L.kvp_append_scatter(C.byref(a), None) == kvb.KVP_EINVAL
    c = kvb.CowArgs()
    c.kv_dtype, c.n_pairs, c.num_layers, c.kv_heads, c.head_dim, c.block_size = kvb.BF16, 1, 1, 1, 4, 1
    assert L.kvp_cow_copy(C.byref(c), None) == kvb.KVP_EINVAL  # 8-byte blocks
    s = kvb.SwapArgs()
    s.kv_dtype, s.num_layers, s.kv_heads, s.head_dim, s.block_size, s.n = kvb.BF16, 1, 1, 8, 1, 1
    blocks = (C.c_int32 * 1)(-1)
    slots = (C.c_int64 * 1)(0)
    s.blocks, s.host_slots = blocks, slots
    s.k_cache = s.v_cache = s.host_pool = 1 << 20
    s.host_pool_slots = 4
    assert L.kvp_swap_out(C.byref(s), None) == kvb.KVP_EBOUNDS  # negative block id
    blocks[0], slots[0] = 0, 4
    assert L.kvp_swap_in(C.byref(s), None) == kvb.KVP_EBOUNDS   # host slot beyond the pool


def test_decoder_config_validation(kvb):
    L = kvb.lib()
    c = kvb.DecoderConfig()
    assert L.kvp_decoder_workspace_size(C.byref(c)) == 0  # all-zero shape is invalid
    c.num_layers, c.num_heads, c.kv_heads, c.head_dim, c.block_size = 2, 8, 2, 64, 16
    c.kv_dtype, c.q_dtype, c.out_dtype, c.num_blocks, c.max_seqs, c.max_blocks_per_seq = 2, 2, 0, 64, 4, 8
    n = L.kvp_decoder_workspace_size(C.byref(c))
    assert n > 2 * 4 * 8 * 64 * 2  # at least the query staging
    m = kvb.KVManager(64, 16)
    assert not L.kvp_decoder_create(C.byref(c), m.handle)  # no pools / workspace
    c.split_tiles = -1
    assert L.kvp_decoder_workspace_size(C.byref(c)) < n  # no split-K partials reserved


def test_ctypes_struct_layouts_match_the_header(kvb, tmp_path):
    """Every argument struct the Python binding passes has the header's field order, offsets and size
    (the header compiled with gcc prints them)."""
    structs = {"kvp_attn_args": kvb.AttnArgs, "kvp_append_args": kvb.AppendArgs, "kvp_cow_args": kvb.CowArgs,
               "kvp_swap_args": kvb.SwapArgs, "kvp_decoder_config": kvb.DecoderConfig,
               "kvp_migrate_args": kvb.MigrateArgs}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "kvp_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        s, f, v = ln.split()
        got[(s, f)] = int(v)
    for cname, py in structs.items():
        assert got[(cname, "sizeof")] == C.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)


def test_header_constants_match_the_binding(kvb):
    """Every integer #define of include/kvp_b200.h that the Python binding mirrors has the same value, and the
    status, status-bit and attention-flag constants are all mirrored."""
    src = open(os.path.join(ROOT, "include", "kvp_b200.h")).read()
    defs = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+(KVP_\w+)\s+(\d+)\b", src)}
    assert len(defs) >= 11
    for name, value in defs.items():
        if name.startswith(("KVP_STATUS_", "KVP_ATTN_", "KVP_E")) or name == "KVP_OK":
            assert getattr(kvb, name) == value, name


C_PROGRAM = r"""
#include "kvp_b200.h"
#include <stdio.h>

/* A plain-C caller of the host control plane: prefix sharing, a fork, a batched append with copy-on-write,
   dense tables and statistics, printed for comparison with the Python binding. */
int main(void) {
    kvp_mgr* m = kvp_mgr_create(32, 16);
    if (!m) return 2;
    printf("admit %d\n", kvp_mgr_admit(m, 1, 40));
    printf("prefix %d\n", kvp_mgr_admit_with_prefix(m, 2, 1, 36, 50));
    printf("fork %d\n", kvp_mgr_fork(m, 3, 1));
    int64_t rids[3] = {1, 2, 3};
    int32_t slots[3], pairs[6], ncow = 0;
    const int done = kvp_mgr_append_batch(m, rids, 3, slots, pairs, &ncow);
    printf("append %d ncow %d\n", done, ncow);
    printf("slots %d %d %d\n", slots[0], slots[1], slots[2]);
    for (int k = 0; k < ncow; ++k) printf("pair %d %d\n", pairs[2 * k], pairs[2 * k + 1]);
    int32_t tables[3 * 4], lens[3];
    printf("dense %d\n", kvp_mgr_dense_tables(m, rids, 3, 4, -1, tables, lens));
    for (int i = 0; i < 3; ++i)
        printf("row %d %d %d %d len %d\n", tables[4 * i], tables[4 * i + 1], tables[4 * i + 2], tables[4 * i + 3],
               lens[i]);
    int64_t st[10];
    kvp_mgr_stats(m, st);
    for (int i = 0; i < 10; ++i) printf("stat %lld\n", (long long)st[i]);
    char buf[256];
    printf("validate %d\n", kvp_mgr_validate(m, buf, (int32_t)sizeof buf));
    printf("dup %d\n", kvp_mgr_admit(m, 1, 5));  /* a duplicate id is rejected with an error code */
    printf("msg %s\n", kvp_last_error()[0] ? "set" : "empty");
    kvp_mgr_destroy(m);
    return 0;
}
"""


def test_header_is_plain_c_and_drives_the_manager(kvb, tmp_path):
    """include/kvp_b200.h is a C header (what a cgo / JNI / N-API / ctypes binding would include): a C11
    program compiled with -pedantic against it and linked to the library drives the KVManager through the
    C ABI, and its results equal the same calls through the Python binding."""
    import subprocess
    src = tmp_path / "caller.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "caller"
    lib_dir = os.path.dirname(kvb.LIB_PATH)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(src), "-L", lib_dir, "-lkvpage_b200", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines()
    m = kvb.KVManager(32, 16)
    want = [f"admit {int(m.admit(1, 40))}", f"prefix {int(m.admit_with_prefix(2, 1, 36, 50))}",
            f"fork {int(m.fork(3, 1))}"]
    done, slots, pairs = m.append_batch([1, 2, 3])
    want += [f"append {done} ncow {len(pairs)}", "slots " + " ".join(str(int(x)) for x in slots)]
    want += [f"pair {int(a)} {int(b)}" for a, b in pairs]
    tables, lens = m.dense_tables([1, 2, 3], 4, pad=-1)
    want += ["dense 0"] + [f"row {' '.join(str(int(x)) for x in tables[i])} len {int(lens[i])}" for i in range(3)]
    s = m.stats()
    want += [f"stat {int(s[k])}" for k in ("requests", "used_tokens", "allocated_blocks", "allocated_slots",
                                           "internal_waste", "logical_blocks", "blocks_saved", "cow_copies",
                                           "cached_blocks", "cache_evictions")]
    want += ["validate 0"]
    assert out[:len(want)] == want
    assert out[len(want)].startswith("dup ") and int(out[len(want)].split()[1]) < 0
    assert out[len(want) + 1] == "msg set"
    assert len(pairs) == 1  # the fork's first append copied the shared partial block



def test_decoder_host_step_arguments(kvb):
    """The Python decoder's host-step wrapper: shapes [L][n][heads][D] and the config's dtypes are checked
    before the C call (a wrong size would make the copies read past the caller's buffers), host tensors only,
    contiguous or the host_inputs() views; a step that repeats the previous step's objects reuses the checked
    arguments, and a changed data pointer or a fresh list of request ids is checked again.  No GPU: a decoder
    object without a C handle."""
    import numpy as np
    import torch
    L, n, nh, kvh, D = 3, 4, 6, 2, 16
    d = kvb.Decoder.__new__(kvb.Decoder)
    c = kvb.DecoderConfig()
    c.num_layers, c.num_heads, c.kv_heads, c.head_dim = L, nh, kvh, D
    c.q_dtype = c.kv_dtype = c.out_dtype = kvb.BF16
    d.cfg, d._h, d._last_args = c, C.c_void_p(0), None
    stride = n * (nh + 2 * kvh) * D
    buf = torch.zeros(L * stride, dtype=torch.bfloat16)
    q = buf.as_strided((L, n, nh, D), (stride, nh * D, D, 1))
    k = buf.as_strided((L, n, kvh, D), (stride, kvh * D, D, 1), n * nh * D)
    v = buf.as_strided((L, n, kvh, D), (stride, kvh * D, D, 1), n * (nh + kvh) * D)
    d._host_in = ([q, k, v], None)
    out = torch.zeros((L, n, nh, D), dtype=torch.bfloat16)
    rids = np.arange(n, dtype=np.int64)
    a = d._host_step_args(rids, q, k, v, out)
    assert a[1:] == (rids.ctypes.data, n, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
    assert d._host_step_args(rids, q, k, v, out) is a  # the repeat reuses the checked arguments
    out2 = torch.zeros_like(out)
    assert d._host_step_args(rids, q, k, v, out2)[6] == out2.data_ptr()
    lst = list(range(n))
    assert d._host_step_args(lst, q, k, v, out)[2] == n and d._last_args is None  # a list is never remembered
    bad = [
        (rids[:3], q, k, v, out),                                       # n disagrees with the tensors
        (rids, q, k, v, out[:, :3]),                                    # short output
        (rids, q, k, v, out.float()),                                   # wrong dtype
        (rids, q, k, v, torch.zeros((L, nh, n, D), dtype=torch.bfloat16).transpose(1, 2)),  # strided output
        (rids, torch.zeros((L, n, 2 * nh, D), dtype=torch.bfloat16)[:, :, :nh], k, v, out),  # strided, not a view
    ]
    for args in bad:
        with pytest.raises(ValueError):
            d._host_step_args(*args)
    d._host_step_args(rids, torch.zeros((L, n, nh, D), dtype=torch.bfloat16), k, v, out)  # contiguous q: fine
    d._h = None
