// ORACLE -- test infrastructure, not product code.
//
// A C-ABI shim over the reference's own C++ library (prathameshpranjale/paged-kv-cache-manager,
// src/block_allocator.cpp, src/kv_manager.cpp, src/paged_attention.cpp).  oracle/Makefile compiles this
// file together with those reference sources, where they lie, into oracle/_ref/libkvpage_ref.so, so the
// tests can drive the real reference KVManager and the real reference attention functions from Python
// and compare them with the product.  Nothing in the product links or loads it.
//
// Conventions: functions that can throw return an int status: 1/0 for the reference's bool results,
// -2 for std::invalid_argument, -3 for std::logic_error, -4 for any other exception; the message of the
// last exception is available from ref_last_error().
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "kvpage/kv_manager.h"
#include "kvpage/paged_attention.h"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return -2;
    } catch (const std::logic_error& e) {
        g_err = e.what();
        return -3;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -4;
    }
}
kvp::KVManager* M(void* p) { return static_cast<kvp::KVManager*>(p); }
}  // namespace

REF_API const char* ref_last_error() { return g_err.c_str(); }

REF_API void* ref_mgr_new(int num_blocks, int block_size) {
    try {
        return new kvp::KVManager(num_blocks, block_size);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}
REF_API void ref_mgr_delete(void* m) { delete M(m); }
REF_API void ref_mgr_set_check_each_op(void* m, int on) { M(m)->set_check_each_op(on != 0); }

REF_API int ref_mgr_admit(void* m, int64_t r, int prompt) {
    return guarded([&] { return M(m)->admit(r, prompt) ? 1 : 0; });
}
REF_API int ref_mgr_admit_with_prefix(void* m, int64_t r, int64_t parent, int shared, int prompt) {
    return guarded([&] { return M(m)->admit_with_prefix(r, parent, shared, prompt) ? 1 : 0; });
}
REF_API int ref_mgr_fork(void* m, int64_t r, int64_t parent) {
    return guarded([&] { return M(m)->fork(r, parent) ? 1 : 0; });
}
REF_API int ref_mgr_append_token(void* m, int64_t r) {
    return guarded([&] { return M(m)->append_token(r) ? 1 : 0; });
}
REF_API int ref_mgr_free(void* m, int64_t r) {
    return guarded([&] {
        M(m)->free(r);
        return 1;
    });
}
REF_API int ref_mgr_contains(void* m, int64_t r) { return M(m)->contains(r) ? 1 : 0; }
REF_API int ref_mgr_num_tokens(void* m, int64_t r) {
    return guarded([&] { return M(m)->table(r).tokens; });
}
// Copies up to `cap` block ids of request r into out; returns the table length (or a negative status).
REF_API int ref_mgr_table(void* m, int64_t r, int32_t* out, int cap) {
    return guarded([&] {
        const auto& b = M(m)->table(r).blocks;
        for (int i = 0; i < static_cast<int>(b.size()) && i < cap; ++i) out[i] = b[i];
        return static_cast<int>(b.size());
    });
}
REF_API int ref_mgr_refcount(void* m, int32_t b) {
    return guarded([&] { return M(m)->allocator().refcount(b); });
}
REF_API int ref_mgr_free_blocks(void* m) { return M(m)->free_blocks(); }
REF_API int ref_mgr_total_blocks(void* m) { return M(m)->total_blocks(); }
REF_API int ref_mgr_available_blocks(void* m) { return M(m)->available_blocks(); }
REF_API int ref_mgr_can_admit(void* m, int prompt) {
    return guarded([&] { return M(m)->can_admit(prompt) ? 1 : 0; });
}
REF_API int ref_mgr_blocks_needed_to_admit(void* m, int64_t parent, int shared, int prompt) {
    return guarded([&] { return M(m)->blocks_needed_to_admit(parent, shared, prompt); });
}
// stats -> out[10]: requests, used_tokens, allocated_blocks, allocated_slots, internal_waste,
// logical_blocks, blocks_saved, cow_copies, cached_blocks, cache_evictions.
static void put_stats(const kvp::KVStats& s, int64_t* out) {
    out[0] = s.requests;
    out[1] = s.used_tokens;
    out[2] = s.allocated_blocks;
    out[3] = s.allocated_slots;
    out[4] = s.internal_waste;
    out[5] = s.logical_blocks;
    out[6] = s.blocks_saved;
    out[7] = s.cow_copies;
    out[8] = s.cached_blocks;
    out[9] = s.cache_evictions;
}
REF_API void ref_mgr_stats(void* m, int64_t* out) { put_stats(M(m)->stats(), out); }
REF_API void ref_mgr_recompute_stats(void* m, int64_t* out) { put_stats(M(m)->recompute_stats(), out); }
// Writes the validate() message (empty when consistent) into buf; returns its length.
REF_API int ref_mgr_validate(void* m, char* buf, int cap) {
    std::string s = M(m)->validate();
    if (cap > 0) {
        std::strncpy(buf, s.c_str(), static_cast<size_t>(cap - 1));
        buf[cap - 1] = '\0';
    }
    return static_cast<int>(s.size());
}
REF_API int ref_mgr_cache_prefix(void* m, int key, int64_t owner, int tokens) {
    return guarded([&] { return M(m)->cache_prefix(key, owner, tokens) ? 1 : 0; });
}
REF_API int ref_mgr_has_cached_prefix(void* m, int key) { return M(m)->has_cached_prefix(key) ? 1 : 0; }
REF_API int ref_mgr_cached_prefix_tokens(void* m, int key) { return M(m)->cached_prefix_tokens(key); }
REF_API int ref_mgr_blocks_needed_to_admit_cached(void* m, int key, int shared, int prompt) {
    return M(m)->blocks_needed_to_admit_cached(key, shared, prompt);
}
REF_API int ref_mgr_admit_with_cached_prefix(void* m, int64_t r, int key, int shared, int prompt) {
    return guarded([&] { return M(m)->admit_with_cached_prefix(r, key, shared, prompt) ? 1 : 0; });
}
REF_API int ref_mgr_evictable_blocks(void* m, int key, int shared_blocks) {
    return M(m)->evictable_blocks(key, shared_blocks);
}
REF_API int ref_mgr_shared_blocks_with_cached(void* m, int key, int shared, int prompt) {
    return M(m)->shared_blocks_with_cached(key, shared, prompt);
}
REF_API int ref_mgr_clear_cache(void* m) {
    return guarded([&] {
        M(m)->clear_cache();
        return 1;
    });
}

// ---- attention: the reference's own CPU functions (src/paged_attention.cpp) ----
REF_API int ref_reference_attention(int nh, int kvh, int hd, int bs, int ns, int max_blocks, const float* q,
                                    const float* k, const float* v, const int32_t* tables, const int32_t* lens,
                                    float* out) {
    return guarded([&] {
        kvp::AttnShape s{nh, kvh, hd, bs};
        kvp::reference_attention(s, ns, max_blocks, q, k, v, tables, lens, out);
        return 0;
    });
}

// The reference's paged_attention_cpu on `nthreads` host threads: sequences are split into contiguous
// slices and each thread calls the reference function on its slice (it is pure, so slices are independent).
REF_API int ref_paged_attention_cpu_mt(int nh, int kvh, int hd, int bs, int ns, int max_blocks, const float* q,
                                       const float* k, const float* v, const int32_t* tables, const int32_t* lens,
                                       float* out, int partitions, int nthreads) {
    return guarded([&] {
        kvp::AttnShape s{nh, kvh, hd, bs};
        if (nthreads < 1) nthreads = 1;
        if (nthreads > ns) nthreads = ns > 0 ? ns : 1;
        if (nthreads == 1) {
            kvp::paged_attention_cpu(s, ns, max_blocks, q, k, v, tables, lens, out, partitions);
            return 0;
        }
        std::vector<std::thread> th;
        std::vector<std::string> errs(static_cast<size_t>(nthreads));
        const size_t qstride = static_cast<size_t>(nh) * hd;
        for (int t = 0; t < nthreads; ++t) {
            const int s0 = static_cast<int>(static_cast<int64_t>(ns) * t / nthreads);
            const int s1 = static_cast<int>(static_cast<int64_t>(ns) * (t + 1) / nthreads);
            th.emplace_back([&, t, s0, s1] {
                try {
                    kvp::paged_attention_cpu(s, s1 - s0, max_blocks, q + s0 * qstride, k, v,
                                             tables + static_cast<size_t>(s0) * max_blocks, lens + s0,
                                             out + s0 * qstride, partitions);
                } catch (const std::exception& e) {
                    errs[static_cast<size_t>(t)] = e.what();
                }
            });
        }
        for (auto& x : th) x.join();
        for (const auto& e : errs)
            if (!e.empty()) throw std::invalid_argument(e);
        return 0;
    });
}

REF_API int ref_paged_attention_cpu(int nh, int kvh, int hd, int bs, int ns, int max_blocks, const float* q,
                                    const float* k, const float* v, const int32_t* tables, const int32_t* lens,
                                    float* out, int partitions) {
    return ref_paged_attention_cpu_mt(nh, kvh, hd, bs, ns, max_blocks, q, k, v, tables, lens, out, partitions, 1);
}
