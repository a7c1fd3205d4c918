// C ABI glue: error reporting, device queries, and the C view of kvp::KVManager including the batched
// decode-step append that turns KVManager decisions into device slot lists and copy-on-write pairs.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

#include "kvp_b200.h"
#include "kvp_internal.h"

namespace kvpi {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return KVP_OK;
    return fail(KVP_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
void clear_error() { g_last_error.clear(); }

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace kvpi

extern "C" KVP_API const char* kvp_last_error(void) { return kvpi::g_last_error.c_str(); }
extern "C" KVP_API const char* kvp_version(void) { return "kvpage-b200 0.1 (sm_100a)"; }

// ------------------------------------------------------------------ KVManager (kvp_mgr is in kvp_internal.h)

namespace {

template <class F>
int guarded(F&& f) {
    kvpi::clear_error();
    try {
        return f();
    } catch (const std::invalid_argument& e) {
        return -kvpi::fail(KVP_EINVAL, e.what());
    } catch (const std::logic_error& e) {
        return -kvpi::fail(KVP_ESTATE, e.what());
    } catch (const std::exception& e) {
        return -kvpi::fail(KVP_ESTATE, e.what());
    }
}

void put_stats(const kvp::KVStats& s, int64_t* out) {
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

}  // namespace

extern "C" {

KVP_API kvp_mgr* kvp_mgr_create(int32_t num_blocks, int32_t block_size) {
    kvpi::clear_error();
    try {
        return new kvp_mgr(num_blocks, block_size);
    } catch (const std::exception& e) {
        kvpi::fail(KVP_EINVAL, e.what());
        return nullptr;
    }
}
KVP_API void kvp_mgr_destroy(kvp_mgr* m) { delete m; }
KVP_API void kvp_mgr_set_check_each_op(kvp_mgr* m, int32_t on) { m->m.set_check_each_op(on != 0); }
KVP_API int kvp_mgr_admit(kvp_mgr* m, int64_t r, int32_t prompt) {
    return guarded([&] { return m->m.admit(r, prompt) ? 1 : 0; });
}
KVP_API int kvp_mgr_admit_with_prefix(kvp_mgr* m, int64_t r, int64_t parent, int32_t shared, int32_t prompt) {
    return guarded([&] { return m->m.admit_with_prefix(r, parent, shared, prompt) ? 1 : 0; });
}
KVP_API int kvp_mgr_fork(kvp_mgr* m, int64_t r, int64_t parent) {
    return guarded([&] { return m->m.fork(r, parent) ? 1 : 0; });
}
KVP_API int kvp_mgr_append_token(kvp_mgr* m, int64_t r) {
    return guarded([&] { return m->m.append_token(r) ? 1 : 0; });
}
KVP_API int kvp_mgr_free(kvp_mgr* m, int64_t r) {
    return guarded([&] {
        m->m.free(r);
        return 1;
    });
}
KVP_API int kvp_mgr_contains(kvp_mgr* m, int64_t r) { return m->m.contains(r) ? 1 : 0; }
KVP_API int kvp_mgr_num_tokens(kvp_mgr* m, int64_t r) {
    return guarded([&] { return m->m.table(r).tokens; });
}
KVP_API int kvp_mgr_table(kvp_mgr* m, int64_t r, int32_t* out, int32_t cap) {
    return guarded([&] {
        const auto& b = m->m.table(r).blocks;
        const int n = static_cast<int>(b.size());
        if (out && cap > 0) std::memcpy(out, b.data(), sizeof(int32_t) * static_cast<size_t>(std::min(n, cap)));
        return n;
    });
}
KVP_API int kvp_mgr_refcount(kvp_mgr* m, int32_t b) {
    return guarded([&] { return m->m.allocator().refcount(b); });
}
KVP_API int kvp_mgr_free_blocks(kvp_mgr* m) { return m->m.free_blocks(); }
KVP_API int kvp_mgr_total_blocks(kvp_mgr* m) { return m->m.total_blocks(); }
KVP_API int kvp_mgr_available_blocks(kvp_mgr* m) { return m->m.available_blocks(); }
KVP_API int kvp_mgr_can_admit(kvp_mgr* m, int32_t prompt) {
    return guarded([&] { return m->m.can_admit(prompt) ? 1 : 0; });
}
KVP_API int kvp_mgr_blocks_needed_to_admit(kvp_mgr* m, int64_t parent, int32_t shared, int32_t prompt) {
    return guarded([&] { return m->m.blocks_needed_to_admit(parent, shared, prompt); });
}
KVP_API void kvp_mgr_stats(kvp_mgr* m, int64_t* out) { put_stats(m->m.stats(), out); }
KVP_API void kvp_mgr_recompute_stats(kvp_mgr* m, int64_t* out) { put_stats(m->m.recompute_stats(), out); }
KVP_API int kvp_mgr_validate(kvp_mgr* m, char* buf, int32_t cap) {
    const std::string s = m->m.validate();
    if (buf && cap > 0) {
        std::strncpy(buf, s.c_str(), static_cast<size_t>(cap - 1));
        buf[cap - 1] = '\0';
    }
    return static_cast<int>(s.size());
}
KVP_API int kvp_mgr_cache_prefix(kvp_mgr* m, int32_t key, int64_t owner, int32_t tokens) {
    return guarded([&] { return m->m.cache_prefix(key, owner, tokens) ? 1 : 0; });
}
KVP_API int kvp_mgr_has_cached_prefix(kvp_mgr* m, int32_t key) { return m->m.has_cached_prefix(key) ? 1 : 0; }
KVP_API int kvp_mgr_cached_prefix_tokens(kvp_mgr* m, int32_t key) { return m->m.cached_prefix_tokens(key); }
KVP_API int kvp_mgr_blocks_needed_to_admit_cached(kvp_mgr* m, int32_t key, int32_t shared, int32_t prompt) {
    return m->m.blocks_needed_to_admit_cached(key, shared, prompt);
}
KVP_API int kvp_mgr_admit_with_cached_prefix(kvp_mgr* m, int64_t r, int32_t key, int32_t shared, int32_t prompt) {
    return guarded([&] { return m->m.admit_with_cached_prefix(r, key, shared, prompt) ? 1 : 0; });
}
KVP_API int kvp_mgr_evictable_blocks(kvp_mgr* m, int32_t key, int32_t shared_blocks) {
    return m->m.evictable_blocks(key, shared_blocks);
}
KVP_API int kvp_mgr_shared_blocks_with_cached(kvp_mgr* m, int32_t key, int32_t shared, int32_t prompt) {
    return m->m.shared_blocks_with_cached(key, shared, prompt);
}
KVP_API int kvp_mgr_clear_cache(kvp_mgr* m) {
    return guarded([&] {
        m->m.clear_cache();
        return 1;
    });
}

KVP_API int kvp_mgr_append_batch(kvp_mgr* m, const int64_t* rids, int32_t n, int32_t* slots, int32_t* cow_pairs,
                                 int32_t* n_cow) {
    return guarded([&] {
        const int B = m->m.block_size();
        int ncow = 0, done = 0;
        for (int i = 0; i < n; ++i) slots[i] = -1;
        for (int i = 0; i < n; ++i) {
            const kvp::BlockTable& t = m->m.table(rids[i]);
            const int pos = t.tokens;
            const kvp::BlockId old_last = t.blocks.empty() ? kvp::kNoBlock : t.blocks.back();
            if (!m->m.append_token(rids[i])) break;
            const kvp::BlockTable& t2 = m->m.table(rids[i]);
            const kvp::BlockId blk = t2.blocks[static_cast<size_t>(pos / B)];
            // A partial last block whose id changed was copied on write (python/paged_model.py:113-117).
            if (pos % B != 0 && t2.blocks.back() != old_last) {
                cow_pairs[2 * ncow] = old_last;
                cow_pairs[2 * ncow + 1] = t2.blocks.back();
                ++ncow;
            }
            slots[i] = blk * B + pos % B;
            ++done;
        }
        if (n_cow) *n_cow = ncow;
        return done;
    });
}

KVP_API int kvp_mgr_dense_tables(kvp_mgr* m, const int64_t* rids, int32_t n, int32_t max_blocks, int32_t pad,
                                 int32_t* tables, int32_t* lens) {
    int rc = guarded([&] {
        for (int i = 0; i < n; ++i) {
            const kvp::BlockTable& t = m->m.table(rids[i]);
            const int nb = static_cast<int>(t.blocks.size());
            if (nb > max_blocks) return -kvpi::fail(KVP_EBOUNDS, "a block table is longer than max_blocks");
            int32_t* row = tables + static_cast<size_t>(i) * max_blocks;
            if (nb) std::memcpy(row, t.blocks.data(), sizeof(int32_t) * static_cast<size_t>(nb));
            for (int j = nb; j < max_blocks; ++j) row[j] = pad;
            if (lens) lens[i] = t.tokens;
        }
        return 0;
    });
    return rc < 0 ? -rc : rc;
}

}  // extern "C"
