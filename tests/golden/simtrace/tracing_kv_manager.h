// Fixture-generation shim, force-included (g++ -include) into the reference's src/simulator.cpp only: every
// `KVManager` the simulator constructs becomes a TracingKVManager, which forwards each call to the reference's
// own kvp::KVManager and records the mutating ones (with their results) and the once-per-step stats() call.
// The recorded list is the scheduler's decision stream; nothing in it is computed here.
#pragma once
#include <array>
#include <cstdint>
#include <string>
#include <vector>

#include "kvpage/kv_manager.h"

namespace kvp {

enum TraceOp : int64_t {
    kTraceStep = 0,         // stats(): the simulator's end-of-step sample
    kTraceAdmitPrefix = 1,  // admit_with_prefix(r, parent, shared_tokens, prompt_tokens)
    kTraceAdmitCached = 2,  // admit_with_cached_prefix(r, key, shared_tokens, prompt_tokens)
    kTraceCachePrefix = 3,  // cache_prefix(key, owner, tokens)
    kTraceFork = 4,         // fork(child, parent)
    kTraceAppend = 5,       // append_token(r)
    kTraceFree = 6,         // free(r); column 2 holds the request's tokens at that moment
    kTraceClearCache = 7,   // clear_cache()
};

// Rows of {op, a, b, c, d, result}.
inline std::vector<std::array<int64_t, 6>>& trace_rows() {
    static std::vector<std::array<int64_t, 6>> rows;
    return rows;
}

class TracingKVManager {
public:
    TracingKVManager(int num_blocks, int block_size) : m_(num_blocks, block_size) {}

    void set_check_each_op(bool on) { m_.set_check_each_op(on); }
    int blocks_needed_to_admit(RequestId p, int s, int n) const { return m_.blocks_needed_to_admit(p, s, n); }
    int blocks_needed_to_admit_cached(int k, int s, int n) const { return m_.blocks_needed_to_admit_cached(k, s, n); }
    int shared_blocks_with_cached(int k, int s, int n) const { return m_.shared_blocks_with_cached(k, s, n); }
    int evictable_blocks(int k = -1, int s = 0) const { return m_.evictable_blocks(k, s); }
    bool has_cached_prefix(int k) const { return m_.has_cached_prefix(k); }
    int free_blocks() const { return m_.free_blocks(); }
    const BlockTable& table(RequestId r) const { return m_.table(r); }
    std::string validate() const { return m_.validate(); }

    bool admit_with_prefix(RequestId r, RequestId parent, int shared, int prompt) {
        const bool ok = m_.admit_with_prefix(r, parent, shared, prompt);
        rec(kTraceAdmitPrefix, r, parent, shared, prompt, ok);
        return ok;
    }
    bool admit_with_cached_prefix(RequestId r, int key, int shared, int prompt) {
        const bool ok = m_.admit_with_cached_prefix(r, key, shared, prompt);
        rec(kTraceAdmitCached, r, key, shared, prompt, ok);
        return ok;
    }
    bool cache_prefix(int key, RequestId owner, int tokens) {
        const bool ok = m_.cache_prefix(key, owner, tokens);
        rec(kTraceCachePrefix, key, owner, tokens, 0, ok);
        return ok;
    }
    bool fork(RequestId child, RequestId parent) {
        const bool ok = m_.fork(child, parent);
        rec(kTraceFork, child, parent, 0, 0, ok);
        return ok;
    }
    bool append_token(RequestId r) {
        const bool ok = m_.append_token(r);
        rec(kTraceAppend, r, 0, 0, 0, ok);
        return ok;
    }
    void free(RequestId r) {
        const int64_t tokens = m_.table(r).tokens;
        m_.free(r);
        rec(kTraceFree, r, tokens, 0, 0, 1);
    }
    void clear_cache() {
        m_.clear_cache();
        rec(kTraceClearCache, 0, 0, 0, 0, 1);
    }
    KVStats stats() const {
        const KVStats s = m_.stats();
        rec(kTraceStep, s.requests, s.allocated_blocks, s.cow_copies, s.cache_evictions, 1);
        return s;
    }

private:
    static void rec(int64_t op, int64_t a, int64_t b, int64_t c, int64_t d, int64_t res) {
        trace_rows().push_back({op, a, b, c, d, res});
    }
    KVManager m_;
};

}  // namespace kvp

#define KVManager TracingKVManager
