// Host control plane: request block tables over a reference-counted pool, with prefix sharing, fork +
// copy-on-write and an LRU prefix cache.  The decisions (which ids, in which order, when a call fails)
// reproduce the reference's src/kv_manager.cpp:155-251 step for step, because the device data plane and
// the parity tests depend on identical block ids:
//   * allocation pops the allocator's LIFO stack; releases push in table order;
//   * admission shares floor(min(shared, parent tokens, prompt) / B) full blocks, retaining them before
//     any cache reclaim, and allocates the rest with per-block fill min(B, remaining);
//   * append: block boundary -> new block; shared partial last block -> copy-on-write into a new block;
//     otherwise in place; the cache is reclaimed first when a block is needed and none is free;
//   * cache reclaim evicts, one entry at a time, the least recently used entry that still holds a block
//     no request references, until enough blocks are free (src/kv_manager.cpp:75-88).
#include "kvpage/kv_manager.h"

#include <algorithm>
#include <stdexcept>

namespace kvp {

namespace {
int clamp_shared(int a, int b, int c) { return std::max(0, std::min(a, std::min(b, c))); }
}  // namespace

KVManager::KVManager(int num_blocks, int block_size) : block_size_(block_size), pool_(num_blocks) {
    if (block_size <= 0) throw std::invalid_argument("KVManager: block_size must be positive");
    fill_.assign(static_cast<size_t>(num_blocks), 0);
}

const BlockTable& KVManager::table(RequestId r) const {
    auto it = requests_.find(r);
    if (it == requests_.end()) throw std::logic_error("KVManager: no request " + std::to_string(r));
    return it->second;
}

void KVManager::checkpoint() const {
    if (!check_each_op_) return;
    const std::string problem = validate();
    if (!problem.empty()) throw std::logic_error("KVManager invariant broken: " + problem);
}

void KVManager::drop_ref(BlockId b) {
    pool_.release(b);
    if (pool_.refcount(b) == 0) {
        filled_slots_ -= fill_[static_cast<size_t>(b)];
        fill_[static_cast<size_t>(b)] = 0;
    }
}

BlockId KVManager::take_block(int fill) {
    const BlockId b = pool_.allocate();
    if (b != kNoBlock) {
        fill_[static_cast<size_t>(b)] = fill;
        filled_slots_ += fill;
    }
    return b;
}

// ------------------------------------------------------------------ prefix cache

std::unordered_map<BlockId, int> KVManager::cache_holds() const {
    std::unordered_map<BlockId, int> holds;
    for (const auto& kv : cache_)
        for (BlockId b : kv.second.blocks) holds[b] += 1;
    return holds;
}

void KVManager::evict(CacheMap::iterator it) {
    for (BlockId b : it->second.blocks) drop_ref(b);
    cache_.erase(it);
    evictions_ += 1;
}

bool KVManager::make_room(int blocks) {
    while (pool_.free_blocks() < blocks) {
        const auto holds = cache_holds();
        auto only_cached = [&](BlockId b) {
            auto h = holds.find(b);
            return h != holds.end() && pool_.refcount(b) == h->second;
        };
        CacheMap::iterator oldest = cache_.end();
        for (auto it = cache_.begin(); it != cache_.end(); ++it) {
            const auto& bl = it->second.blocks;
            if (std::none_of(bl.begin(), bl.end(), only_cached)) continue;
            if (oldest == cache_.end() || it->second.stamp < oldest->second.stamp) oldest = it;
        }
        if (oldest == cache_.end()) return false;
        evict(oldest);
    }
    return true;
}

int KVManager::shared_blocks_with_cached(int key, int shared_tokens, int prompt_tokens) const {
    auto it = cache_.find(key);
    if (it == cache_.end()) return 0;
    return clamp_shared(shared_tokens, it->second.tokens, prompt_tokens) / block_size_;
}

int KVManager::evictable_blocks(int key, int shared_blocks) const {
    auto holds = cache_holds();
    if (key >= 0) {
        auto it = cache_.find(key);
        if (it != cache_.end()) {
            const int keep = std::min(shared_blocks, static_cast<int>(it->second.blocks.size()));
            for (int i = 0; i < keep; ++i) holds.erase(it->second.blocks[static_cast<size_t>(i)]);
        }
    }
    int n = 0;
    for (const auto& h : holds) n += pool_.refcount(h.first) == h.second;
    return n;
}

int KVManager::cache_only_blocks() const { return cache_.empty() ? 0 : evictable_blocks(); }

bool KVManager::cache_prefix(int key, RequestId owner, int tokens) {
    if (cache_.count(key)) return false;
    const BlockTable& t = table(owner);
    const int full = std::max(0, std::min(tokens, t.tokens)) / block_size_;
    if (full == 0) return false;
    PrefixEntry e;
    e.blocks.assign(t.blocks.begin(), t.blocks.begin() + full);
    for (BlockId b : e.blocks) pool_.retain(b);
    e.tokens = full * block_size_;
    e.stamp = ++clock_;
    cache_.emplace(key, std::move(e));
    checkpoint();
    return true;
}

int KVManager::cached_prefix_tokens(int key) const {
    auto it = cache_.find(key);
    return it == cache_.end() ? 0 : it->second.tokens;
}

int KVManager::blocks_needed_to_admit_cached(int key, int shared_tokens, int prompt_tokens) const {
    return ceil_div(prompt_tokens, block_size_) - shared_blocks_with_cached(key, shared_tokens, prompt_tokens);
}

void KVManager::clear_cache() {
    while (!cache_.empty()) evict(cache_.begin());
    evictions_ = 0;
    checkpoint();
}

// ------------------------------------------------------------------ requests

int KVManager::blocks_needed_to_admit(RequestId parent, int shared_tokens, int prompt_tokens) const {
    int shared = 0;
    if (parent != kNoRequest) shared = clamp_shared(shared_tokens, table(parent).tokens, prompt_tokens) / block_size_;
    return ceil_div(prompt_tokens, block_size_) - shared;
}

bool KVManager::can_admit(int prompt_tokens) const {
    return available_blocks() >= blocks_needed_to_admit(kNoRequest, 0, prompt_tokens);
}

bool KVManager::admit(RequestId r, int prompt_tokens) { return admit_with_prefix(r, kNoRequest, 0, prompt_tokens); }

// Common tail of both prefix admissions: `shared` are the leading full blocks to share (not yet retained).
bool KVManager::admit_shared(RequestId r, const std::vector<BlockId>& shared, int prompt_tokens) {
    for (BlockId b : shared) pool_.retain(b);  // before reclaim, so eviction cannot free them
    const int n_shared = static_cast<int>(shared.size());
    const int fresh = ceil_div(prompt_tokens, block_size_) - n_shared;
    if (!make_room(fresh)) {
        for (BlockId b : shared) drop_ref(b);
        return false;
    }
    BlockTable t;
    t.tokens = prompt_tokens;
    t.blocks.reserve(static_cast<size_t>(n_shared + fresh));
    t.blocks.insert(t.blocks.end(), shared.begin(), shared.end());
    for (int i = 0; i < fresh; ++i) {
        const int remaining = prompt_tokens - (n_shared + i) * block_size_;
        t.blocks.push_back(take_block(std::min(block_size_, remaining)));
    }
    table_entries_ += static_cast<int64_t>(t.blocks.size());
    requests_.emplace(r, std::move(t));
    ++table_changes_;
    checkpoint();
    return true;
}

bool KVManager::admit_with_prefix(RequestId r, RequestId parent, int shared_tokens, int prompt_tokens) {
    if (requests_.count(r)) throw std::logic_error("KVManager: request " + std::to_string(r) + " already admitted");
    if (prompt_tokens < 0) throw std::invalid_argument("KVManager: negative prompt length");
    const int fresh = blocks_needed_to_admit(parent, shared_tokens, prompt_tokens);
    const int n_shared = ceil_div(prompt_tokens, block_size_) - fresh;
    std::vector<BlockId> shared;
    if (n_shared > 0) {
        const auto& pb = table(parent).blocks;
        shared.assign(pb.begin(), pb.begin() + n_shared);
    }
    return admit_shared(r, shared, prompt_tokens);
}

bool KVManager::admit_with_cached_prefix(RequestId r, int key, int shared_tokens, int prompt_tokens) {
    if (requests_.count(r)) throw std::logic_error("KVManager: request " + std::to_string(r) + " already admitted");
    if (prompt_tokens < 0) throw std::invalid_argument("KVManager: negative prompt length");
    std::vector<BlockId> shared;
    auto it = cache_.find(key);
    if (it != cache_.end()) {
        it->second.stamp = ++clock_;
        const int n = shared_blocks_with_cached(key, shared_tokens, prompt_tokens);
        shared.assign(it->second.blocks.begin(), it->second.blocks.begin() + n);
    }
    return admit_shared(r, shared, prompt_tokens);
}

bool KVManager::fork(RequestId r, RequestId parent) {
    if (requests_.count(r)) throw std::logic_error("KVManager: request " + std::to_string(r) + " already admitted");
    BlockTable child = table(parent);
    for (BlockId b : child.blocks) pool_.retain(b);
    table_entries_ += static_cast<int64_t>(child.blocks.size());
    requests_.emplace(r, std::move(child));
    ++table_changes_;
    checkpoint();
    return true;
}

bool KVManager::append_token(RequestId r) {
    auto it = requests_.find(r);
    if (it == requests_.end()) throw std::logic_error("KVManager: no request " + std::to_string(r));
    BlockTable& t = it->second;
    const int used_in_last = t.tokens % block_size_;
    const bool boundary = used_in_last == 0;
    // Reclaim cache blocks first when a block will be needed; reclaiming can lower the last block's
    // refcount, so the copy-on-write decision is taken afterwards.
    if ((boundary || pool_.refcount(t.blocks.back()) > 1) && pool_.free_blocks() < 1) make_room(1);
    if (boundary) {
        const BlockId b = take_block(1);
        if (b == kNoBlock) return false;
        t.blocks.push_back(b);
        table_entries_ += 1;
    } else if (pool_.refcount(t.blocks.back()) > 1) {
        const BlockId b = take_block(used_in_last + 1);
        if (b == kNoBlock) return false;
        drop_ref(t.blocks.back());  // the other holders keep the old block and its fill
        t.blocks.back() = b;
        cow_events_ += 1;
    } else {
        fill_[static_cast<size_t>(t.blocks.back())] += 1;
        filled_slots_ += 1;
    }
    t.tokens += 1;
    ++table_changes_;
    checkpoint();
    return true;
}

void KVManager::free(RequestId r) {
    auto it = requests_.find(r);
    if (it == requests_.end()) throw std::logic_error("KVManager: no request " + std::to_string(r));
    for (BlockId b : it->second.blocks) drop_ref(b);
    table_entries_ -= static_cast<int64_t>(it->second.blocks.size());
    requests_.erase(it);
    ++table_changes_;
    checkpoint();
}

// ------------------------------------------------------------------ statistics and validation

KVStats KVManager::stats() const {
    KVStats s;
    s.requests = static_cast<int>(requests_.size());
    s.used_tokens = filled_slots_;
    s.logical_blocks = table_entries_;
    s.allocated_blocks = pool_.referenced_blocks();
    s.allocated_slots = s.allocated_blocks * block_size_;
    s.internal_waste = s.allocated_slots - s.used_tokens;
    s.blocks_saved = s.logical_blocks - (s.allocated_blocks - cache_only_blocks());
    s.cow_copies = cow_events_;
    s.cache_evictions = evictions_;
    for (const auto& kv : cache_) s.cached_blocks += static_cast<int64_t>(kv.second.blocks.size());
    return s;
}

KVStats KVManager::recompute_stats() const {
    KVStats s;
    s.requests = static_cast<int>(requests_.size());
    std::vector<int> fill(static_cast<size_t>(pool_.total_blocks()), 0);
    for (const auto& kv : requests_) {
        const BlockTable& t = kv.second;
        s.logical_blocks += static_cast<int64_t>(t.blocks.size());
        for (size_t i = 0; i < t.blocks.size(); ++i) {
            const int f = std::min(block_size_, t.tokens - static_cast<int>(i) * block_size_);
            int& slot = fill[static_cast<size_t>(t.blocks[i])];
            slot = std::max(slot, f);
        }
    }
    for (const auto& kv : cache_) {
        for (BlockId b : kv.second.blocks) fill[static_cast<size_t>(b)] = block_size_;  // cached blocks are full
        s.cached_blocks += static_cast<int64_t>(kv.second.blocks.size());
    }
    for (int f : fill) s.used_tokens += f;
    s.allocated_blocks = pool_.referenced_blocks();
    s.allocated_slots = s.allocated_blocks * block_size_;
    s.internal_waste = s.allocated_slots - s.used_tokens;
    s.blocks_saved = s.logical_blocks - (s.allocated_blocks - cache_only_blocks());
    s.cow_copies = cow_events_;
    s.cache_evictions = evictions_;
    return s;
}

std::string KVManager::validate() const {
    std::string problem = pool_.validate();
    if (!problem.empty()) return problem;
    const int n = pool_.total_blocks();
    std::vector<int64_t> refs(static_cast<size_t>(n), 0);
    int64_t entries = 0;
    for (const auto& kv : requests_) {
        const BlockTable& t = kv.second;
        if (static_cast<int>(t.blocks.size()) != ceil_div(t.tokens, block_size_))
            return "request " + std::to_string(kv.first) + " has a table length that does not match its tokens";
        for (BlockId b : t.blocks) {
            if (b < 0 || b >= n) return "request " + std::to_string(kv.first) + " holds a block outside the pool";
            refs[static_cast<size_t>(b)] += 1;
            entries += 1;
        }
    }
    for (const auto& kv : cache_) {
        const PrefixEntry& e = kv.second;
        if (e.tokens != static_cast<int>(e.blocks.size()) * block_size_)
            return "prefix entry " + std::to_string(kv.first) + " token count does not match its blocks";
        for (BlockId b : e.blocks) {
            if (b < 0 || b >= n) return "prefix entry " + std::to_string(kv.first) + " holds a block outside the pool";
            if (fill_[static_cast<size_t>(b)] != block_size_) return "a cached block is not completely filled";
            refs[static_cast<size_t>(b)] += 1;
            entries += 1;
        }
    }
    int64_t total = 0;
    for (int b = 0; b < n; ++b) {
        if (refs[static_cast<size_t>(b)] != pool_.refcount(b))
            return "block " + std::to_string(b) + " refcount differs from its table and cache references";
        total += pool_.refcount(b);
    }
    if (total != entries) return "refcount total differs from the number of table and cache entries";
    const KVStats a = stats(), b = recompute_stats();
    if (a.used_tokens != b.used_tokens || a.logical_blocks != b.logical_blocks || a.blocks_saved != b.blocks_saved ||
        a.internal_waste != b.internal_waste || a.cached_blocks != b.cached_blocks)
        return "incremental statistics differ from recomputed ones";
    return std::string();
}

}  // namespace kvp
