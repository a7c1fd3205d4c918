// Host control plane of the paged KV cache: which physical blocks each request owns or shares.
//
// Public API and observable behaviour are those of the reference's include/kvpage/kv_manager.h:26-77
// (admit, admit_with_prefix, fork, append_token, free, table, stats, the persistent prefix cache and
// validate), so block ids, refcounts, return values and statistics are identical for the same call
// sequence.  The device data plane (append scatter, copy-on-write copies, swap) acts on the decisions
// this class makes; see kvp_b200.h.  Not thread-safe: one instance per GPU shard, one host thread.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "kvpage/block_allocator.h"
#include "kvpage/block_table.h"

namespace kvp {

struct KVStats {
    int requests = 0;
    int64_t used_tokens = 0;       // filled token slots, a shared block counted once
    int64_t allocated_blocks = 0;  // physical blocks with refcount > 0
    int64_t allocated_slots = 0;   // allocated_blocks * block_size
    int64_t internal_waste = 0;    // allocated_slots - used_tokens
    int64_t logical_blocks = 0;    // sum of all block-table lengths
    int64_t blocks_saved = 0;      // logical_blocks - blocks held by requests (sharing)
    int64_t cow_copies = 0;        // copy-on-write events so far
    int64_t cached_blocks = 0;     // entries held by the prefix cache
    int64_t cache_evictions = 0;   // prefix-cache entries evicted so far
};

class KVPAGE_EXPORT KVManager {
public:
    KVManager(int num_blocks, int block_size);

    // ceil(prompt/B) minus the full blocks that would be shared with `parent` (kNoRequest: none).
    int blocks_needed_to_admit(RequestId parent, int shared_tokens, int prompt_tokens) const;
    bool can_admit(int prompt_tokens) const;

    bool admit(RequestId r, int prompt_tokens);
    // Shares parent's completely filled leading blocks (never a partial one) and allocates the rest.
    // On failure nothing changes except prefix-cache entries evicted while looking for room.
    bool admit_with_prefix(RequestId r, RequestId parent, int shared_tokens, int prompt_tokens);
    // Shares every block of `parent`, a partial last block included.
    bool fork(RequestId r, RequestId parent);
    // One more token: a new block at a block boundary, a copy-on-write block when the partial last block
    // is shared, otherwise the same block.  false (state unchanged) when no block can be found.
    bool append_token(RequestId r);
    void free(RequestId r);

    bool contains(RequestId r) const { return requests_.count(r) != 0; }
    const BlockTable& table(RequestId r) const;
    KVStats stats() const;            // O(1) apart from the cache terms
    KVStats recompute_stats() const;  // from scratch; validate() compares the two

    int block_size() const { return block_size_; }
    int free_blocks() const { return pool_.free_blocks(); }
    int total_blocks() const { return pool_.total_blocks(); }
    const BlockAllocator& allocator() const { return pool_; }

    // ---- persistent prefix cache (full blocks that outlive their request; LRU-reclaimed on demand) ----
    bool cache_prefix(int key, RequestId owner, int tokens);
    bool has_cached_prefix(int key) const { return cache_.count(key) != 0; }
    int cached_prefix_tokens(int key) const;
    int blocks_needed_to_admit_cached(int key, int shared_tokens, int prompt_tokens) const;
    bool admit_with_cached_prefix(RequestId r, int key, int shared_tokens, int prompt_tokens);
    // Blocks referenced only by the cache; with `key`, the first `shared_blocks` blocks of that entry are
    // left out (a request about to share them keeps them alive).
    int evictable_blocks(int key = -1, int shared_blocks = 0) const;
    int shared_blocks_with_cached(int key, int shared_tokens, int prompt_tokens) const;
    int available_blocks() const { return free_blocks() + evictable_blocks(); }
    void clear_cache();

    // "" when every invariant holds (table lengths, refcounts, cache contents, stats), else a description.
    std::string validate() const;
    // When on, every mutating call validates and throws std::logic_error on a violation.  Default: on in
    // builds without NDEBUG.
    void set_check_each_op(bool on) { check_each_op_ = on; }
    // Calls so far that created, changed or removed a block table (admissions, forks, appends, frees): a caller
    // mirroring tables elsewhere (the decode-step runtime's staged rows) can tell whether any table changed since
    // it last looked.  Not part of the reference's interface.
    uint64_t table_changes() const { return table_changes_; }

private:
    struct PrefixEntry {
        std::vector<BlockId> blocks;  // completely filled blocks, in token order
        int tokens = 0;               // blocks.size() * block_size
        int64_t stamp = 0;            // logical time of the last use (LRU order)
    };
    using CacheMap = std::map<int, PrefixEntry>;

    void checkpoint() const;
    void drop_ref(BlockId b);
    BlockId take_block(int fill);
    bool make_room(int blocks);
    void evict(CacheMap::iterator it);
    std::unordered_map<BlockId, int> cache_holds() const;
    int cache_only_blocks() const;
    bool admit_shared(RequestId r, const std::vector<BlockId>& shared, int prompt_tokens);

    int block_size_;
    BlockAllocator pool_;
    std::map<RequestId, BlockTable> requests_;
    CacheMap cache_;
    std::vector<int> fill_;       // filled slots of each physical block (0 while free)
    int64_t filled_slots_ = 0;    // sum of fill_
    int64_t table_entries_ = 0;   // sum of table lengths
    int64_t cow_events_ = 0;
    int64_t evictions_ = 0;
    int64_t clock_ = 0;
    uint64_t table_changes_ = 0;
#ifdef NDEBUG
    bool check_each_op_ = false;
#else
    bool check_each_op_ = true;
#endif
};

}  // namespace kvp
