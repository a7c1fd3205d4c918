// Reference-counted block pool.  Observable behaviour follows the reference's src/block_allocator.cpp:7-60:
// LIFO reuse with the lowest id handed out first from a fresh pool, std::logic_error on misuse.
#include "kvpage/block_allocator.h"

#include <stdexcept>

namespace kvp {

BlockAllocator::BlockAllocator(int num_blocks) {
    if (num_blocks < 0) throw std::invalid_argument("BlockAllocator: negative pool size");
    count_.resize(static_cast<size_t>(num_blocks), 0);
    stack_.resize(static_cast<size_t>(num_blocks));
    // back() is handed out first, so store the ids in descending order.
    for (int i = 0; i < num_blocks; ++i) stack_[static_cast<size_t>(i)] = num_blocks - 1 - i;
}

void BlockAllocator::require_valid(BlockId b) const {
    if (b < 0 || b >= total_blocks()) throw std::logic_error("BlockAllocator: block id " + std::to_string(b) + " outside the pool");
}

BlockId BlockAllocator::allocate() {
    if (stack_.empty()) return kNoBlock;
    const BlockId b = stack_.back();
    stack_.pop_back();
    count_[static_cast<size_t>(b)] = 1;
    return b;
}

void BlockAllocator::retain(BlockId b) {
    require_valid(b);
    int& c = count_[static_cast<size_t>(b)];
    if (c < 1) throw std::logic_error("BlockAllocator: retain of unallocated block " + std::to_string(b));
    c += 1;
}

void BlockAllocator::release(BlockId b) {
    require_valid(b);
    int& c = count_[static_cast<size_t>(b)];
    if (c < 1) throw std::logic_error("BlockAllocator: release of unallocated block " + std::to_string(b));
    c -= 1;
    if (c == 0) stack_.push_back(b);
}

int BlockAllocator::refcount(BlockId b) const {
    require_valid(b);
    return count_[static_cast<size_t>(b)];
}

std::string BlockAllocator::validate() const {
    const int n = total_blocks();
    std::vector<unsigned char> seen(static_cast<size_t>(n), 0);
    for (BlockId b : stack_) {
        if (b < 0 || b >= n) return "free stack holds id " + std::to_string(b) + " outside the pool";
        if (seen[static_cast<size_t>(b)]) return "block " + std::to_string(b) + " appears twice on the free stack";
        seen[static_cast<size_t>(b)] = 1;
        if (count_[static_cast<size_t>(b)] != 0) return "free block " + std::to_string(b) + " has a nonzero refcount";
    }
    int held = 0;
    for (int b = 0; b < n; ++b) {
        const int c = count_[static_cast<size_t>(b)];
        if (c < 0) return "block " + std::to_string(b) + " has a negative refcount";
        if (c == 0 && !seen[static_cast<size_t>(b)]) return "block " + std::to_string(b) + " is unreferenced but not free";
        held += c > 0;
    }
    if (held + free_blocks() != n) return "held + free blocks do not add up to the pool size";
    return std::string();
}

}  // namespace kvp
