// Reference-counted pool of equally sized physical blocks (public API of the reference's
// include/kvpage/block_allocator.h:11-31).
#pragma once
#include <string>
#include <vector>

#include "kvpage/types.h"

namespace kvp {

// Free blocks are kept on a LIFO stack that starts as 0 on top, then 1, 2, ...: a fresh pool hands out the
// lowest ids first and a released block is the next one handed out.  Bad ids and retain/release of a free
// block throw std::logic_error; a negative pool size throws std::invalid_argument.
class KVPAGE_EXPORT BlockAllocator {
public:
    explicit BlockAllocator(int num_blocks);

    BlockId allocate();  // kNoBlock when the pool is empty; otherwise refcount becomes 1
    void retain(BlockId b);
    void release(BlockId b);  // back on the stack when the count reaches 0
    int refcount(BlockId b) const;
    int free_blocks() const { return static_cast<int>(stack_.size()); }
    int total_blocks() const { return static_cast<int>(count_.size()); }
    int referenced_blocks() const { return total_blocks() - free_blocks(); }

    // "" when the stack and the counts agree, else the first inconsistency found.
    std::string validate() const;

private:
    void require_valid(BlockId b) const;

    std::vector<int> count_;       // references per block
    std::vector<BlockId> stack_;   // free blocks; back() is handed out next
};

}  // namespace kvp
