// Logical-to-physical map of one request (reference include/kvpage/block_table.h:10-13).
#pragma once
#include <vector>

#include "kvpage/types.h"

namespace kvp {

// blocks[i] holds tokens [i*B, (i+1)*B) of the request; blocks.size() == ceil(tokens / B) always.
struct BlockTable {
    std::vector<BlockId> blocks;
    int tokens = 0;
};

}  // namespace kvp
