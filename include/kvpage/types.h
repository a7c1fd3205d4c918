// Core ids of the kvpage API.  Same names and meanings as the reference's include/kvpage/types.h:6-11,
// so code written against the reference compiles unchanged against this library.
#pragma once
#include <cstdint>

// Marks the C++ API exported by libkvpage_b200.so (the library is built with hidden default visibility).
#if defined(__GNUC__)
#define KVPAGE_EXPORT __attribute__((visibility("default")))
#else
#define KVPAGE_EXPORT
#endif

namespace kvp {

using BlockId = int32_t;    // physical block index inside one pool
using RequestId = int64_t;  // caller-chosen request handle
constexpr BlockId kNoBlock = -1;
constexpr RequestId kNoRequest = -1;

// Number of b-sized blocks needed to hold a items (a >= 0, b > 0).
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace kvp
