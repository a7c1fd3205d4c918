// Decode attention over a paged KV cache -- the C++ entry point of this library.
//
// The reference declares its CPU implementations here (include/kvpage/paged_attention.h:8-35:
// AttnShape, reference_attention, paged_attention_cpu).  This library keeps AttnShape and the layout
// contract unchanged and provides the device implementation behind the same shape description; it runs
// only on the GPU (there is no CPU fallback) and forwards to the C ABI in kvp_b200.h.
//
// Layouts (row-major, contiguous), unchanged from the reference:
//   q, out        [num_seqs][num_heads][head_dim]
//   k_cache,
//   v_cache       [num_blocks][block_size][kv_heads][head_dim]
//   block_tables  [num_seqs][max_blocks]   int32 physical block ids; entries past a sequence are ignored
//   seq_lens      [num_seqs]               >= 1
// Query head h uses kv head h / (num_heads / kv_heads); scale = 1/sqrt(head_dim).
#pragma once
#include <cstddef>
#include <cstdint>

#include "kvpage/types.h"

namespace kvp {

struct AttnShape {
    int num_heads = 8;
    int kv_heads = 2;
    int head_dim = 64;
    int block_size = 16;
};

enum class DType : int32_t { F32 = 0, F16 = 1, BF16 = 2 };

// Device pointers throughout; asynchronous on `stream` (a cudaStream_t).  Throws std::invalid_argument
// for shapes the kernel does not support or that the reference rejects (num_heads % kv_heads != 0), and
// std::runtime_error when a CUDA call fails.  `workspace` (kvp_attention_workspace_size bytes) enables
// splitting long contexts across CTAs; pass nullptr to run one CTA per sequence.
KVPAGE_EXPORT void paged_attention(const AttnShape& s, int num_seqs, int max_blocks, const void* q, DType q_dtype,
                     const void* k_cache, const void* v_cache, DType kv_dtype, int64_t num_blocks,
                     const int32_t* block_tables, const int32_t* seq_lens, void* out, DType out_dtype,
                     void* workspace = nullptr, size_t workspace_bytes = 0, void* stream = nullptr);

// The reference's two entry points with their exact parameter lists (include/kvpage/paged_attention.h:25-35 of
// the reference), so its callers -- tests/test_attention.cpp, python/kvpage_py.cpp -- link unchanged.  Host
// buffers, fp32 throughout; both run the same device path (kvp_paged_attention_host: copy in, the fp32
// CUDA-core kernel, copy out) and return once `out` is written.  The reference's checks throw
// std::invalid_argument with its messages ("num_heads % kv_heads != 0", "bad seq_len", "partitions < 1"), as
// does a negative block id; a CUDA failure throws std::runtime_error.  `partitions` is checked (>= 1) but does
// not change the result beyond float rounding: the kernel splits the context its own way.
KVPAGE_EXPORT void reference_attention(const AttnShape& s, int num_seqs, int max_blocks, const float* q,
                                       const float* k_cache, const float* v_cache, const int32_t* block_tables,
                                       const int32_t* seq_lens, float* out);
KVPAGE_EXPORT void paged_attention_cpu(const AttnShape& s, int num_seqs, int max_blocks, const float* q,
                                       const float* k_cache, const float* v_cache, const int32_t* block_tables,
                                       const int32_t* seq_lens, float* out, int partitions);

}  // namespace kvp
