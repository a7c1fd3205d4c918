// C++ entry points of the device attention path; all forward to the C ABI.
//   kvp::paged_attention  -- device form of the reference's paged_attention entry points
//                            (include/kvpage/paged_attention.h:25-35 of the reference)
//   kvp::reference_attention / kvp::paged_attention_cpu -- the reference's host-buffer signatures, on the
//                            device path (kvp_paged_attention_host)
//   launch_paged_attention -- same signature and error behaviour as the reference's GPU entry point
//                            (cuda/paged_attention.cuh:16-19, cuda/paged_attention.cu:100-115)
#include "kvpage/paged_attention.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "kvp_b200.h"
#include "paged_attention.cuh"

namespace kvp {

void paged_attention(const AttnShape& s, int num_seqs, int max_blocks, const void* q, DType q_dtype,
                     const void* k_cache, const void* v_cache, DType kv_dtype, int64_t num_blocks,
                     const int32_t* block_tables, const int32_t* seq_lens, void* out, DType out_dtype,
                     void* workspace, size_t workspace_bytes, void* stream) {
    kvp_attn_args a{};
    a.q = q;
    a.q_dtype = static_cast<int32_t>(q_dtype);
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.kv_dtype = static_cast<int32_t>(kv_dtype);
    a.num_blocks = num_blocks;
    a.block_tables = block_tables;
    a.seq_lens = seq_lens;
    a.out = out;
    a.out_dtype = static_cast<int32_t>(out_dtype);
    a.num_seqs = num_seqs;
    a.num_heads = s.num_heads;
    a.kv_heads = s.kv_heads;
    a.head_dim = s.head_dim;
    a.block_size = s.block_size;
    a.max_blocks = max_blocks;
    a.split_tiles = workspace ? 0 : -1;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    const int rc = kvp_paged_attention(&a, stream);
    if (rc == KVP_EINVAL || rc == KVP_ENOSPACE) throw std::invalid_argument(kvp_last_error());
    if (rc != KVP_OK) throw std::runtime_error(kvp_last_error());
}

namespace {

void host_attention(const AttnShape& s, int num_seqs, int max_blocks, const float* q, const float* k_cache,
                    const float* v_cache, const int32_t* block_tables, const int32_t* seq_lens, float* out,
                    int partitions) {
    const int rc = kvp_paged_attention_host(s.num_heads, s.kv_heads, s.head_dim, s.block_size, num_seqs, max_blocks,
                                            q, k_cache, v_cache, block_tables, seq_lens, out, partitions);
    if (rc == KVP_EINVAL || rc == KVP_EBOUNDS) throw std::invalid_argument(kvp_last_error());
    if (rc != KVP_OK) throw std::runtime_error(kvp_last_error());
}

}  // namespace

void reference_attention(const AttnShape& s, int num_seqs, int max_blocks, const float* q, const float* k_cache,
                         const float* v_cache, const int32_t* block_tables, const int32_t* seq_lens, float* out) {
    host_attention(s, num_seqs, max_blocks, q, k_cache, v_cache, block_tables, seq_lens, out, 1);
}

void paged_attention_cpu(const AttnShape& s, int num_seqs, int max_blocks, const float* q, const float* k_cache,
                         const float* v_cache, const int32_t* block_tables, const int32_t* seq_lens, float* out,
                         int partitions) {
    host_attention(s, num_seqs, max_blocks, q, k_cache, v_cache, block_tables, seq_lens, out, partitions);
}

}  // namespace kvp

namespace {

// The drop-in entry point keeps its split partials in the library's no-allocation scratch, which all such
// calls on a device share.  The reference's entry point lets callers use any streams concurrently, so calls
// are ordered through one event per device: each call's stream waits for the previous call's launch (a wait
// on the same stream costs nothing).  Streams being captured skip the ordering; the graph's order applies.
struct DropInOrder {
    std::mutex mu;
    cudaEvent_t ev[64] = {};
};
DropInOrder& drop_in_order() {
    static DropInOrder o;
    return o;
}

}  // namespace

cudaError_t launch_paged_attention(const __half* q, const __half* k_cache, const __half* v_cache,
                                   const int* block_tables, const int* seq_lens, __half* out, int num_seqs,
                                   int num_heads, int kv_heads, int head_dim, int block_size, int max_blocks,
                                   int warps, cudaStream_t stream) {
    // Argument checks of the reference (cuda/paged_attention.cu:104-105, 112).
    if (warps < 1 || warps > 8 || kv_heads <= 0 || num_heads % kv_heads != 0 || num_seqs <= 0)
        return cudaErrorInvalidValue;
    if (!(head_dim == 32 || head_dim == 64 || head_dim == 96 || head_dim == 128 || head_dim == 256))
        return cudaErrorInvalidValue;
    kvp_attn_args a{};
    a.q = q;
    a.q_dtype = KVP_DTYPE_F16;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.kv_dtype = KVP_DTYPE_F16;
    a.num_blocks = 0;  // unknown pool size: unchecked, as in the reference
    a.block_tables = block_tables;
    a.seq_lens = seq_lens;
    a.out = out;
    a.out_dtype = KVP_DTYPE_F16;
    a.num_seqs = num_seqs;
    a.num_heads = num_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.block_size = block_size;
    a.max_blocks = max_blocks;
    a.split_tiles = 0;  // balanced schedule, partials in the library's scratch (this signature has no workspace)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    DropInOrder& o = drop_in_order();
    std::lock_guard<std::mutex> lock(o.mu);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool ordered = cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
    if (ordered) {
        if (!o.ev[dev]) e = cudaEventCreateWithFlags(&o.ev[dev], cudaEventDisableTiming);
        else e = cudaStreamWaitEvent(stream, o.ev[dev], 0);
        if (e != cudaSuccess) return e;
    }
    const int rc = kvp_paged_attention_noalloc(&a, stream);
    if (rc == KVP_OK && ordered) {
        e = cudaEventRecord(o.ev[dev], stream);
        if (e != cudaSuccess) return e;
    }
    if (rc == KVP_OK) return cudaSuccess;
    if (rc == KVP_ECUDA) {
        const cudaError_t e = cudaGetLastError();
        return e != cudaSuccess ? e : cudaErrorLaunchFailure;
    }
    return cudaErrorInvalidValue;
}
