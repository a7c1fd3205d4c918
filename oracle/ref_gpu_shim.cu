// C-ABI entry for the reference's own GPU kernel (cuda/paged_attention.cu of
// prathameshpranjale/paged-kv-cache-manager), compiled from its source by oracle/Makefile into
// _ref/libref_gpu_attention.so.  Test and baseline infrastructure only: the parity tests compare this
// library's attention with it, and bench.py's reference arm times it; the product never loads it.  Its C++
// launch_paged_attention stays hidden inside that .so, so it cannot clash with the drop-in of the same name.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "paged_attention.cuh"

extern "C" __attribute__((visibility("default"))) int ref_gpu_launch_paged_attention(
    const void* q, const void* k_cache, const void* v_cache, const int* block_tables, const int* seq_lens, void* out,
    int num_seqs, int num_heads, int kv_heads, int head_dim, int block_size, int max_blocks, int warps,
    void* stream) {
    return static_cast<int>(launch_paged_attention(
        static_cast<const __half*>(q), static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
        block_tables, seq_lens, static_cast<__half*>(out), num_seqs, num_heads, kv_heads, head_dim, block_size,
        max_blocks, warps, static_cast<cudaStream_t>(stream)));
}
