// Host-buffer attention with the parameter list of the reference's CPU entry points (reference_attention /
// paged_attention_cpu, include/kvpage/paged_attention.h:25-35 of prathameshpranjale/paged-kv-cache-manager):
// the inputs are copied to the current device, attended by the fp32 CUDA-core kernel and the outputs copied
// back.  The reference's argument checks (src/paged_attention.cpp:12-17, 72) come first, with its messages.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "kvp_b200.h"
#include "kvp_internal.h"

namespace {

// Device buffers of one call, freed on every path out.
struct DeviceBuffers {
    void* p[7] = {};
    cudaStream_t stream = nullptr;
    ~DeviceBuffers() {
        if (stream) cudaStreamSynchronize(stream);
        for (void* x : p)
            if (x) cudaFree(x);
        if (stream) cudaStreamDestroy(stream);
    }
};

}  // namespace

extern "C" KVP_API int kvp_paged_attention_host(int32_t num_heads, int32_t kv_heads, int32_t head_dim,
                                                int32_t block_size, int32_t num_seqs, int32_t max_blocks,
                                                const float* q, const float* k_cache, const float* v_cache,
                                                const int32_t* block_tables, const int32_t* seq_lens, float* out,
                                                int32_t partitions) {
    using namespace kvpi;
    clear_error();
    if (kv_heads <= 0 || num_heads % kv_heads != 0) return fail(KVP_EINVAL, "num_heads % kv_heads != 0");
    if (num_seqs < 0 || block_size < 1 || max_blocks < 0) return fail(KVP_EINVAL, "bad num_seqs / block_size / max_blocks");
    if (num_seqs > 0 && (!seq_lens || !block_tables || !q || !k_cache || !v_cache || !out))
        return fail(KVP_EINVAL, "null buffer");
    for (int i = 0; i < num_seqs; ++i)
        if (seq_lens[i] < 1 || (static_cast<long long>(seq_lens[i]) + block_size - 1) / block_size > max_blocks)
            return fail(KVP_EINVAL, "bad seq_len");
    if (partitions < 1) return fail(KVP_EINVAL, "partitions < 1");
    if (num_seqs == 0) return KVP_OK;
    // The pool's extent is not part of the reference's parameter list: read the blocks up to the largest id any
    // sequence's table uses (entries past a sequence are never read).
    long long top = -1;
    for (int i = 0; i < num_seqs; ++i) {
        const int nb = (seq_lens[i] + block_size - 1) / block_size;
        const int32_t* row = block_tables + static_cast<size_t>(i) * max_blocks;
        for (int j = 0; j < nb; ++j) {
            if (row[j] < 0) return fail(KVP_EBOUNDS, "negative block id in the table of sequence " + std::to_string(i));
            top = std::max<long long>(top, row[j]);
        }
    }
    const long long pool_blocks = top + 1;
    const size_t row_elems = static_cast<size_t>(block_size) * kv_heads * head_dim;
    const size_t qo = static_cast<size_t>(num_seqs) * num_heads * head_dim * sizeof(float);
    const size_t kv = static_cast<size_t>(pool_blocks) * row_elems * sizeof(float);
    const size_t tb = static_cast<size_t>(num_seqs) * max_blocks * sizeof(int32_t);
    const size_t lb = static_cast<size_t>(num_seqs) * sizeof(int32_t);
    DeviceBuffers d;
    cudaError_t e = cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking);
    const size_t sizes[7] = {qo, kv, kv, tb, lb, qo, sizeof(int32_t)};
    for (int i = 0; i < 7 && e == cudaSuccess; ++i) e = cudaMalloc(&d.p[i], sizes[i]);
    if (e != cudaSuccess) return cuda_status(e, "device buffers for the host-buffer attention");
    const void* src[5] = {q, k_cache, v_cache, block_tables, seq_lens};
    for (int i = 0; i < 5 && e == cudaSuccess; ++i)
        e = cudaMemcpyAsync(d.p[i], src[i], sizes[i], cudaMemcpyHostToDevice, d.stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(d.p[6], 0, sizeof(int32_t), d.stream);
    if (e != cudaSuccess) return cuda_status(e, "copy-in of the host-buffer attention");
    kvp_attn_args a;
    std::memset(&a, 0, sizeof(a));
    a.q = d.p[0];
    a.q_dtype = KVP_DTYPE_F32;
    a.k_cache = d.p[1];
    a.v_cache = d.p[2];
    a.kv_dtype = KVP_DTYPE_F32;
    a.num_blocks = pool_blocks;
    a.block_tables = static_cast<const int32_t*>(d.p[3]);
    a.seq_lens = static_cast<const int32_t*>(d.p[4]);
    a.out = d.p[5];
    a.out_dtype = KVP_DTYPE_F32;
    a.num_seqs = num_seqs;
    a.num_heads = num_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.block_size = block_size;
    a.max_blocks = max_blocks;
    a.status = static_cast<int32_t*>(d.p[6]);
    int rc = kvp_paged_attention(&a, d.stream);
    if (rc != KVP_OK) return rc;
    int32_t status = 0;
    e = cudaMemcpyAsync(out, d.p[5], qo, cudaMemcpyDeviceToHost, d.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, d.p[6], sizeof(status), cudaMemcpyDeviceToHost, d.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess) return cuda_status(e, "host-buffer attention");
    if (status != 0) return fail(KVP_ECUDA, "attention kernel reported status " + std::to_string(status));
    return KVP_OK;
}
