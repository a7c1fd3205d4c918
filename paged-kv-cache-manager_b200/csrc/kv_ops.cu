// Device data plane of the KVManager decisions: append scatter, copy-on-write block copies, swap, and block
// migration between shards.
//
// All are pure byte movement: HBM-bound (swap: host-link bound; migration from a peer GPU: NVLink-bound).  Copies use 16-byte vectors with
// several loads in flight per thread; grids are sized in multiples of the SM count.  Results are bit-exact
// copies, as in the reference's Python data plane (python/paged_model.py:54-55, 92-95, 113-117, 145-146).
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "kvp_device.cuh"
#include "kvp_internal.h"

namespace kvpd {

// ---------------------------------------------------------------- append scatter
// A group of 2^lpr_shift lanes copies one token row (kv_heads * head_dim elements, row_u 16-byte units) of K
// and of V for one (layer, sequence): the slot is loaded once per row, every lane keeps up to U units of K and
// U of V in flight before it stores them, and no index needs an integer division.  Grid: x strides over row
// groups, y over layers.  Rows are copied whole, so for a decode step (one row per sequence, 2 KB at the
// Llama-3-8B head shape) and for a prompt (consecutive positions: rows contiguous within a block) every store
// fills whole 128-byte lines.
struct AppendParams {
    const uint4* k_new;
    const uint4* v_new;
    uint4* k_cache;
    uint4* v_cache;
    const int32_t* slots;
    int32_t* status;
    long long layer_stride_u;  // 16-byte units between layer pools
    long long num_slots;       // num_blocks * block_size (0: unchecked)
    int num_layers, num_seqs, row_u;  // row_u: 16-byte units per token row
    int lpr_shift;                    // log2(lanes per row), at most 5
};

template <int U>
__global__ void __launch_bounds__(256) append_scatter_kernel(const AppendParams p) {
    const int lane = threadIdx.x & 31;
    const int lpr = 1 << p.lpr_shift;
    const int el = lane & (lpr - 1);
    const int rows_per_warp = 32 >> p.lpr_shift;
    const int warps = blockDim.x >> 5;
    const int first = (blockIdx.x * warps + (threadIdx.x >> 5)) * rows_per_warp + (lane >> p.lpr_shift);
    const int stride = gridDim.x * warps * rows_per_warp;
    for (int layer = blockIdx.y; layer < p.num_layers; layer += gridDim.y) {
        const long long src_layer = static_cast<long long>(layer) * p.num_seqs * p.row_u;
        const long long dst_layer = static_cast<long long>(layer) * p.layer_stride_u;
        for (int seq = first; seq < p.num_seqs; seq += stride) {
            const int slot = __ldg(p.slots + seq);
            if (slot < 0) continue;
            if (p.num_slots > 0 && slot >= p.num_slots) {
                if (el == 0 && layer == 0) report(p.status, KVP_STATUS_BAD_BLOCK);
                continue;
            }
            const uint4* ks = p.k_new + src_layer + static_cast<long long>(seq) * p.row_u;
            const uint4* vs = p.v_new + src_layer + static_cast<long long>(seq) * p.row_u;
            uint4* kd = p.k_cache + dst_layer + static_cast<long long>(slot) * p.row_u;
            uint4* vd = p.v_cache + dst_layer + static_cast<long long>(slot) * p.row_u;
            for (int e0 = el; e0 < p.row_u; e0 += lpr * U) {
                uint4 kb[U], vb[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int e = e0 + k * lpr;
                    if (e < p.row_u) {
                        kb[k] = __ldcs(ks + e);  // read once: do not keep the new rows in L2
                        vb[k] = __ldcs(vs + e);
                    }
                }
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int e = e0 + k * lpr;
                    if (e < p.row_u) {
                        kd[e] = kb[k];  // default policy: the attention that follows may find the row in L2
                        vd[e] = vb[k];
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------- whole-block copies
// Copy-on-write (source and destination pools the same) and migration between two shards' pools (the
// source possibly on a peer GPU, read with plain loads over NVLink).  Work item = (pair, layer, K|V): copies
// block_u 16-byte units.  Each thread moves UNROLL units per round so several loads are in flight before
// the stores (more for peer reads, whose latency is higher).
struct BlockCopyParams {
    const uint4* src_k;
    const uint4* src_v;
    uint4* dst_k;
    uint4* dst_v;
    const int32_t* pairs;
    int32_t* status;
    long long src_layer_u, dst_layer_u;  // 16-byte units between layer pools
    long long src_blocks, dst_blocks;    // 0: unchecked
    int n_pairs, num_layers, block_u;
};

template <int UNROLL>
__global__ void __launch_bounds__(256) block_copy_kernel(const BlockCopyParams p) {
    const long long items = static_cast<long long>(p.n_pairs) * p.num_layers * 2;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
        const int kv = static_cast<int>(it & 1);
        const long long pl = it >> 1;
        const int pair = static_cast<int>(pl / p.num_layers);
        const int layer = static_cast<int>(pl - static_cast<long long>(pair) * p.num_layers);
        const int src = __ldg(p.pairs + 2 * pair), dst = __ldg(p.pairs + 2 * pair + 1);
        if (src < 0 || dst < 0 || (p.src_blocks > 0 && src >= p.src_blocks) || (p.dst_blocks > 0 && dst >= p.dst_blocks)) {
            if (threadIdx.x == 0 && layer == 0 && kv == 0) report(p.status, KVP_STATUS_BAD_BLOCK);
            continue;
        }
        const uint4* s = (kv ? p.src_v : p.src_k) + layer * p.src_layer_u + static_cast<long long>(src) * p.block_u;
        uint4* d = (kv ? p.dst_v : p.dst_k) + layer * p.dst_layer_u + static_cast<long long>(dst) * p.block_u;
        for (int u0 = threadIdx.x; u0 < p.block_u; u0 += blockDim.x * UNROLL) {
            uint4 buf[UNROLL];
#pragma unroll
            for (int k = 0; k < UNROLL; ++k) {
                const int u = u0 + k * blockDim.x;
                if (u < p.block_u) buf[k] = s[u];
            }
#pragma unroll
            for (int k = 0; k < UNROLL; ++k) {
                const int u = u0 + k * blockDim.x;
                if (u < p.block_u) d[u] = buf[k];
            }
        }
    }
}

}  // namespace kvpd

namespace kvpi {
namespace {

long long resolve_layer_stride(long long given, long long num_blocks, int block_size, int kvh, int D) {
    return given > 0 ? given : num_blocks * block_size * kvh * static_cast<long long>(D);
}

}  // namespace
}  // namespace kvpi

extern "C" KVP_API int kvp_append_scatter(const kvp_append_args* a, void* stream) {
    using namespace kvpi;
    clear_error();
    if (!a) return fail(KVP_EINVAL, "null arguments");
    if (!(a->kv_dtype == KVP_DTYPE_F16 || a->kv_dtype == KVP_DTYPE_BF16))
        return fail(KVP_EINVAL, "pool dtype must be fp16 or bf16");
    if (a->num_layers < 0 || a->num_seqs < 0 || a->kv_heads < 1 || a->head_dim < 1 || a->block_size < 1 ||
        a->num_blocks < 0)
        return fail(KVP_EINVAL, "bad shape");
    const long long row_bytes = static_cast<long long>(a->kv_heads) * a->head_dim * 2;
    if (row_bytes % 16 != 0) return fail(KVP_EINVAL, "kv_heads * head_dim * 2 must be a multiple of 16 bytes");
    if (a->num_layers == 0 || a->num_seqs == 0) return KVP_OK;
    if (!a->k_new || !a->v_new || !a->k_cache || !a->v_cache || !a->slots) return fail(KVP_EINVAL, "null buffer");
    if (!aligned16(a->k_new) || !aligned16(a->v_new) || !aligned16(a->k_cache) || !aligned16(a->v_cache))
        return fail(KVP_EINVAL, "buffers must be 16-byte aligned");
    const long long ls = resolve_layer_stride(a->layer_stride, a->num_blocks, a->block_size, a->kv_heads, a->head_dim);
    if ((ls * 2) % 16 != 0) return fail(KVP_EINVAL, "layer stride must be a multiple of 16 bytes");
    if (a->num_layers > 1 && ls <= 0) return fail(KVP_EINVAL, "layer_stride or num_blocks required for several layers");
    kvpd::AppendParams p;
    p.k_new = static_cast<const uint4*>(a->k_new);
    p.v_new = static_cast<const uint4*>(a->v_new);
    p.k_cache = static_cast<uint4*>(a->k_cache);
    p.v_cache = static_cast<uint4*>(a->v_cache);
    p.slots = a->slots;
    p.status = a->status;
    p.layer_stride_u = ls * 2 / 16;
    p.num_slots = a->num_blocks * static_cast<long long>(a->block_size);
    p.num_layers = a->num_layers;
    p.num_seqs = a->num_seqs;
    p.row_u = static_cast<int>(row_bytes / 16);
    // lanes per row: the largest power of two <= min(32, row_u)
    p.lpr_shift = 0;
    while (p.lpr_shift < 5 && (2 << p.lpr_shift) <= p.row_u) ++p.lpr_shift;
    const int threads = 256, rows_per_block = (threads / 32) * (32 >> p.lpr_shift);
    const int gy = std::min(a->num_layers, 65535);
    const long long want_x = (static_cast<long long>(a->num_seqs) + rows_per_block - 1) / rows_per_block;
    const long long cap_x = std::max<long long>(1, (static_cast<long long>(sm_count()) * 32 + gy - 1) / gy);
    const dim3 grid(static_cast<unsigned>(std::min(want_x, cap_x)), static_cast<unsigned>(gy));
    kvpd::append_scatter_kernel<4><<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return cuda_status(cudaGetLastError(), "append scatter launch");
}

extern "C" KVP_API int kvp_cow_copy(const kvp_cow_args* a, void* stream) {
    using namespace kvpi;
    clear_error();
    if (!a) return fail(KVP_EINVAL, "null arguments");
    if (!(a->kv_dtype == KVP_DTYPE_F16 || a->kv_dtype == KVP_DTYPE_BF16))
        return fail(KVP_EINVAL, "pool dtype must be fp16 or bf16");
    if (a->n_pairs < 0 || a->num_layers < 0 || a->kv_heads < 1 || a->head_dim < 1 || a->block_size < 1 ||
        a->num_blocks < 0)
        return fail(KVP_EINVAL, "bad shape");
    const long long block_bytes = static_cast<long long>(a->block_size) * a->kv_heads * a->head_dim * 2;
    if (block_bytes % 16 != 0) return fail(KVP_EINVAL, "block bytes must be a multiple of 16");
    if (a->n_pairs == 0 || a->num_layers == 0) return KVP_OK;
    if (!a->k_cache || !a->v_cache || !a->pairs) return fail(KVP_EINVAL, "null buffer");
    if (!aligned16(a->k_cache) || !aligned16(a->v_cache)) return fail(KVP_EINVAL, "pools must be 16-byte aligned");
    const long long ls = resolve_layer_stride(a->layer_stride, a->num_blocks, a->block_size, a->kv_heads, a->head_dim);
    if ((ls * 2) % 16 != 0) return fail(KVP_EINVAL, "layer stride must be a multiple of 16 bytes");
    if (a->num_layers > 1 && ls <= 0) return fail(KVP_EINVAL, "layer_stride or num_blocks required for several layers");
    kvpd::BlockCopyParams p;
    p.src_k = static_cast<const uint4*>(a->k_cache);
    p.src_v = static_cast<const uint4*>(a->v_cache);
    p.dst_k = static_cast<uint4*>(a->k_cache);
    p.dst_v = static_cast<uint4*>(a->v_cache);
    p.pairs = a->pairs;
    p.status = a->status;
    p.src_layer_u = p.dst_layer_u = ls * 2 / 16;
    p.src_blocks = p.dst_blocks = a->num_blocks;
    p.n_pairs = a->n_pairs;
    p.num_layers = a->num_layers;
    p.block_u = static_cast<int>(block_bytes / 16);
    const long long items = static_cast<long long>(a->n_pairs) * a->num_layers * 2;
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(items, static_cast<long long>(sm_count()) * 8)));
    kvpd::block_copy_kernel<4><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return cuda_status(cudaGetLastError(), "copy-on-write launch");
}

// ---------------------------------------------------------------- migration between shards
namespace {

// Device of a device-memory pointer, or -1 (host / unregistered memory).
int device_of(const void* ptr) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return at.type == cudaMemoryTypeDevice ? at.device : -1;
}

}  // namespace

extern "C" KVP_API int kvp_enable_peer_access(int32_t peer_device) {
    using namespace kvpi;
    clear_error();
    int cur = 0, n = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess) e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_status(e, "device query");
    if (peer_device < 0 || peer_device >= n) return fail(KVP_EINVAL, "peer device out of range");
    if (peer_device == cur) return KVP_OK;
    int can = 0;
    e = cudaDeviceCanAccessPeer(&can, cur, peer_device);
    if (e != cudaSuccess) return cuda_status(e, "peer access query");
    if (!can) return fail(KVP_EINVAL, "device " + std::to_string(cur) + " cannot access device " + std::to_string(peer_device));
    e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return KVP_OK;
    }
    return cuda_status(e, "enable peer access");
}

extern "C" KVP_API int kvp_migrate_blocks(const kvp_migrate_args* a, void* stream) {
    using namespace kvpi;
    clear_error();
    if (!a) return fail(KVP_EINVAL, "null arguments");
    if (!(a->kv_dtype == KVP_DTYPE_F16 || a->kv_dtype == KVP_DTYPE_BF16))
        return fail(KVP_EINVAL, "pool dtype must be fp16 or bf16");
    if (a->n_pairs < 0 || a->num_layers < 0 || a->kv_heads < 1 || a->head_dim < 1 || a->block_size < 1 ||
        a->src_num_blocks < 0 || a->dst_num_blocks < 0)
        return fail(KVP_EINVAL, "bad shape");
    const long long block_bytes = static_cast<long long>(a->block_size) * a->kv_heads * a->head_dim * 2;
    if (block_bytes % 16 != 0) return fail(KVP_EINVAL, "block bytes must be a multiple of 16");
    if (a->n_pairs == 0 || a->num_layers == 0) return KVP_OK;
    if (!a->src_k_cache || !a->src_v_cache || !a->dst_k_cache || !a->dst_v_cache || !a->pairs)
        return fail(KVP_EINVAL, "null buffer");
    if (!aligned16(a->src_k_cache) || !aligned16(a->src_v_cache) || !aligned16(a->dst_k_cache) || !aligned16(a->dst_v_cache))
        return fail(KVP_EINVAL, "pools must be 16-byte aligned");
    const long long sls = resolve_layer_stride(a->src_layer_stride, a->src_num_blocks, a->block_size, a->kv_heads, a->head_dim);
    const long long dls = resolve_layer_stride(a->dst_layer_stride, a->dst_num_blocks, a->block_size, a->kv_heads, a->head_dim);
    if ((sls * 2) % 16 != 0 || (dls * 2) % 16 != 0) return fail(KVP_EINVAL, "layer strides must be multiples of 16 bytes");
    if (a->num_layers > 1 && (sls <= 0 || dls <= 0))
        return fail(KVP_EINVAL, "layer strides or pool sizes required for several layers");
    int cur = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_status(e, "device query");
    const int sdev = device_of(a->src_k_cache), ddev = device_of(a->dst_k_cache);
    if (sdev < 0 || ddev < 0 || device_of(a->src_v_cache) != sdev || device_of(a->dst_v_cache) != ddev)
        return fail(KVP_EINVAL, "pools must be device memory (K and V of one shard on one device)");
    if (ddev != cur) return fail(KVP_EINVAL, "launch on the destination pools' device");
    if (sdev != cur) {
        const int rc = kvp_enable_peer_access(sdev);
        if (rc != KVP_OK) return rc;
    }
    kvpd::BlockCopyParams p;
    p.src_k = static_cast<const uint4*>(a->src_k_cache);
    p.src_v = static_cast<const uint4*>(a->src_v_cache);
    p.dst_k = static_cast<uint4*>(a->dst_k_cache);
    p.dst_v = static_cast<uint4*>(a->dst_v_cache);
    p.pairs = a->pairs;
    p.status = a->status;
    p.src_layer_u = sls * 2 / 16;
    p.dst_layer_u = dls * 2 / 16;
    p.src_blocks = a->src_num_blocks;
    p.dst_blocks = a->dst_num_blocks;
    p.n_pairs = a->n_pairs;
    p.num_layers = a->num_layers;
    p.block_u = static_cast<int>(block_bytes / 16);
    const long long items = static_cast<long long>(a->n_pairs) * a->num_layers * 2;
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(items, static_cast<long long>(sm_count()) * 8)));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (sdev != cur)
        kvpd::block_copy_kernel<8><<<grid, 256, 0, s>>>(p);
    else
        kvpd::block_copy_kernel<4><<<grid, 256, 0, s>>>(p);
    return cuda_status(cudaGetLastError(), "migration launch");
}

// ---------------------------------------------------------------- swap (host link)
namespace {

// One cudaMemcpy2DAsync per (block, K|V): rows = layers, width = block bytes, device pitch = layer stride,
// host pitch = block bytes (the slot layout keeps one layer's block after another).
int swap_copy(const kvp_swap_args* a, void* stream, bool out) {
    using namespace kvpi;
    clear_error();
    if (!a) return fail(KVP_EINVAL, "null arguments");
    if (!(a->kv_dtype == KVP_DTYPE_F16 || a->kv_dtype == KVP_DTYPE_BF16))
        return fail(KVP_EINVAL, "pool dtype must be fp16 or bf16");
    if (a->n < 0 || a->num_layers < 1 || a->kv_heads < 1 || a->head_dim < 1 || a->block_size < 1 || a->num_blocks < 0)
        return fail(KVP_EINVAL, "bad shape");
    if (a->n == 0) return KVP_OK;
    if (!a->k_cache || !a->v_cache || !a->blocks || !a->host_slots || !a->host_pool) return fail(KVP_EINVAL, "null buffer");
    const size_t bb = static_cast<size_t>(a->block_size) * a->kv_heads * a->head_dim * 2;
    const long long ls = resolve_layer_stride(a->layer_stride, a->num_blocks, a->block_size, a->kv_heads, a->head_dim);
    if (a->num_layers > 1 && ls <= 0) return fail(KVP_EINVAL, "layer_stride or num_blocks required for several layers");
    const size_t pitch_dev = static_cast<size_t>(ls) * 2;
    const size_t slot_bytes = 2 * static_cast<size_t>(a->num_layers) * bb;
    for (int i = 0; i < a->n; ++i) {
        if (a->blocks[i] < 0 || (a->num_blocks > 0 && a->blocks[i] >= a->num_blocks) || a->host_slots[i] < 0 ||
            a->host_slots[i] >= a->host_pool_slots)
            return fail(KVP_EBOUNDS, "swap block id or host slot out of range at index " + std::to_string(i));
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < a->n; ++i) {
        const int blk = a->blocks[i];
        char* host = static_cast<char*>(a->host_pool) + static_cast<size_t>(a->host_slots[i]) * slot_bytes;
        for (int kv = 0; kv < 2; ++kv) {
            char* dev = static_cast<char*>(kv ? a->v_cache : a->k_cache) + static_cast<size_t>(blk) * bb;
            char* h = host + static_cast<size_t>(kv) * a->num_layers * bb;
            cudaError_t e = out ? cudaMemcpy2DAsync(h, bb, dev, pitch_dev, bb, static_cast<size_t>(a->num_layers),
                                                    cudaMemcpyDeviceToHost, s)
                                : cudaMemcpy2DAsync(dev, pitch_dev, h, bb, bb, static_cast<size_t>(a->num_layers),
                                                    cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_status(e, out ? "swap-out copy" : "swap-in copy");
        }
    }
    return KVP_OK;
}

}  // namespace

extern "C" KVP_API int kvp_swap_out(const kvp_swap_args* a, void* stream) { return swap_copy(a, stream, true); }
extern "C" KVP_API int kvp_swap_in(const kvp_swap_args* a, void* stream) { return swap_copy(a, stream, false); }
