// Paged decode attention over fp32 K/V pools -- the reference's own float layout
// (include/kvpage/paged_attention.h:8-21 of prathameshpranjale/paged-kv-cache-manager) -- on CUDA cores in fp32
// arithmetic, so its results match the reference's paged_attention_cpu (src/paged_attention.cpp:68-114) to
// float rounding rather than to 16-bit storage.  The tensor-core kernel serves fp16/bf16 pools; this one is the
// device path of the host-buffer entry points (kvp_paged_attention_host) and of fp32 pools given to
// kvp_paged_attention.
//
// One CTA per (sequence, kv head): the g query heads of the group share every K/V row the CTA reads.  Warp w
// takes tokens w*TOK .. w*TOK+TOK-1, then the next nw*TOK, ... (TOK rows of K and V in flight per warp); lane l
// holds dims l, l+32, ... of the queries and of the running output, each score is a warp reduction, and each
// warp keeps an online softmax (m, l, acc) per query head in the log2 domain.  The warps' states are merged
// through shared memory at the end, one head at a time.
#include <cuda_runtime.h>

#include <cmath>

#include "attention_common.h"
#include "kvp_device.cuh"

namespace kvpd {

struct F32Params {
    const void* q;
    const float* k;
    const float* v;
    const int32_t* tables;
    const int32_t* lens;
    void* out;
    int32_t* status;
    long long num_blocks;  // 0: unchecked
    int q_dtype, out_dtype;
    int num_seqs, nh, kvh, g, B, max_blocks;
    float sl2;  // scale * log2(e)
};

constexpr int kF32Warps = 8;
constexpr int kF32Tok = 2;

template <int D, int G>
__global__ void __launch_bounds__(kF32Warps * 32) paged_decode_f32_kernel(const F32Params p) {
    constexpr int DPL = D / 32;  // dims per lane: lane holds dims i * 32 + lane
    __shared__ float merge[kF32Warps][D + 2];
    const int seq = blockIdx.x / p.kvh, head = blockIdx.x - seq * p.kvh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int len = p.lens[seq];
    const size_t out0 = (static_cast<size_t>(seq) * p.nh + static_cast<size_t>(head) * p.g) * D;
    if (len < 1 || (static_cast<long long>(len) + p.B - 1) / p.B > p.max_blocks) {
        if (threadIdx.x == 0 && head == 0) report(p.status, KVP_STATUS_BAD_LEN);
        for (int i = threadIdx.x; i < p.g * D; i += blockDim.x) store_any(p.out, out0 + i, p.out_dtype, 0.f);
        return;
    }
    float q[G][DPL], acc[G][DPL], m[G], l[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            acc[j][i] = 0.f;
            q[j][i] = j < p.g ? load_any(p.q, out0 + static_cast<size_t>(j) * D + i * 32 + lane, p.q_dtype) * p.sl2 : 0.f;
        }
    }
    const int32_t* trow = p.tables + static_cast<size_t>(seq) * p.max_blocks;
    for (int t0 = warp * kF32Tok; t0 < len; t0 += kF32Warps * kF32Tok) {
        float kr[kF32Tok][DPL], vr[kF32Tok][DPL];
#pragma unroll
        for (int u = 0; u < kF32Tok; ++u) {
            const int t = t0 + u;
            bool use = t < len;
            size_t row = 0;
            if (use) {
                const int blk = __ldg(trow + t / p.B);
                if (blk < 0 || (p.num_blocks > 0 && blk >= p.num_blocks)) {
                    if (lane == 0) report(p.status, KVP_STATUS_BAD_BLOCK);
                    use = false;  // read as zeros, as the tensor-core kernel's zero-filled tile would be
                } else {
                    row = ((static_cast<size_t>(blk) * p.B + t % p.B) * p.kvh + head) * D;
                }
            }
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
                kr[u][i] = use ? __ldg(p.k + row + i * 32 + lane) : 0.f;
                vr[u][i] = use ? __ldg(p.v + row + i * 32 + lane) : 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < kF32Tok; ++u) {
            if (t0 + u >= len) break;
#pragma unroll
            for (int j = 0; j < G; ++j) {
                if (j >= p.g) break;
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < DPL; ++i) s = fmaf(q[j][i], kr[u][i], s);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                const float mn = fmaxf(m[j], s);
                const float corr = exp2f(m[j] - mn);  // 0 on the first token (m = -inf)
                const float w = exp2f(s - mn);
                l[j] = l[j] * corr + w;
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[j][i] = fmaf(acc[j][i], corr, w * vr[u][i]);
                m[j] = mn;
            }
        }
    }
    // Merge the warps' states head by head; a warp that saw no token has m = -inf and contributes nothing.
#pragma unroll
    for (int j = 0; j < G; ++j) {
        if (j >= p.g) break;
#pragma unroll
        for (int i = 0; i < DPL; ++i) merge[warp][i * 32 + lane] = acc[j][i];
        if (lane == 0) {
            merge[warp][D] = m[j];
            merge[warp][D + 1] = l[j];
        }
        __syncthreads();
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            float M = -INFINITY;
            for (int w = 0; w < kF32Warps; ++w) M = fmaxf(M, merge[w][D]);
            float L = 0.f, o = 0.f;
            for (int w = 0; w < kF32Warps; ++w) {
                const float mw = merge[w][D];
                if (mw == -INFINITY) continue;
                const float c = exp2f(mw - M);
                L = fmaf(merge[w][D + 1], c, L);
                o = fmaf(merge[w][d], c, o);
            }
            store_any(p.out, out0 + static_cast<size_t>(j) * D + d, p.out_dtype, o / L);
        }
        __syncthreads();
    }
}

namespace {

template <int D>
int launch_d(const F32Params& prm, unsigned grid, cudaStream_t s) {
    if (prm.g <= 8) {
        paged_decode_f32_kernel<D, 8><<<grid, kF32Warps * 32, 0, s>>>(prm);
    } else {
        if constexpr (D <= 128) paged_decode_f32_kernel<D, 16><<<grid, kF32Warps * 32, 0, s>>>(prm);
        else return kvpi::fail(KVP_EINVAL, "head_dim 256 supports at most 8 query heads per kv head");
    }
    return kvpi::cuda_status(cudaGetLastError(), "fp32 attention kernel launch");
}

}  // namespace

}  // namespace kvpd

namespace kvpi {

int launch_attention_f32(const kvp_attn_args& a, cudaStream_t s) {
    const int D = a.head_dim;
    if (!(D == 32 || D == 64 || D == 96 || D == 128 || D == 256))
        return fail(KVP_EINVAL, "head_dim must be one of 32, 64, 96, 128, 256");
    if (a.kv_heads <= 0 || a.num_heads <= 0 || a.num_heads % a.kv_heads != 0)
        return fail(KVP_EINVAL, "num_heads % kv_heads != 0");
    const int g = a.num_heads / a.kv_heads;
    if (g > 16) return fail(KVP_EINVAL, "more than 16 query heads per kv head are not supported");
    if (g > 8 && D > 128) return fail(KVP_EINVAL, "head_dim 256 supports at most 8 query heads per kv head");
    if (a.block_size < 1 || a.max_blocks < 1 || a.num_seqs < 0) return fail(KVP_EINVAL, "bad block_size / max_blocks / num_seqs");
    if (a.k_new || a.v_new) return fail(KVP_EINVAL, "the fused append needs fp16 or bf16 pools");
    if (a.inputs_ready) return fail(KVP_EINVAL, "inputs_ready needs fp16 or bf16 pools");
    if ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 3u)
        return fail(KVP_EINVAL, "fp32 pools must be 4-byte aligned");
    if (static_cast<long long>(a.num_seqs) * a.kv_heads > 0x7fffffffLL) return fail(KVP_EINVAL, "too many sequences");
    if (a.num_seqs == 0) return KVP_OK;
    kvpd::F32Params prm;
    prm.q = a.q;
    prm.k = static_cast<const float*>(a.k_cache);
    prm.v = static_cast<const float*>(a.v_cache);
    prm.tables = a.block_tables;
    prm.lens = a.seq_lens;
    prm.out = a.out;
    prm.status = a.status;
    prm.num_blocks = a.num_blocks > 0 ? a.num_blocks : 0;
    prm.q_dtype = a.q_dtype;
    prm.out_dtype = a.out_dtype;
    prm.num_seqs = a.num_seqs;
    prm.nh = a.num_heads;
    prm.kvh = a.kv_heads;
    prm.g = g;
    prm.B = a.block_size;
    prm.max_blocks = a.max_blocks;
    const float scale = a.scale > 0.f ? a.scale : 1.0f / std::sqrt(static_cast<float>(D));
    prm.sl2 = scale * 1.4426950408889634f;
    const unsigned grid = static_cast<unsigned>(a.num_seqs * a.kv_heads);
    switch (D) {
        case 32: return kvpd::launch_d<32>(prm, grid, s);
        case 64: return kvpd::launch_d<64>(prm, grid, s);
        case 96: return kvpd::launch_d<96>(prm, grid, s);
        case 128: return kvpd::launch_d<128>(prm, grid, s);
        default: return kvpd::launch_d<256>(prm, grid, s);
    }
}

}  // namespace kvpi
