// Paged decode attention kernels for sm_100a: flash-decoding over 16-token tiles of the context.
//
// Two schedules share the same tile pipeline:
//   * stream-K (default): a persistent grid of as many CTAs as fit on the GPU; the step's tiles (all
//     sequences, concatenated) are divided evenly between CTAs regardless of sequence boundaries, so every
//     CTA streams the same number of bytes with one pipeline ramp per launch.  A CTA's range is cut into
//     segments at sequence boundaries; a segment that covers a whole sequence is normalised and written
//     directly, the others leave (m, l, unnormalised O) partials, counted per sequence, and the CTA whose
//     count completes a sequence merges it in the same kernel.  With an early start (programmatic dependent
//     launch) the prologue -- and with an early load the first ring of K/V loads -- overlaps the previous
//     kernel on the stream.
//   * fixed splits: one CTA per (sequence, kv-head group, split of split_tiles tiles), partials merged by
//     merge_splits_kernel; split_tiles large enough means one CTA per sequence and no workspace at all (the
//     reference's signature).
//
// Tile pipeline (per CTA): a producer warp reads block ids from the sequence's table row (32 entries per
// coalesced load) and issues TMA tiled loads of the K and V rows of every kv head of the CTA's group into a
// ring of shared-memory stages (128B/64B swizzled; completion counted on an mbarrier); at the start of a
// segment it also bulk-copies the sequence's queries into a query slot and, with the fused append, first
// writes the sequence's newest K/V row.  One or two consumer warps per kv head compute, per tile,
//     S^T[16 tokens x 8 heads] = K_tile[16 x D] . Q^T[D x 8]      (mma.sync m16n8k16, fp32 accumulate)
// so the GQA group of query heads (up to 8 per n-tile) shares every K/V byte; an online softmax in the
// log2 domain with warp-shuffle reductions; then
//     O^T[D x 8] += V_tile^T[D x 16] . P^T[16 x 8]
// with P^T obtained from the S^T accumulator by movmatrix.  P (and a query in another dtype, QLO) are split
// into a 16-bit high part plus a 16-bit residual, so the result keeps close to fp32 accuracy.
//
// Numerics follow the reference's paged_attention_cpu (src/paged_attention.cpp:68-114): per-partition
// running (m, l, acc) with rescaling by exp(m_old - m_new), partitions merged by exp(m_p - M).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <type_traits>

#include "attention_common.h"
#include "kvp_device.cuh"

namespace kvpd {

// Block index of a token position: a shift for power-of-two block sizes (no integer division in the
// per-tile paths).
__device__ __forceinline__ int blk_of(const AttnParams& p, int tok) { return p.Bshift >= 0 ? tok >> p.Bshift : tok / p.B; }

// Sequence length in 16-token tiles, or 0 when the length is invalid (len < 1 or more blocks than a
// table row holds).
__device__ __forceinline__ int tiles_of_len(const AttnParams& p, int len) {
    const long long nblk = (static_cast<long long>(len) + p.B - 1) / p.B;
    if (len < 1 || nblk > p.max_blocks) return 0;
    return (len + 15) >> 4;
}

template <int D>
struct Geo {
    static constexpr int W = (D % 64 == 0) ? 64 : 32;  // elements per smem row
    static constexpr int ROWB = W * 2;                  // bytes per smem row
    static constexpr int NCH = D / W;
    static constexpr int KS = D / 16;                   // k-steps of the score MMA / m-tiles of the PV MMA
    static constexpr uint32_t SWM = (ROWB == 128) ? 7u : 3u;
};

// ---------------------------------------------------------------- producer: one tile into one stage
// All 32 lanes call this (the table cache is a warp-wide register array); lane 0 issues the copies.
template <int D>
__device__ __forceinline__ void produce_tile(const AttnParams& p, const CUtensorMap* km, const CUtensorMap* vm,
                                             uint32_t kst, uint32_t vst, uint32_t fb, int tb, int len,
                                             const int32_t* trow, int kvh0, int lane, int& cache_lo,
                                             int32_t& cached) {
    using G_ = Geo<D>;
    const int nr = min(p.nruns, (len - tb + p.R - 1) / p.R);
    if (lane == 0) mbar_arrive_expect_tx(fb, static_cast<uint32_t>(nr) * G_::NCH * 2u * p.box_tx);
    for (int j = 0; j < nr; ++j) {
        const int tok = tb + j * p.R;
        const int bi = blk_of(p, tok);
        if (bi < cache_lo || bi >= cache_lo + 32) {
            cache_lo = bi;
            cached = (bi + lane < p.max_blocks) ? __ldg(trow + bi + lane) : 0;
        }
        const int32_t blk = __shfl_sync(0xffffffffu, cached, bi - cache_lo);
        int row = blk * p.B + (tok - bi * p.B);
        if (p.num_blocks > 0 && (blk < 0 || blk >= p.num_blocks)) {
            if (lane == 0) report(p.status, KVP_STATUS_BAD_BLOCK);
            row = p.oob_row;
        }
        if (lane == 0) {
#pragma unroll
            for (int c = 0; c < G_::NCH; ++c) {
                const uint32_t off = static_cast<uint32_t>(j * G_::NCH + c) * p.box_slot;
                if (!p.per_head) {
                    tma_load_3d(kst + off, km, fb, c * G_::W, row, kvh0);
                    tma_load_3d(vst + off, vm, fb, c * G_::W, row, kvh0);
                } else {
                    for (int w = 0; w < p.kvh_cta; ++w) {
                        const uint32_t ho = off + static_cast<uint32_t>(w) * p.head_stride;
                        tma_load_3d(kst + ho, km, fb, c * G_::W, kvh0 + w, row);
                        tma_load_3d(vst + ho, vm, fb, c * G_::W, kvh0 + w, row);
                    }
                }
            }
        }
    }
}

// Fused append: the producer warp writes the newest token's K and V rows of the CTA's kv heads (position
// len - 1, one contiguous kvh_cta * D run per pool) before it issues the copies of the segment holding that
// position.  Each lane fences its stores against the async proxy and the warp synchronises, so the TMA loads
// issued afterwards by any lane see the new rows.  An out-of-range block id is skipped here (the tile load
// reports it and zero-fills).
template <int D>
__device__ __forceinline__ void append_new_token(const AttnParams& p, int seq, int len, const int32_t* trow, int kvh0,
                                                 int lane) {
    const int pos = len - 1;
    const int bi = blk_of(p, pos);
    const int32_t blk = __ldg(trow + bi);
    if (blk >= 0 && blk < p.num_blocks) {
        const size_t row = static_cast<size_t>(blk) * p.B + (pos - bi * p.B);
        const size_t src = (static_cast<size_t>(seq) * p.kvh + kvh0) * D / 8;  // 16-byte chunks
        const size_t dst = (row * p.kvh + kvh0) * D / 8;
        const uint4* ks = static_cast<const uint4*>(p.k_new) + src;
        const uint4* vs = static_cast<const uint4*>(p.v_new) + src;
        uint4* kd = static_cast<uint4*>(p.k_pool) + dst;
        uint4* vd = static_cast<uint4*>(p.v_pool) + dst;
        const int chunks = p.kvh_cta * D / 8;
        for (int c = lane; c < chunks; c += 32) {  // coherent loads: another stream's copy may have written them
            kd[c] = __ldcg(ks + c);
            vd[c] = __ldcg(vs + c);
        }
    }
    fence_proxy_async_global();
    __syncwarp();
}

// Up to 8 consecutive tiles of one sequence at once, lane k producing tile `tile + k` into stage
// (i + k) % S: each lane waits for its own stage, arms its own barrier and issues its own copies, so the
// per-tile issue cost is paid in parallel.  Only for one run per tile (block_size a multiple of 16).  The
// tile counter i is passed as (st0, r0) = (i % S, i / S); nb <= S.  Returns false (after reporting) if a wait
// gave up; `issued` is then the mask of the lanes that did issue their copies.
template <int D>
__device__ __forceinline__ bool produce_batch(const AttnParams& p, const CUtensorMap* km, const CUtensorMap* vm,
                                              uint32_t smem_base, uint64_t* full_bar, uint64_t* empty_bar, int st0,
                                              int r0, int tile, int nb, int len, const int32_t* trow, int kvh0,
                                              int lane, int& cache_lo, int32_t& cached, unsigned& issued) {
    using G_ = Geo<D>;
    const int S = p.stages;
    const int bi_first = blk_of(p, tile * 16);
    const int bi_last = blk_of(p, min((tile + nb) * 16, len) - 1);
    if (bi_first < cache_lo || bi_last >= cache_lo + 32) {
        cache_lo = bi_first;
        cached = (bi_first + lane < p.max_blocks) ? __ldg(trow + bi_first + lane) : 0;
    }
    const bool act = lane < nb;
    const int tok = (tile + (act ? lane : 0)) * 16;
    const int bi = blk_of(p, tok);
    const int32_t blk = __shfl_sync(0xffffffffu, cached, bi - cache_lo);
    bool ok = true;
    if (act) {
        int row = blk * p.B + (tok - bi * p.B);
        if (p.num_blocks > 0 && (blk < 0 || blk >= p.num_blocks)) {
            report(p.status, KVP_STATUS_BAD_BLOCK);
            row = p.oob_row;
        }
        int st = st0 + lane, r = r0;
        if (st >= S) {
            st -= S;
            ++r;
        }
        if (r >= 1 && !mbar_wait(smem_u32(&empty_bar[st]), static_cast<uint32_t>((r - 1) & 1), p.wait_limit)) {
            report(p.status, KVP_STATUS_TIMEOUT);
            ok = false;
        }
        if (ok) {
            const uint32_t fb = smem_u32(&full_bar[st]);
            const uint32_t kst = smem_base + static_cast<uint32_t>(st) * p.stage_bytes;
            const uint32_t vst = kst + p.stage_half;
            mbar_arrive_expect_tx(fb, static_cast<uint32_t>(G_::NCH) * 2u * p.box_tx);
#pragma unroll
            for (int c = 0; c < G_::NCH; ++c) {
                const uint32_t off = static_cast<uint32_t>(c) * p.box_slot;
                if (!p.per_head) {
                    tma_load_3d(kst + off, km, fb, c * G_::W, row, kvh0);
                    tma_load_3d(vst + off, vm, fb, c * G_::W, row, kvh0);
                } else {
                    for (int w = 0; w < p.kvh_cta; ++w) {
                        const uint32_t ho = off + static_cast<uint32_t>(w) * p.head_stride;
                        tma_load_3d(kst + ho, km, fb, c * G_::W, kvh0 + w, row);
                        tma_load_3d(vst + ho, vm, fb, c * G_::W, kvh0 + w, row);
                    }
                }
            }
        }
    }
    const unsigned failed = __ballot_sync(0xffffffffu, !ok);
    issued = ((nb >= 32 ? 0u : (1u << nb)) - 1u) & ~failed;
    return failed == 0;
}

// ---------------------------------------------------------------- consumer: one warp, one kv head
template <int D, int NT, class KV, bool QLO>
struct Consumer {
    using G_ = Geo<D>;
    using Tr = F16Traits<KV>;
    static constexpr int KS = G_::KS;
    uint32_t k_row_off, v_row_off, k_x, v_x;
    int k_doff, v_doff;
    uint32_t qhi[NT][KS][2], qlo[NT][KS][2];
    float o[NT][KS][4];
    float m_run[NT][2], l_run[NT][2];

    // Per-lane shared-memory geometry.  For ldmatrix matrix index jm = lane >> 3 and row rr = lane & 7:
    //   score operand (K, non-transposed): token (jm & 1) * 8 + rr, dim offset (jm >> 1) * 8
    //   PV operand    (V, transposed):     token (jm >> 1) * 8 + rr, dim offset (jm & 1) * 8
    __device__ __forceinline__ void init_geometry(const AttnParams& p, int warp, int lane) {
        const int jm = lane >> 3, rr = lane & 7;
        const int tk = (jm & 1) * 8 + rr;
        const int tv = (jm >> 1) * 8 + rr;
        const uint32_t hoff = static_cast<uint32_t>(warp) * p.head_stride;
        k_row_off = static_cast<uint32_t>(tk / p.R) * G_::NCH * p.box_slot + hoff + static_cast<uint32_t>(tk % p.R) * G_::ROWB;
        v_row_off = static_cast<uint32_t>(tv / p.R) * G_::NCH * p.box_slot + hoff + static_cast<uint32_t>(tv % p.R) * G_::ROWB;
        k_x = (k_row_off >> 7) & G_::SWM;  // swizzle phase of this row (box slots are 1024-byte aligned)
        v_x = (v_row_off >> 7) & G_::SWM;
        k_doff = (jm >> 1) * 8;
        v_doff = (jm & 1) * 8;
    }

    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m_run[nt][0] = m_run[nt][1] = -INFINITY;
            l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) o[nt][ks][0] = o[nt][ks][1] = o[nt][ks][2] = o[nt][ks][3] = 0.f;
        }
    }

    __device__ __forceinline__ void set_q(int nt, int ks, int h, float x0, float x1) {
        const uint32_t hi = Tr::pack(x0, x1);
        qhi[nt][ks][h] = hi;
        if constexpr (QLO) qlo[nt][ks][h] = Tr::pack(x0 - Tr::unpack_lo(hi), x1 - Tr::unpack_hi(hi));
    }

    // Query fragments (B operand of the score MMA): head nt*8+gid, dims ks*16 + 2*c4 (+1, +8, +9), read from
    // global memory.
    __device__ __forceinline__ void load_q_global(const AttnParams& p, int seq, int kvh_global, int lane) {
        const int gid = lane >> 2, c4 = lane & 3;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int j = nt * 8 + gid;
            const bool live = j < p.g;
            const size_t qbase = (static_cast<size_t>(seq) * p.nh + kvh_global * p.g + (live ? j : 0)) * D;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int d = ks * 16 + 2 * c4 + h * 8;
                    set_q(nt, ks, h, live ? load_any(p.q, qbase + d, p.q_dtype) : 0.f,
                          live ? load_any(p.q, qbase + d + 1, p.q_dtype) : 0.f);
                }
        }
    }

    // Same from the query area of a stage: [kvh_cta * g heads][D] in the query dtype (a generic pointer into
    // shared memory; every load is issued before the conversions).
    __device__ __forceinline__ void load_q_smem(const AttnParams& p, const uint8_t* qs, int warp, int lane) {
        const int gid = lane >> 2, c4 = lane & 3;
        if (p.q_dtype == KVP_DTYPE_F32) {
            float2 v[NT][KS][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int j = nt * 8 + gid;
                const float* row = reinterpret_cast<const float*>(qs) + (warp * p.g + (j < p.g ? j : 0)) * D;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        v[nt][ks][h] = *reinterpret_cast<const float2*>(row + ks * 16 + 2 * c4 + h * 8);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const bool live = nt * 8 + gid < p.g;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        set_q(nt, ks, h, live ? v[nt][ks][h].x : 0.f, live ? v[nt][ks][h].y : 0.f);
            }
        } else {
            uint32_t v[NT][KS][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int j = nt * 8 + gid;
                const uint16_t* row = reinterpret_cast<const uint16_t*>(qs) + (warp * p.g + (j < p.g ? j : 0)) * D;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        v[nt][ks][h] = *reinterpret_cast<const uint32_t*>(row + ks * 16 + 2 * c4 + h * 8);
            }
            const bool f16 = p.q_dtype == KVP_DTYPE_F16;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const bool live = nt * 8 + gid < p.g;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t x = v[nt][ks][h];
                        float x0 = f16 ? F16Traits<__half>::unpack_lo(x) : F16Traits<__nv_bfloat16>::unpack_lo(x);
                        float x1 = f16 ? F16Traits<__half>::unpack_hi(x) : F16Traits<__nv_bfloat16>::unpack_hi(x);
                        set_q(nt, ks, h, live ? x0 : 0.f, live ? x1 : 0.f);
                    }
            }
        }
    }

    // One 16-token tile: `valid` rows hold context tokens.
    __device__ __forceinline__ void tile(const AttnParams& p, uint32_t kst, uint32_t vst, int valid, int warp,
                                         int lane) {
        const int gid = lane >> 2;
        float sacc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
        // ---- scores S^T = K . Q^T
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int d = ks * 16 + k_doff;
            const uint32_t addr = kst + k_row_off + static_cast<uint32_t>(d / G_::W) * p.box_slot +
                                  ((static_cast<uint32_t>((d % G_::W) >> 3) ^ k_x) << 4);
            uint32_t a[4];
            ldsm_x4(addr, a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                mma16816<KV>(sacc[nt], a, qhi[nt][ks][0], qhi[nt][ks][1]);
                if constexpr (QLO) mma16816<KV>(sacc[nt], a, qlo[nt][ks][0], qlo[nt][ks][1]);
            }
        }
        // ---- online softmax (log2 domain); rows gid / gid+8 are tokens, columns 2*c4, 2*c4+1 heads
        uint32_t pb_hi[NT][2], pb_lo[NT][2];
        const bool row0_ok = gid < valid, row1_ok = gid + 8 < valid;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float sv[4];
            sv[0] = row0_ok ? sacc[nt][0] * p.sl2 : -INFINITY;
            sv[1] = row0_ok ? sacc[nt][1] * p.sl2 : -INFINITY;
            sv[2] = row1_ok ? sacc[nt][2] * p.sl2 : -INFINITY;
            sv[3] = row1_ok ? sacc[nt][3] * p.sl2 : -INFINITY;
            float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
            const float corr0 = fast_exp2(m_run[nt][0] - mn0), corr1 = fast_exp2(m_run[nt][1] - mn1);
            m_run[nt][0] = mn0;
            m_run[nt][1] = mn1;
            const float p0 = fast_exp2(sv[0] - mn0), p1 = fast_exp2(sv[1] - mn1);
            const float p2 = fast_exp2(sv[2] - mn0), p3 = fast_exp2(sv[3] - mn1);
            l_run[nt][0] = l_run[nt][0] * corr0 + (p0 + p2);
            l_run[nt][1] = l_run[nt][1] * corr1 + (p1 + p3);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                o[nt][ks][0] *= corr0;
                o[nt][ks][1] *= corr1;
                o[nt][ks][2] *= corr0;
                o[nt][ks][3] *= corr1;
            }
            const uint32_t h01 = Tr::pack(p0, p1), h23 = Tr::pack(p2, p3);
            const uint32_t l01 = Tr::pack(p0 - Tr::unpack_lo(h01), p1 - Tr::unpack_hi(h01));
            const uint32_t l23 = Tr::pack(p2 - Tr::unpack_lo(h23), p3 - Tr::unpack_hi(h23));
            pb_hi[nt][0] = movmatrix_trans(h01);
            pb_hi[nt][1] = movmatrix_trans(h23);
            pb_lo[nt][0] = movmatrix_trans(l01);
            pb_lo[nt][1] = movmatrix_trans(l23);
        }
        // ---- rows past the end of the context: zero this head's V rows so stale bytes cannot turn
        // 0 * garbage into NaN in the PV product.
        if (valid < 16) {
            constexpr int UPR = G_::NCH * (G_::W / 8);  // 16-byte units per token row of one head
            const int units = (16 - valid) * UPR;
            for (int u = lane; u < units; u += 32) {
                const int t = valid + u / UPR;
                const int rem = u % UPR;
                const int c = rem / (G_::W / 8), cu = rem % (G_::W / 8);
                const uint32_t ro = static_cast<uint32_t>(t / p.R) * G_::NCH * p.box_slot +
                                    static_cast<uint32_t>(c) * p.box_slot + static_cast<uint32_t>(warp) * p.head_stride +
                                    static_cast<uint32_t>(t % p.R) * G_::ROWB;
                const uint32_t a = vst + ro + ((static_cast<uint32_t>(cu) ^ ((ro >> 7) & G_::SWM)) << 4);
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
            }
            __syncwarp();
        }
        // ---- O^T += V^T . P^T
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            const int d = mt * 16 + v_doff;
            const uint32_t addr = vst + v_row_off + static_cast<uint32_t>(d / G_::W) * p.box_slot +
                                  ((static_cast<uint32_t>((d % G_::W) >> 3) ^ v_x) << 4);
            uint32_t a[4];
            ldsm_x4_trans(addr, a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                mma16816<KV>(o[nt][mt], a, pb_hi[nt][0], pb_hi[nt][1]);
                mma16816<KV>(o[nt][mt], a, pb_lo[nt][0], pb_lo[nt][1]);
            }
        }
        if (valid < 16) fence_proxy_async_smem();  // generic writes above precede the next TMA into this stage
    }

    // Lane-wise state exchange between the warps of one kv head: NREG floats per lane.
    static constexpr int NREG = NT * KS * 4 + NT * 4;
    __device__ __forceinline__ void store_state(float* area, int lane) const {
        int r = 0;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int e = 0; e < 4; ++e) area[(r++) * 32 + lane] = o[nt][ks][e];
            area[(r++) * 32 + lane] = m_run[nt][0];
            area[(r++) * 32 + lane] = m_run[nt][1];
            area[(r++) * 32 + lane] = l_run[nt][0];
            area[(r++) * 32 + lane] = l_run[nt][1];
        }
    }
    // Folds another warp's state (same lane layout) into this one: per head column, rescale both sides to
    // the larger running max.  A warp that saw no tile has m = -inf and contributes nothing.
    __device__ __forceinline__ void merge_state(const float* area, int lane) {
        int r = 0;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int rm = r + KS * 4;
            float a[2], b[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float m2 = area[(rm + e) * 32 + lane];
                const float l2 = area[(rm + 2 + e) * 32 + lane];
                const float M = fmaxf(m_run[nt][e], m2);
                a[e] = M == -INFINITY ? 0.f : fast_exp2(m_run[nt][e] - M);
                b[e] = M == -INFINITY ? 0.f : fast_exp2(m2 - M);
                l_run[nt][e] = l_run[nt][e] * a[e] + l2 * b[e];
                m_run[nt][e] = M;
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float v = area[(r++) * 32 + lane];
                    o[nt][ks][e] = o[nt][ks][e] * a[e & 1] + v * b[e & 1];
                }
            r += 4;
        }
    }

    // Segment epilogue: the final normalised output (`single`) or a partial row `part_row` (nh heads).
    __device__ __forceinline__ void finish(const AttnParams& p, int lane, int seq, int kvh_global, bool single,
                                           size_t part_row) {
        const int gid = lane >> 2, c4 = lane & 3;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float l = l_run[nt][e];
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
                l_run[nt][e] = l;
            }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = nt * 8 + 2 * c4 + e;
                if (j >= p.g) continue;
                const int hq = kvh_global * p.g + j;
                if (single) {
                    const float inv = 1.f / l_run[nt][e];
                    const size_t ob = (static_cast<size_t>(seq) * p.nh + hq) * D;
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt) {
                        store_any(p.out, ob + mt * 16 + gid, p.out_dtype, o[nt][mt][e] * inv);
                        store_any(p.out, ob + mt * 16 + gid + 8, p.out_dtype, o[nt][mt][2 + e] * inv);
                    }
                } else {
                    float* wo = p.ws_o + (part_row + hq) * D;
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt) {
                        wo[mt * 16 + gid] = o[nt][mt][e];
                        wo[mt * 16 + gid + 8] = o[nt][mt][2 + e];
                    }
                    if (gid == 0) p.ws_ml[part_row + hq] = make_float2(m_run[nt][e], l_run[nt][e]);
                }
            }
    }
};

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// One attention segment: tiles [tile0, tile1) of sequence `seq`, written as the final output (`single`) or
// as the partial row `part_row`.
struct Segment {
    int seq, tile0, tile1;
    int len;  // the sequence's context length
    bool single;
    size_t part_row;
    int c0, nseg;  // stream-K: first CTA holding part of the sequence and how many do (0: merged elsewhere;
                   // -1: split, Segs::span() gives them)
};

// Fixed splits: the CTA's one segment.
struct SplitSegments {
    static constexpr bool lazy_span = false;
    Segment seg;
    bool done;
    __device__ __forceinline__ bool next(Segment& s) {
        if (done) return false;
        s = seg;
        done = true;
        return true;
    }
};

// floor(a * b / c) for 0 <= a * b < 2^53 and c > 0: a double-precision quotient (the product is exact in a
// double) corrected by one integer step, instead of a 64-bit integer division routine.
__device__ __forceinline__ long long muldiv_floor(long long a, long long b, long long c) {
    const long long n = a * b;
    long long q = static_cast<long long>(static_cast<double>(n) / static_cast<double>(c));
    if (q * c > n) --q;
    else if ((q + 1) * c <= n) ++q;
    return q;
}

// CTA c of Ge owns tiles [c*T/Ge, (c+1)*T/Ge) of the concatenation of all sequences' tiles (T in total).
// The owner of tile t: the c with c*T < (t+1)*G <= (c+1)*T, i.e. floor(((t+1)*G - 1) / T).  The quotient is
// below 2^16, so a single-precision estimate is off by at most one and one integer step corrects it.
__device__ __forceinline__ int cta_of_tile(long long t, long long T, int G) {
    const long long n = (t + 1) * G - 1;
    long long c = static_cast<long long>(static_cast<float>(n) / static_cast<float>(T));
    if (c * T > n) --c;
    else if ((c + 1) * T <= n) ++c;
    return static_cast<int>(c);
}

// The division of the step's T units between Ge CTAs.  Even: CTA c owns [c*T/Ge, (c+1)*T/Ge).  Tapered: CTAs
// are dispatched in index order into the SM slots the previous grid frees, so when launches run back to back
// the last ones start late -- by up to the length of a prologue; the last m CTAs each give up D units, spread
// evenly over all CTAs:
//   begin(c) = floor(c * (T + D m) / Ge) - D * max(0, c - (Ge - m)).
// D is dropped when the even share is below D + 2 units, so every CTA keeps at least one unit (the merge counts
// assume it).  Integer arithmetic throughout; begin() is the one function a CTA's own range and the owner of a
// unit both come from.
struct Partition {
    int T;         // units (the prefix sums are 32-bit)
    int Ge, m, D;  // D == 0: even split
    Partition() = default;
    __device__ __forceinline__ Partition(long long T_, int Ge_, int taper_m, int taper_d) : T(static_cast<int>(T_)), Ge(Ge_) {
        m = min(taper_m, Ge);
        D = (m > 0 && Ge > 0 && T >= static_cast<long long>(Ge) * (taper_d + 2)) ? taper_d : 0;
    }
    __device__ __forceinline__ long long begin(long long c) const {
        if (D == 0) return muldiv_floor(c, T, Ge);
        return muldiv_floor(c, static_cast<long long>(T) + static_cast<long long>(D) * m, Ge) -
               static_cast<long long>(D) * max(0LL, c - (Ge - m));
    }
    // The CTA whose range holds unit t (the last c with begin(c) <= t).
    __device__ __forceinline__ int owner(long long t) const {
        if (D == 0) return cta_of_tile(t, T, Ge);
        const long long Tp = static_cast<long long>(T) + static_cast<long long>(D) * m;
        const int cr = Ge - m;
        if (t < muldiv_floor(cr, Tp, Ge)) return cta_of_tile(t, Tp, Ge);  // before the taper: an even split of Tp
        // in the taper begin(c) ~ c (Tp / Ge - D) + D cr: estimate, then step to the exact owner
        long long c = cr + static_cast<long long>(static_cast<double>(t - muldiv_floor(cr, Tp, Ge)) /
                                                  (static_cast<double>(Tp) / Ge - D));
        c = min(max(c, static_cast<long long>(cr)), static_cast<long long>(Ge - 1));
        while (c > cr && begin(c) > t) --c;
        while (c + 1 < Ge && begin(c + 1) <= t) ++c;
        return static_cast<int>(c);
    }
};

// Stream-K: the CTA's tile range [t, end) of the concatenated sequences, cut at sequence boundaries.
// The concatenated space is counted in units: each valid sequence spans X start-cost units (the time a CTA
// spends switching to a new sequence, in tiles) followed by its tiles, so the balanced split charges that
// cost to the CTA that starts the sequence.  A CTA whose range holds only a sequence's start-cost units does
// no work for it; the CTAs holding its tiles are c0 .. c0 + nseg - 1.  Lazy: a split segment's span is not
// found here but by the one thread that records it (span()), with the partition rebuilt from the launch
// parameters -- for the register-heavy instantiations, where keeping it in every warp costs spills; the others
// find it here, in every warp at once (faster: Qwen2.5-0.5B-shaped steps 137.0k against 133.1k tok/s on B200).
template <bool Lazy>
struct StreamSegments {
    static constexpr bool lazy_span = Lazy;
    const int32_t* P;  // unit prefix sums in shared memory
    const uint8_t* R;  // tokens in each sequence's last tile, in shared memory
    long long t, end;
    Partition part;    // (not read when Lazy)
    int s, cta, nh, X;
    __device__ __forceinline__ bool next(Segment& sg) {
        while (t < end) {
            while (P[s + 1] <= t) ++s;
            const long long e = min(end, static_cast<long long>(P[s + 1]));
            const long long first = static_cast<long long>(P[s]) + X;  // the sequence's first tile, in units
            const long long a = max(t, first);
            t = e;
            if (a >= e) continue;  // only start-cost units of this sequence here
            sg.seq = s;
            sg.len = (P[s + 1] - P[s] - X - 1) * 16 + R[s];
            sg.tile0 = static_cast<int>(a - first);
            sg.tile1 = static_cast<int>(e - first);
            sg.single = (a == first) && (e == P[s + 1]);
            sg.part_row = static_cast<size_t>(cta + s) * nh;
            if (sg.single) {
                sg.c0 = cta;
                sg.nseg = 1;
            } else if constexpr (Lazy) {
                sg.c0 = cta;
                sg.nseg = -1;
            } else {
                sg.c0 = part.owner(first);
                sg.nseg = part.owner(P[s + 1] - 1) - sg.c0 + 1;
            }
            return true;
        }
        return false;
    }
    // The CTAs holding parts of sequence s (Lazy only), from the launch parameters and the prefix sums.
    __device__ __forceinline__ void span(const AttnParams& p, int s, int& c0, int& nseg) const {
        const int T = P[p.num_seqs];
        const Partition pt(T, min(p.G, T), p.taper_m, p.taper_d);
        c0 = pt.owner(static_cast<long long>(P[s]) + X);
        nseg = pt.owner(static_cast<long long>(P[s + 1]) - 1) - c0 + 1;
    }
};

__device__ __forceinline__ void init_barriers(const AttnParams& p, uint64_t* full_bar, uint64_t* empty_bar,
                                              uint64_t* qfull, uint64_t* qempty, PipeState* ps) {
    if (threadIdx.x == 0) {
        ps->abort = 0;
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), static_cast<uint32_t>(p.kvh_cta));
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&qfull[s]), 1);
            mbar_init(smem_u32(&qempty[s]), static_cast<uint32_t>(p.kvh_cta * p.wph));
        }
        fence_barrier_init();
    }
    __syncthreads();
}

// The work of one CTA over its segments.  Warp kvh_cta * wph is the producer; consumer warp w serves kv head
// w % kvh_cta and takes the tiles whose stage index is congruent to w / kvh_cta modulo wph (the stage count
// is a multiple of wph, so each stage always has the same kvh_cta consumers).  At the end of a segment the
// wph warps of a head combine their (m, l, O) lane by lane through shared memory.
//
// Every wait is bounded: a warp that gives up reports KVP_STATUS_TIMEOUT, raises ps->abort and then runs
// through the rest of its control flow without waiting (so the named barriers of its partner warps are still
// reached).  The producer stops issuing once one of its own waits gave up (a consumer that gave up stops
// freeing stages, so the producer's next wait gives up too) and, before it returns, waits (bounded) for every
// copy it issued that no consumer waited for, so the CTA never exits with a bulk copy in flight into its
// shared memory.  What it issued is known from registers: every tile before the counter (okst, okr) after its
// last fully issued batch, plus the lanes `fmask` of the batch at (fst0, fr0) that failed; query loads: jq.
template <int D>
__device__ __forceinline__ void merge_rows(const AttnParams& p, size_t row0, size_t stride, int n, size_t out_off,
                                           int lane);
template <int D, int IT, int U>
__device__ __forceinline__ void merge_group(const AttnParams& p, int seq, int c0, int nseg, int hq0, int heads,
                                            int tid, int nthreads);

// Merge batch shape per kernel instantiation (items per thread x partials per load round), the widest that
// keeps the kernel free of register spills; 0 = one warp per head (merge_rows) for the instantiations whose
// main loop already needs nearly every register (more than 8 query heads per kv head at head_dim >= 96, and
// head_dim 256).
template <int D, int NT>
struct MergeShape {
    static constexpr bool per_warp = (NT == 2 && D >= 96) || D >= 256;
    static constexpr int IT = 2;
    static constexpr int U = (D <= 64 && NT == 1) ? 4 : 2;
};

// After a wait gave up: lane 0 of the producer waits (bounded) for the last copy issued into each stage and
// query slot; a stage whose last round a consumer already waited for completes at once.  `stall`: stage 0's
// round 0 was the failure-detection test's phantom (nothing in flight), skipped.
__device__ __forceinline__ void drain_copies(const AttnParams& p, uint64_t* full_bar, uint64_t* qfull, int lane, int okst,
                                             int okr, int fst0, int fr0, unsigned fmask, int jq, bool stall) {
    __syncwarp();
    if (lane == 0) {
        auto wait = [&](uint32_t bar, int round) {
            if (!mbar_wait(bar, static_cast<uint32_t>(round & 1), p.wait_limit)) report(p.status, KVP_STATUS_TIMEOUT);
        };
        for (int st = 0; st < p.stages; ++st) {
            const int n = okr + (st < okst ? 1 : 0);  // rounds issued into stage st before the failed batch
            if (n > 0 && !(stall && st == 0 && n == 1)) wait(smem_u32(&full_bar[st]), n - 1);
        }
        for (int k = 0; k < 32; ++k) {
            if (!((fmask >> k) & 1u)) continue;
            int st = fst0 + k, r = fr0;
            if (st >= p.stages) {
                st -= p.stages;
                ++r;
            }
            wait(smem_u32(&full_bar[st]), r);
        }
        for (int k = max(0, jq - 2); k < jq; ++k) wait(smem_u32(&qfull[k & 1]), k >> 1);
    }
    __syncwarp();
}

template <int D, int NT, class KV, bool QLO, class Segs>
__device__ __forceinline__ void cta_body(const AttnParams& p, const CUtensorMap* km, const CUtensorMap* vm, Segs segs,
                                         uint8_t* dyn, uint32_t smem_base, uint64_t* full_bar, uint64_t* empty_bar,
                                         uint64_t* qfull, uint64_t* qempty, int grp, int* pend, bool waited,
                                         PipeState* ps) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int NC = p.kvh_cta * p.wph;
    const int S = p.stages;
    const uint32_t qelem = p.q_dtype == KVP_DTYPE_F32 ? 4u : 2u;
    const uint32_t q_bytes = static_cast<uint32_t>(p.kvh_cta * p.g * D) * qelem;
    const int kvh0 = grp * p.kvh_cta;
    Segment sg;
    if (warp == NC) {
        // ------------------------------------------------------------ producer warp
        if (lane == 0) {
            prefetch_tensormap(km);
            prefetch_tensormap(vm);
        }
        bool ok = true;
        int pst = 0, pr = 0, j = 0;  // stage and round (i % S, i / S) of the running tile counter i
        int okst = 0, okr = 0, fst0 = 0, fr0 = 0, jq = 0;  // what was issued (see above)
        unsigned fmask = 0;
        // Failure-detection test only (kvp_attention_wait_test): in every CTA of the grid's first row (kv-head group
        // 0 of the balanced schedule, split 0 of the fixed splits -- rows that always hold CTAs with tiles) stage 0
        // is armed for 16 bytes of a copy that is never issued and the tiles start at stage 1, so the consumers,
        // which expect the first tile in stage 0, wait until their limit.  Nothing is ever in flight for stage 0.
        const bool stall = p.stall_first_stage && blockIdx.y == 0;
        if (stall) {
            if (lane == 0) mbar_arrive_expect_tx(smem_u32(&full_bar[0]), 16u);
            __syncwarp();
            pst = okst = 1;  // the stage count is at least 2
        }
        while (segs.next(sg)) {
            const int len = sg.len;
            const int32_t* trow = p.tables + static_cast<size_t>(sg.seq) * p.max_blocks;
            int cache_lo = -(1 << 30);
            int32_t cached = 0;
            // One run per tile: issue in batches of up to 8 tiles (one per lane); else one tile at a time.
            const int nb_max = p.nruns == 1 ? min(8, S) : 1;
            auto produce_range = [&](int from, int to) {
                for (int tile = from; tile < to;) {
                    const int nb = min(nb_max, to - tile);
                    bool sent_all = false;
                    if (ok) {
                        if (nb_max > 1) {
                            unsigned issued = 0;
                            ok = produce_batch<D>(p, km, vm, smem_base, full_bar, empty_bar, pst, pr, tile, nb, len, trow,
                                                  kvh0, lane, cache_lo, cached, issued);
                            if (!ok) {
                                fst0 = pst;
                                fr0 = pr;
                                fmask = issued;
                            }
                            sent_all = ok;
                        } else {
                            const int st = pst;
                            if (pr >= 1 && !mbar_wait(smem_u32(&empty_bar[st]), static_cast<uint32_t>((pr - 1) & 1),
                                                      p.wait_limit)) {
                                if (lane == 0) report(p.status, KVP_STATUS_TIMEOUT);
                                ok = false;
                            } else {
                                const uint32_t kst = smem_base + static_cast<uint32_t>(st) * p.stage_bytes;
                                produce_tile<D>(p, km, vm, kst, kst + p.stage_half, smem_u32(&full_bar[st]), tile * 16,
                                                len, trow, kvh0, lane, cache_lo, cached);
                                sent_all = true;
                            }
                        }
                        __syncwarp();
                    }
                    tile += nb;
                    pst += nb;
                    if (pst >= S) {
                        pst -= S;
                        ++pr;
                    }
                    if (sent_all) {
                        okst = pst;
                        okr = pr;
                    }
                }
            };
            const bool appends = p.k_new != nullptr && sg.tile1 == ((len + 15) >> 4);
            int first = sg.tile0;
            if (!waited) {
                // Early load: the first tiles of the CTA's range -- one ring at most, so no stage has to be freed
                // by the consumers, and short of the tile the fused append writes into -- before waiting for the
                // previous kernel; queries, the append and every write come after the wait.  Queries that a copy
                // on another stream produces (inputs_ready) are not the previous kernel's: they are loaded before
                // the wait too, so the consumers may work through the first ring during the previous kernel
                // (they wait for it before their first global write).
                first = min(sg.tile1 - (appends ? 1 : 0), sg.tile0 + S);
                produce_range(sg.tile0, first);
                if (p.inputs_ready == nullptr) {
                    griddep_wait();
                    waited = true;
                }
            }
            if (j == 0 && p.inputs_ready != nullptr && ok && !warp_wait_flag(p.inputs_ready, p.inputs_epoch, p.wait_limit)) {
                if (lane == 0) report(p.status, KVP_STATUS_TIMEOUT);
                ok = false;
            }
            if (p.q_area != 0) {
                const int slot = j & 1;
                if (ok && j >= 2 &&
                    !mbar_wait(smem_u32(&qempty[slot]), static_cast<uint32_t>(((j >> 1) - 1) & 1), p.wait_limit)) {
                    if (lane == 0) report(p.status, KVP_STATUS_TIMEOUT);
                    ok = false;
                }
                if (ok && lane == 0) {
                    const uint32_t qb = smem_u32(&qfull[slot]);
                    mbar_arrive_expect_tx(qb, q_bytes);
                    const char* src = static_cast<const char*>(p.q) +
                                      (static_cast<size_t>(sg.seq) * p.nh + static_cast<size_t>(kvh0) * p.g) * D * qelem;
                    bulk_load(smem_base + p.q_off + static_cast<uint32_t>(slot) * p.q_area, src, q_bytes, qb);
                }
            }
            if (p.q_area != 0 && ok) jq = j + 1;  // query loads 0 .. j issued
            if (!waited) {
                griddep_wait();
                waited = true;
            }
            if (appends && ok) append_new_token<D>(p, sg.seq, len, trow, kvh0, lane);
            produce_range(first, sg.tile1);
            ++j;
        }
        if (!ok || *reinterpret_cast<volatile int*>(&ps->abort))
            drain_copies(p, full_bar, qfull, lane, okst, okr, fst0, fr0, fmask, jq, stall);
        return;
    }
    if (warp > NC) return;

    // ---------------------------------------------------------------- consumer warps
    const int head = warp % p.kvh_cta, sub = warp / p.kvh_cta;
    const int kvh_global = kvh0 + head;
    Consumer<D, NT, KV, QLO> cs;
    cs.init_geometry(p, head, lane);
    float* comb = reinterpret_cast<float*>(dyn + p.comb_off);
    constexpr int NREG = Consumer<D, NT, KV, QLO>::NREG;
    bool ok = true;
    int j = 0;
    int cst = 0, cph = 0, turn = 0;  // stage, its phase and the sub-warp whose turn it is, for the next tile
    // Split segments of this CTA: at most two (only the first and the last segment of a CTA's range can be
    // parts of a longer sequence); pend[k] flags a merge, pend[2 + 3k ..] holds (seq, c0, nseg); old0 / old1
    // hold a writer warp's counter values from before its adds.
    int np = 0, old0 = -1, old1 = -1;
    // Consumers can only run ahead of the producer's wait for the previous kernel when the queries came from
    // another stream's copy (see the producer); then each segment's global writes wait for that kernel first
    // (at once after the first time).
    const bool write_wait = !waited && p.inputs_ready != nullptr;
    while (segs.next(sg)) {
        const int len = sg.len;
        if (p.q_area != 0) {
            const int slot = j & 1;
            if (ok && !mbar_wait(smem_u32(&qfull[slot]), static_cast<uint32_t>((j >> 1) & 1), p.wait_limit)) {
                if (lane == 0) {
                    report(p.status, KVP_STATUS_TIMEOUT);
                    *reinterpret_cast<volatile int*>(&ps->abort) = 1;
                }
                ok = false;
            }
            if (ok) cs.load_q_smem(p, dyn + p.q_off + static_cast<size_t>(slot) * p.q_area, head, lane);
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(smem_u32(&qempty[slot]));
        } else {
            if (j == 0 && p.inputs_ready != nullptr && ok && !warp_wait_flag(p.inputs_ready, p.inputs_epoch, p.wait_limit)) {
                if (lane == 0) {
                    report(p.status, KVP_STATUS_TIMEOUT);
                    *reinterpret_cast<volatile int*>(&ps->abort) = 1;
                }
                ok = false;
            }
            // queries the previous kernel may write: read them once it is done (the producer's wait does not
            // order these loads; with inputs_ready they come from the flagged copy instead)
            if (j == 0 && !waited && p.inputs_ready == nullptr) griddep_wait();
            cs.load_q_global(p, sg.seq, kvh_global, lane);
        }
        cs.reset();
        for (int tile = sg.tile0; tile < sg.tile1; ++tile) {
            const int st = cst, ph = cph;
            const bool mine = turn == sub;
            if (++cst == S) {
                cst = 0;
                cph ^= 1;
            }
            if (++turn == p.wph) turn = 0;
            if (!ok || !mine) continue;
            if (!mbar_wait(smem_u32(&full_bar[st]), static_cast<uint32_t>(ph), p.wait_limit)) {
                if (lane == 0) {
                    report(p.status, KVP_STATUS_TIMEOUT);
                    *reinterpret_cast<volatile int*>(&ps->abort) = 1;
                }
                ok = false;
                continue;
            }
            const uint32_t kst = smem_base + static_cast<uint32_t>(st) * p.stage_bytes;
            cs.tile(p, kst, kst + p.stage_half, min(16, len - tile * 16), head, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[st]));
        }
        if (p.wph > 1) {
            float* area = comb + static_cast<size_t>(head) * NREG * 32;
            const size_t stride = static_cast<size_t>(p.kvh_cta) * NREG * 32;
            if (sub > 0) cs.store_state(area + (sub - 1) * stride, lane);
            named_barrier(1 + head, p.wph * 32);
            if (sub == 0)
                for (int k = 1; k < p.wph; ++k) cs.merge_state(area + (k - 1) * stride, lane);
            named_barrier(1 + head, p.wph * 32);  // the area is rewritten by the next segment
        }
        if (write_wait) griddep_wait();
        if (sub == 0 && ok) cs.finish(p, lane, sg.seq, kvh_global, sg.single, sg.part_row);
        // Stream-K, sequence split across CTAs: each head's writer warp counts its partial rows as done with
        // one releasing add (the warp barrier orders its lanes' rows before it); a sequence is complete when
        // every writer warp of every CTA holding part of it has added (nseg * kvh_cta).  The add's old value
        // is only examined after the CTA's last segment, so no warp waits for its round trip or for another
        // warp here.
        if (!sg.single && sg.nseg != 0) {
            if (sub == 0) {
                __syncwarp();
                if (lane == 0 && ok) {
                    const int old = atom_add_acq_rel_gpu(p.counters + static_cast<size_t>(sg.seq) * p.groups + grp, 1);
                    if (np == 0) old0 = old; else old1 = old;
                }
            }
            if (warp == 0 && lane == 0) {
                int c0 = sg.c0, nseg = sg.nseg;
                if constexpr (Segs::lazy_span) {
                    if (nseg < 0) segs.span(p, sg.seq, c0, nseg);
                }
                pend[2 + 3 * np] = sg.seq;
                pend[3 + 3 * np] = c0;
                pend[4 + 3 * np] = nseg;
            }
            ++np;
        }
        ++j;
    }
    // The writer warp whose add completed a sequence's count resets the counter and flags the merge; the CTA
    // then merges (that acquiring add made the other parts' rows visible; the barrier extends it to every
    // merging thread).
    if (np > 0) {
        named_barrier(kMaxConsumerWarps + 1, NC * 32);  // pend coordinates written
        if (sub == 0 && lane == 0 && ok) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                if (k >= np || (k ? old1 : old0) != pend[4 + 3 * k] * p.kvh_cta - 1) continue;
                atomicExch(p.counters + static_cast<size_t>(pend[2 + 3 * k]) * p.groups + grp, 0);
                pend[k] = 1;
            }
        }
        named_barrier(kMaxConsumerWarps + 1, NC * 32);  // merge flags written
        for (int k = 0; k < np; ++k) {
            if (!pend[k]) continue;
            const int seq = pend[2 + 3 * k], c0 = pend[3 + 3 * k], nseg = pend[4 + 3 * k];
            using MS = MergeShape<D, NT>;
            if constexpr (MS::per_warp) {
                for (int jj = warp; jj < p.kvh_cta * p.g; jj += NC) {
                    const int hq = kvh0 * p.g + jj;
                    merge_rows<D>(p, static_cast<size_t>(c0 + seq) * p.nh + hq, static_cast<size_t>(p.nh), nseg,
                                  (static_cast<size_t>(seq) * p.nh + hq) * D, lane);
                }
            } else {
                // all consumer threads merge the group's query heads, a 4-float column each
                merge_group<D, MS::IT, MS::U>(p, seq, c0, nseg, kvh0 * p.g, p.kvh_cta * p.g, threadIdx.x, NC * 32);
            }
        }
    }
}

// ---------------------------------------------------------------- fixed-split schedule
template <int D, int NT, class KV, bool QLO>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const AttnParams p) {
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
    __shared__ __align__(8) uint64_t qfull[2], qempty[2];
    __shared__ PipeState ps;
    extern __shared__ uint8_t dyn_smem[];

    const int seq = blockIdx.x / p.groups;
    const int grp = blockIdx.x - seq * p.groups;
    const int split = blockIdx.y;
    const int len = p.lens[seq];
    const int ntiles = tiles_of_len(p, len);
    const int nsplit = (ntiles + p.split_tiles - 1) / p.split_tiles;
    if (ntiles == 0) {
        // Invalid length: report once and write zeros so the output is deterministic.
        if (split == 0) {
            if (threadIdx.x == 0) report(p.status, KVP_STATUS_BAD_LEN);
            const int heads = p.kvh_cta * p.g;
            for (int i = threadIdx.x; i < heads * D; i += blockDim.x) {
                const int hq = grp * heads + i / D;
                store_any(p.out, (static_cast<size_t>(seq) * p.nh + hq) * D + i % D, p.out_dtype, 0.f);
            }
        }
        return;
    }
    if (split >= nsplit) return;
    const uint32_t base_off = ((smem_u32(dyn_smem) + 1023u) & ~1023u) - smem_u32(dyn_smem);
    init_barriers(p, full_bar, empty_bar, qfull, qempty, &ps);
    SplitSegments segs;
    segs.seg.seq = seq;
    segs.seg.len = len;
    segs.seg.tile0 = split * p.split_tiles;
    segs.seg.tile1 = min(ntiles, segs.seg.tile0 + p.split_tiles);
    segs.seg.single = nsplit == 1;
    segs.seg.part_row = (static_cast<size_t>(seq) * p.max_splits + split) * p.nh;
    segs.seg.c0 = 0;
    segs.seg.nseg = 0;
    segs.done = false;
    cta_body<D, NT, KV, QLO>(p, &kmap, &vmap, segs, dyn_smem + base_off, smem_u32(dyn_smem) + base_off, full_bar,
                        empty_bar, qfull, qempty, grp, nullptr, true, &ps);
}

// ---------------------------------------------------------------- stream-K schedule

// Unit prefix sums P[0..ns] of all sequences into shared memory (a valid sequence counts seq_units start-cost
// units plus its tiles, an invalid length counts nothing), and R[s] =
// the tokens in sequence s's last tile, so segment starts need no global load of the length.
__device__ __forceinline__ void build_prefix(const AttnParams& p, int32_t* P, uint8_t* R, int32_t* warp_tot) {
    const int ns = p.num_seqs, nthr = blockDim.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = (nthr + 31) >> 5;
    const int per = (ns + nthr - 1) / nthr;
    const int b = min(tid * per, ns), e = min(b + per, ns);
    int local = 0;
    for (int i = b; i < e; ++i) {
        const int n = tiles_of_len(p, __ldg(p.lens + i));
        local += n ? n + p.seq_units : 0;
    }
    int x = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int v = lane < nwarps ? warp_tot[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, v, off);
            if (lane >= off) v += y;
        }
        if (lane < nwarps) warp_tot[lane] = v;
    }
    __syncthreads();
    int run = (warp > 0 ? warp_tot[warp - 1] : 0) + (x - local);
    for (int i = b; i < e; ++i) {
        const int len = __ldg(p.lens + i);
        P[i] = run;
        const int n = tiles_of_len(p, len);
        run += n ? n + p.seq_units : 0;
        R[i] = static_cast<uint8_t>(((len - 1) & 15) + 1);
    }
    if (tid == nthr - 1) P[ns] = warp_tot[nwarps - 1];
    __syncthreads();
}

// First sequence whose tile range ends after tile t (P[s+1] > t).
__device__ __forceinline__ int seq_of_tile(const int32_t* P, int ns, long long t) {
    int lo = 0, hi = ns - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (P[mid + 1] > t) hi = mid; else lo = mid + 1;
    }
    return lo;
}

template <int D, int NT, class KV, bool QLO>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1)
    paged_decode_streamk_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                                const AttnParams p) {
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
    __shared__ __align__(8) uint64_t qfull[2], qempty[2];
    __shared__ int32_t warp_tot[32];
    __shared__ PipeState ps;
    extern __shared__ uint8_t dyn_smem[];

    // Let the next kernel on the stream (a programmatic dependent launch) be scheduled now: its CTAs then take
    // each SM slot this grid frees, and run their prologue and early loads during this grid's tail.  Its
    // griddepcontrol.wait still waits for this whole grid to complete; the trigger only moves its scheduling.
    griddep_launch_dependents();
    const int c = blockIdx.x, grp = blockIdx.y;
    const uint32_t base_off = ((smem_u32(dyn_smem) + 1023u) & ~1023u) - smem_u32(dyn_smem);
    int32_t* P = reinterpret_cast<int32_t*>(dyn_smem + base_off + p.pre_off);
    uint8_t* R = reinterpret_cast<uint8_t*>(P + p.num_seqs + 1);
    build_prefix(p, P, R, warp_tot);
    const int ns = p.num_seqs;
    const long long T = P[ns];
    // With fewer tiles than CTAs only the first T CTAs work, so every working CTA owns >= 1 tile.
    const int Ge = static_cast<int>(min(static_cast<long long>(p.G), T));
    StreamSegments<MergeShape<D, NT>::per_warp> segs;
    segs.P = P;
    segs.R = R;
    const Partition part(T, Ge, p.taper_m, p.taper_d);
    segs.part = part;
    segs.X = p.seq_units;
    segs.t = Ge > 0 ? part.begin(c) : 0;
    segs.end = Ge > 0 ? part.begin(c + 1) : 0;
    segs.s = seq_of_tile(P, ns, segs.t);
    segs.cta = c;
    segs.nh = p.nh;
    __shared__ int pend[8];  // merge flags and coordinates of the CTA's split segments
    if (threadIdx.x < 2) pend[threadIdx.x] = 0;
    init_barriers(p, full_bar, empty_bar, qfull, qempty, &ps);  // (its barrier also publishes pend)
    // Everything above reads only seq_lens and shared memory; with an early start (programmatic dependent
    // launch) it overlaps the previous kernel's tail.  What follows may read what that kernel wrote or write
    // what it reads, so it waits for it -- with an early load, the producer warps first issue their CTA's
    // first tile loads (CTA 0, which may write zero rows below, waits here).
    const bool waited = !p.early_load || c == 0;
    if (waited) griddep_wait();
    if (c == 0) {
        // Sequences with an invalid length own no tile: report them and write zeros for this group's heads.
        // The scan is spread over the threads; the (rare) zero writes only run when it found one.
        bool bad = false;
        for (int s = threadIdx.x; s < ns; s += blockDim.x) bad |= P[s + 1] == P[s];
        if (__syncthreads_or(bad)) {
            const int heads = p.kvh_cta * p.g;
            for (int s = 0; s < ns; ++s) {
                if (P[s + 1] != P[s]) continue;
                if (threadIdx.x == 0 && grp == 0) report(p.status, KVP_STATUS_BAD_LEN);
                for (int i = threadIdx.x; i < heads * D; i += blockDim.x)
                    store_any(p.out, (static_cast<size_t>(s) * p.nh + grp * heads + i / D) * D + i % D, p.out_dtype, 0.f);
            }
        }
    }
    if (c >= Ge) return;
    cta_body<D, NT, KV, QLO>(p, &kmap, &vmap, segs, dyn_smem + base_off, smem_u32(dyn_smem) + base_off, full_bar,
                        empty_bar, qfull, qempty, grp, pend, waited, &ps);
}

// ---------------------------------------------------------------- merges
// Combines `n` partial rows of one (sequence, head) -- rows row0 + k * stride -- into the output: one warp.
// Lane k holds partial k's (m, l) (one L2 round trip), the weights stay in registers and the output loop's
// loads are independent of each other.  Partials written by other CTAs of the same launch are read through
// L2 (ld.global.cg).
template <int D>
__device__ __forceinline__ void merge_rows(const AttnParams& p, size_t row0, size_t stride, int n, size_t out_off,
                                           int lane) {
    constexpr int PER = (D + 31) / 32;
    float acc[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) acc[q] = 0.f;
    float M = -INFINITY, L = 0.f;
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int kk = k0 + lane;
        const float2 ml = kk < n ? __ldcg(&p.ws_ml[row0 + kk * stride]) : make_float2(-INFINITY, 0.f);
        float Mc = ml.x;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Mc = fmaxf(Mc, __shfl_xor_sync(0xffffffffu, Mc, off));
        const float Mn = fmaxf(M, Mc);
        const float rescale = M == -INFINITY ? 0.f : fast_exp2(M - Mn);
        const float w = kk < n ? fast_exp2(ml.x - Mn) : 0.f;
        float Lc = ml.y * w;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Lc += __shfl_xor_sync(0xffffffffu, Lc, off);
        L = L * rescale + Lc;
#pragma unroll
        for (int q = 0; q < PER; ++q) acc[q] *= rescale;
        M = Mn;
        const int cnt = min(32, n - k0);
#pragma unroll 4
        for (int k = 0; k < cnt; ++k) {
            const float wk = __shfl_sync(0xffffffffu, w, k);
            const float* src = p.ws_o + (row0 + static_cast<size_t>(k0 + k) * stride) * D;
#pragma unroll
            for (int q = 0; q < PER; ++q) {
                const int d = q * 32 + lane;
                if (d < D) acc[q] += __ldcg(src + d) * wk;
            }
        }
    }
    const float invL = 1.f / L;
#pragma unroll
    for (int q = 0; q < PER; ++q) {
        const int d = q * 32 + lane;
        if (d < D) store_any(p.out, out_off + d, p.out_dtype, acc[q] * invL);
    }
}

// Stream-K merge of one sequence's partials (CTAs c0 .. c0 + nseg - 1, rows (c + seq) * nh + head) for `heads`
// query heads from hq0, by nthreads threads: item = (head, 4-float column of the output).  Every partial's
// (m, l) and column are loaded U partials at a time, for IT items of a thread at once, before they are
// combined (a running max with rescaling), so a merge costs about one L2 round trip per U partials and IT items
// instead of a dependent chain per head.  Partials
// written by other CTAs of the same launch are read through L2 (ld.global.cg).
template <int D, int IT, int U>
__device__ __forceinline__ void merge_group(const AttnParams& p, int seq, int c0, int nseg, int hq0, int heads,
                                            int tid, int nthreads) {
    constexpr int C4 = D / 4;
    const int items = heads * C4;
    for (int base = tid; base < items; base += nthreads * IT) {
        float M[IT], Lsum[IT];
        float4 acc[IT];
        size_t row0[IT];
        int col[IT];
        bool on[IT];
#pragma unroll
        for (int t = 0; t < IT; ++t) {
            const int item = base + t * nthreads;
            on[t] = item < items;
            const int h = on[t] ? item / C4 : 0;
            col[t] = on[t] ? item - h * C4 : 0;
            row0[t] = static_cast<size_t>(c0 + seq) * p.nh + hq0 + h;
            M[t] = -INFINITY;
            Lsum[t] = 0.f;
            acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int k0 = 0; k0 < nseg; k0 += U) {
            float2 ml[IT][U];
            float4 o[IT][U];
#pragma unroll
            for (int t = 0; t < IT; ++t) {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (on[t] && k0 + u < nseg) {
                        const size_t row = row0[t] + static_cast<size_t>(k0 + u) * p.nh;
                        ml[t][u] = __ldcg(&p.ws_ml[row]);
                        o[t][u] = __ldcg(reinterpret_cast<const float4*>(p.ws_o + row * D) + col[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < IT; ++t) {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (on[t] && k0 + u < nseg) {
                        const float Mn = fmaxf(M[t], ml[t][u].x);
                        const float a = M[t] == -INFINITY ? 0.f : fast_exp2(M[t] - Mn);
                        const float b = fast_exp2(ml[t][u].x - Mn);
                        Lsum[t] = Lsum[t] * a + ml[t][u].y * b;
                        acc[t].x = acc[t].x * a + o[t][u].x * b;
                        acc[t].y = acc[t].y * a + o[t][u].y * b;
                        acc[t].z = acc[t].z * a + o[t][u].z * b;
                        acc[t].w = acc[t].w * a + o[t][u].w * b;
                        M[t] = Mn;
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < IT; ++t) {
            if (!on[t]) continue;
            const float inv = 1.f / Lsum[t];
            const size_t out = (row0[t] - static_cast<size_t>(c0) * p.nh) * D + static_cast<size_t>(col[t]) * 4;
            store_any(p.out, out + 0, p.out_dtype, acc[t].x * inv);
            store_any(p.out, out + 1, p.out_dtype, acc[t].y * inv);
            store_any(p.out, out + 2, p.out_dtype, acc[t].z * inv);
            store_any(p.out, out + 3, p.out_dtype, acc[t].w * inv);
        }
    }
}

// Fixed-split schedule: one warp per (sequence, head) whose context was split.
template <int D>
__global__ void __launch_bounds__(128) merge_splits_kernel(const AttnParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long idx = static_cast<long long>(blockIdx.x) * 4 + warp;
    if (idx >= static_cast<long long>(p.num_seqs) * p.nh) return;
    const int seq = static_cast<int>(idx / p.nh), hq = static_cast<int>(idx % p.nh);
    const int ntiles = tiles_of_len(p, p.lens[seq]);
    const int nsplit = (ntiles + p.split_tiles - 1) / p.split_tiles;
    if (nsplit <= 1) return;
    merge_rows<D>(p, static_cast<size_t>(seq) * p.max_splits * p.nh + hq, static_cast<size_t>(p.nh), nsplit,
                  (static_cast<size_t>(seq) * p.nh + hq) * D, lane);
}


// ---------------------------------------------------------------- kernels and launches of one variant
template <int D, int NT, class KV, bool QLO>
struct Kernels {
    static const void* decode() { return reinterpret_cast<const void*>(&paged_decode_kernel<D, NT, KV, QLO>); }
    static const void* streamk() { return reinterpret_cast<const void*>(&paged_decode_streamk_kernel<D, NT, KV, QLO>); }
};

template <class KV, bool QLO, int D>
const void* pick_d(int NT, bool streamk) {
    if (NT == 1) return streamk ? Kernels<D, 1, KV, QLO>::streamk() : Kernels<D, 1, KV, QLO>::decode();
    if constexpr (D <= 128) return streamk ? Kernels<D, 2, KV, QLO>::streamk() : Kernels<D, 2, KV, QLO>::decode();
    return nullptr;
}

template <class KV, bool QLO>
const void* pick_kv(int D, int NT, bool streamk) {
    switch (D) {
        case 32: return pick_d<KV, QLO, 32>(NT, streamk);
        case 64: return pick_d<KV, QLO, 64>(NT, streamk);
        case 96: return pick_d<KV, QLO, 96>(NT, streamk);
        case 128: return pick_d<KV, QLO, 128>(NT, streamk);
        case 256: return pick_d<KV, QLO, 256>(NT, streamk);
        default: return nullptr;
    }
}

template <int D>
int launch_merge(const kvp_attn_args& a, const kvpi::AttnPlan& pl, const AttnParams& prm, cudaStream_t stream) {
    const long long pairs = static_cast<long long>(a.num_seqs) * a.num_heads;
    if (pairs == 0) return KVP_OK;
    const unsigned blocks = static_cast<unsigned>((pairs + 3) / 4);
    if (pl.streamk || pl.max_splits <= 1) return KVP_OK;  // stream-K merges inside the attention kernel
    merge_splits_kernel<D><<<blocks, 128, 0, stream>>>(prm);
    return kvpi::cuda_status(cudaGetLastError(), "split merge kernel launch");
}

template <int D, int NT, class KV, bool QLO>
int launch_typed(const kvp_attn_args& a, const kvpi::AttnPlan& pl, const AttnParams& prm, const CUtensorMap& km,
                 const CUtensorMap& vm, cudaStream_t stream) {
    const void* fn = pl.streamk ? Kernels<D, NT, KV, QLO>::streamk() : Kernels<D, NT, KV, QLO>::decode();
    int rc = kvpi::allow_smem(fn);
    if (rc != KVP_OK) return rc;
    if (a.num_seqs == 0) return KVP_OK;
    dim3 block(static_cast<unsigned>((pl.kvh_cta * pl.wph + 1) * 32));
    if (pl.streamk) {
        dim3 grid(static_cast<unsigned>(pl.G), static_cast<unsigned>(pl.groups));
        if (a.flags & (KVP_ATTN_EARLY_START | KVP_ATTN_EARLY_LOAD)) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = grid;
            cfg.blockDim = block;
            cfg.dynamicSmemBytes = pl.smem;
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t e = cudaLaunchKernelEx(&cfg, paged_decode_streamk_kernel<D, NT, KV, QLO>, km, vm, prm);
            if (e != cudaSuccess) return kvpi::cuda_status(e, "attention kernel launch");
        } else {
            paged_decode_streamk_kernel<D, NT, KV, QLO><<<grid, block, pl.smem, stream>>>(km, vm, prm);
        }
    } else {
        dim3 grid(static_cast<unsigned>(a.num_seqs * pl.groups), static_cast<unsigned>(pl.max_splits));
        paged_decode_kernel<D, NT, KV, QLO><<<grid, block, pl.smem, stream>>>(km, vm, prm);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return kvpi::cuda_status(e, "attention kernel launch");
    return launch_merge<D>(a, pl, prm, stream);
}

template <int D, class KV, bool QLO>
int launch_nt(const kvp_attn_args& a, const kvpi::AttnPlan& pl, const AttnParams& prm, const CUtensorMap& km,
              const CUtensorMap& vm, cudaStream_t s) {
    if (prm.g <= 8) return launch_typed<D, 1, KV, QLO>(a, pl, prm, km, vm, s);
    if constexpr (D <= 128) return launch_typed<D, 2, KV, QLO>(a, pl, prm, km, vm, s);
    return kvpi::fail(KVP_EINVAL, "head_dim 256 supports at most 8 query heads per kv head");
}

template <class KV, bool QLO>
int launch_d(const kvp_attn_args& a, const kvpi::AttnPlan& pl, const AttnParams& prm, const CUtensorMap& km,
             const CUtensorMap& vm, cudaStream_t s) {
    switch (a.head_dim) {
        case 32: return launch_nt<32, KV, QLO>(a, pl, prm, km, vm, s);
        case 64: return launch_nt<64, KV, QLO>(a, pl, prm, km, vm, s);
        case 96: return launch_nt<96, KV, QLO>(a, pl, prm, km, vm, s);
        case 128: return launch_nt<128, KV, QLO>(a, pl, prm, km, vm, s);
        case 256: return launch_nt<256, KV, QLO>(a, pl, prm, km, vm, s);
        default: return kvpi::fail(KVP_EINVAL, "unsupported head_dim");
    }
}

// Defines the entry points of one variant (used once per instantiation translation unit).
#define KVPD_DEFINE_VARIANT(name, KV, QLO)                                                                     \
    const void* kernel_##name(int D, int NT, bool streamk) { return pick_kv<KV, QLO>(D, NT, streamk); }        \
    int launch_##name(const kvp_attn_args& a, const kvpi::AttnPlan& pl, const AttnParams& prm, const CUtensorMap& km, \
                      const CUtensorMap& vm, cudaStream_t s) {                                                 \
        return launch_d<KV, QLO>(a, pl, prm, km, vm, s);                                                       \
    }

}  // namespace kvpd
