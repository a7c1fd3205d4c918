// Launch parameters of the paged-attention kernels, shared by the host planner (attention.cu) and the kernel
// translation units (attention_inst_*.cu, one per kv dtype x query residual, compiled in parallel).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kvp_internal.h"

namespace kvpi {
// Opts a kernel into the whole dynamic shared-memory budget, once per device.
int allow_smem(const void* fn);
}  // namespace kvpi

namespace kvpd {

constexpr int kMaxStages = 16;
constexpr int kMaxConsumerWarps = 8;
constexpr int kMaxKvhPerCta = 8;
constexpr int kMaxStreamSeqs = 8192;  // stream-K keeps the tile prefix sums of all sequences in smem

struct AttnParams {
    const void* q;
    const int32_t* tables;
    const int32_t* lens;
    void* out;
    float2* ws_ml;   // partial (m in log2 units, l) rows of nh heads
    float* ws_o;     // partial unnormalised outputs, D per row
    int32_t* counters;  // stream-K: [num_seqs][groups] finished-segment counters (zero between calls)
    int32_t* status;
    long long num_blocks;  // 0: unchecked
    int q_dtype, out_dtype;
    int num_seqs, nh, g, max_blocks, B, R, nruns;
    int kvh_cta, groups, stages, split_tiles, max_splits, per_head;
    int G;                 // stream-K CTAs per kv-head group
    int wph;               // consumer warps per kv head (they take turns over the stages)
    uint32_t head_stride, box_slot, stage_half, box_tx;
    uint32_t stage_bytes;  // stride between stages (2 * stage_half)
    uint32_t q_area;       // bytes of one query slot (0: queries read from global memory)
    uint32_t q_off;        // offset of the two query slots in dynamic smem
    uint32_t comb_off;     // offset of the warp-combine area in dynamic smem
    uint32_t pre_off;      // stream-K: offset of the prefix sums in dynamic smem
    int oob_row;           // a row coordinate outside the tensor map (zero fill) used for skipped blocks
    int Bshift;            // log2(block_size) when it is a power of two, else -1
    float sl2;             // scale * log2(e)
    // Fused append (null when off): [num_seqs][kvh][D] K/V of each sequence's newest token, written into the
    // pools at position len - 1 before the tile that holds it is loaded.
    const void* k_new;
    const void* v_new;
    void* k_pool;
    void* v_pool;
    int kvh;
    int early_load;  // the producer may load the first K/V tiles before waiting for the previous kernel
    int seq_units;   // stream-K: start-cost units charged ahead of each sequence's tiles
    // Stream-K taper: the last taper_m CTAs -- dispatched last, into the SM slots the previous grid frees last
    // when launches run back to back -- get taper_d fewer units each; 0: even split.
    int taper_m;
    int taper_d;
    long long wait_limit;  // clock cycles after which a pipeline wait gives up (KVP_STATUS_TIMEOUT)
    // Failure-detection test (kvp_attention_wait_test): the producer of every CTA with blockIdx.y == 0 arms stage 0
    // for 16 bytes of a copy it never issues and starts its tiles at stage 1, so the consumers' first wait runs
    // out; nothing is ever in flight for stage 0.
    int stall_first_stage;
    // Inputs produced by copies on another stream (null: none): the queries and the fused append's new K/V are
    // read only once this word is non-zero -- or, with inputs_epoch, once (word - *inputs_epoch) >= 0 as a
    // 32-bit signed difference (bounded wait, KVP_STATUS_TIMEOUT).
    const int32_t* inputs_ready;
    const int32_t* inputs_epoch;
};

// Per-CTA pipeline state in shared memory: `abort` is raised by a consumer warp whose wait gave up, so the
// producer drains its copies before it returns even when its own waits all succeeded.
struct PipeState {
    int abort;
};

// Per-variant entry points: K/V dtype x whether the query needs a low-half residual MMA (its dtype differs
// from the K/V dtype).  kernel_*: the kernel for (head_dim, n-tiles, schedule); launch_*: a planned call.
#define KVPD_DECLARE_VARIANT(name)                                                                              \
    const void* kernel_##name(int D, int NT, bool streamk);                                                    \
    int launch_##name(const kvp_attn_args& a, const kvpi::AttnPlan& pl, const AttnParams& prm, const CUtensorMap& km, \
                      const CUtensorMap& vm, cudaStream_t s);
KVPD_DECLARE_VARIANT(f16)
KVPD_DECLARE_VARIANT(f16_qres)
KVPD_DECLARE_VARIANT(bf16)
KVPD_DECLARE_VARIANT(bf16_qres)
#undef KVPD_DECLARE_VARIANT

}  // namespace kvpd
