// Host-side internals shared by the C-ABI translation units (not part of the public interface).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kvp_b200.h"
#include "kvpage/kv_manager.h"

// The C handle of a host control plane: one kvp::KVManager.
struct kvp_mgr {
    kvp::KVManager m;
    kvp_mgr(int nb, int bs) : m(nb, bs) {}
};

namespace kvpi {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const std::string& msg);
// Maps a CUDA error to KVP_ECUDA with a message naming `what`; KVP_OK for cudaSuccess.
int cuda_status(cudaError_t e, const char* what);
void clear_error();

inline int dtype_bytes(int dt) { return dt == KVP_DTYPE_F32 ? 4 : 2; }
inline bool valid_dtype(int dt) { return dt == KVP_DTYPE_F32 || dt == KVP_DTYPE_F16 || dt == KVP_DTYPE_BF16; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count();  // SMs of the current device (cached per device)

// Launch plan of the attention kernel, derived only from the arguments (so the workspace query and the
// launch agree).
struct AttnPlan {
    int R = 16;           // tokens per TMA run: gcd(block_size, 16)
    int nruns = 1;        // runs per 16-token tile
    int W = 64;           // elements per swizzled smem row (64: 128B swizzle, 32: 64B swizzle)
    int nch = 1;          // W-wide chunks per head_dim
    int kvh_cta = 1;      // kv heads per CTA (one consumer warp each)
    int groups = 1;       // kv_heads / kvh_cta
    int stages = 2;       // pipeline depth (16-token tiles in flight)
    int per_head = 0;     // 1: one TMA box per kv head (fallback tensor-map shape)
    int split_tiles = 1;  // tiles per CTA
    int max_tiles = 1;    // tiles of the longest possible sequence
    int max_splits = 1;
    uint32_t head_stride = 0, box_slot = 0, stage_half = 0, box_tx = 0;
    int streamk = 0;        // 1: persistent balanced schedule (grid of G CTAs per kv-head group)
    int G = 0;              // stream-K CTAs per group = SMs x resident CTAs per SM
    int wph = 1;            // consumer warps per kv head
    uint32_t q_area = 0;    // bytes of one of the two query slots (0: queries read from global memory)
    uint32_t stage_bytes = 0;
    uint32_t q_off = 0, comb_off = 0;  // offsets of the query slots and of the warp-combine area
    uint32_t pre_off = 0;   // stream-K: offset of the prefix sums
    int seq_units = 0;      // stream-K: start-cost units charged ahead of each sequence's tiles
    int taper_m = 0;        // stream-K: the last CTAs, which get fewer units (0: even split)
    int taper_d = 0;        // units each of them gives up
    size_t smem = 0, ws_bytes = 0;
    size_t ws_ml_off = 0;   // byte offset of the partial (m, l) pairs in the workspace
    size_t ws_o_off = 0;    // byte offset of the partial outputs in the workspace
    size_t ws_cnt_off = 0;  // stream-K: byte offset of the per-sequence segment counters (a fixed-size region)
};
int plan_attention(const kvp_attn_args& a, bool have_workspace, AttnPlan* plan);
// fp32 K/V pools: the CUDA-core kernel (attention_f32.cu); needs no workspace.
int launch_attention_f32(const kvp_attn_args& a, cudaStream_t s);

}  // namespace kvpi
