// Paged decode attention: host side -- launch planning, tensor maps, workspace, the C ABI entry point.  The
// kernels live in attention_kernels.cuh and are compiled by attention_inst_*.cu (one translation unit per
// K/V dtype x query residual).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "attention_common.h"
#include "kvp_device.cuh"

// ============================================================================ host side
namespace kvpi {

namespace {

int gcd_int(int a, int b) {
    while (b) {
        const int t = a % b;
        a = b;
        b = t;
    }
    return a;
}
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
// Dynamic shared memory a CTA may use: the 227 KB opt-in limit less 1 KB for the static barriers.
constexpr int kDynSmemCap = (227 << 10) - 1024;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Tensor map over one layer's pool.  per_head == 0: dims (head_dim, rows = num_blocks*B, kv_heads), box
// (W, R, kvh_cta) -> smem [kvh][R][W].  per_head == 1: dims (head_dim, kv_heads, rows), box (W, 1, R).
int encode_pool_map(CUtensorMap* map, const void* base, int kv_dtype, const kvp_attn_args& a, const AttnPlan& pl,
                    long long rows, int per_head) {
    auto fn = encode_fn();
    if (!fn) return fail(KVP_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const CUtensorMapDataType dt =
        kv_dtype == KVP_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t D = static_cast<uint64_t>(a.head_dim), H = static_cast<uint64_t>(a.kv_heads);
    cuuint64_t dims[3];
    cuuint64_t strides[2];
    cuuint32_t box[3];
    const cuuint32_t estr[3] = {1, 1, 1};
    if (!per_head) {
        dims[0] = D;
        dims[1] = static_cast<cuuint64_t>(rows);
        dims[2] = H;
        strides[0] = H * D * 2;
        strides[1] = D * 2;
        box[0] = static_cast<cuuint32_t>(pl.W);
        box[1] = static_cast<cuuint32_t>(pl.R);
        box[2] = static_cast<cuuint32_t>(pl.kvh_cta);
    } else {
        dims[0] = D;
        dims[1] = H;
        dims[2] = static_cast<cuuint64_t>(rows);
        strides[0] = D * 2;
        strides[1] = H * D * 2;
        box[0] = static_cast<cuuint32_t>(pl.W);
        box[1] = 1;
        box[2] = static_cast<cuuint32_t>(pl.R);
    }
    const CUtensorMapSwizzle sw = pl.W == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KVP_ECUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(r));
    return KVP_OK;
}

// Which tensor-map shape the driver accepts: the 3-D (D, rows, heads) form with one box for all heads of
// a CTA, or the per-head fallback.  Probed once per process with a dummy (host-only) encode.
int pool_map_mode() {
    static int mode = -1;
    static std::once_flag once;
    std::call_once(once, [] {
        auto fn = encode_fn();
        mode = 1;
        if (!fn) return;
        alignas(64) CUtensorMap m;
        static __align__(256) unsigned char dummy[1 << 16];
        cuuint64_t dims[3] = {128, 64, 8};
        cuuint64_t strides[2] = {8 * 128 * 2, 128 * 2};
        cuuint32_t box[3] = {64, 16, 8};
        cuuint32_t estr[3] = {1, 1, 1};
        if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dummy, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
            mode = 0;
    });
    return mode;
}

}  // namespace

// Opts a kernel into the whole dynamic shared-memory budget, once per device.
int allow_smem(const void* fn) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == fn && d.second == dev) return KVP_OK;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmemCap);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention)");
    done.emplace_back(fn, dev);
    return KVP_OK;
}

namespace {

// Resident CTAs per SM of the stream-K kernel for this launch shape (occupancy API; shared-memory estimate
// when no device is present, e.g. for a workspace query on a build machine).
// Cached per (kernel, threads, smem, device): the occupancy query costs far more than a launch.
int streamk_ctas_per_sm(const void* fn, int threads, size_t smem) {
    struct Key {
        const void* fn;
        int threads;
        size_t smem;
        int dev;
        int n;
    };
    static std::mutex mu;
    static std::vector<Key> cache;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto& k : cache)
            if (k.fn == fn && k.threads == threads && k.smem == smem && k.dev == dev) return k.n;
    }
    int n = 0;
    if (!(fn && dev >= 0 && allow_smem(fn) == KVP_OK &&
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) == cudaSuccess && n > 0)) {
        cudaGetLastError();
        n = std::max(1, static_cast<int>((228u << 10) / (smem + 1024)));
    }
    std::lock_guard<std::mutex> lock(mu);
    cache.push_back(Key{fn, threads, smem, dev, n});
    return n;
}

// The kernel of a (kv dtype, query dtype, head_dim, group size, schedule) combination.  The query's low-half
// residual MMA is compiled in only when the query dtype differs from the K/V dtype.
const void* pick_kernel(int kv_dtype, int q_dtype, int D, int g, bool streamk) {
    const int NT = g <= 8 ? 1 : 2;
    const bool qres = q_dtype != kv_dtype;
    if (kv_dtype == KVP_DTYPE_F16) return qres ? kvpd::kernel_f16_qres(D, NT, streamk) : kvpd::kernel_f16(D, NT, streamk);
    return qres ? kvpd::kernel_bf16_qres(D, NT, streamk) : kvpd::kernel_bf16(D, NT, streamk);
}

}  // namespace

int plan_attention(const kvp_attn_args& a, bool have_workspace, AttnPlan* out) {
    AttnPlan pl;
    const int D = a.head_dim;
    if (!(D == 32 || D == 64 || D == 96 || D == 128 || D == 256))
        return fail(KVP_EINVAL, "head_dim must be one of 32, 64, 96, 128, 256");
    if (a.kv_heads <= 0 || a.num_heads <= 0 || a.num_heads % a.kv_heads != 0)
        return fail(KVP_EINVAL, "num_heads % kv_heads != 0");
    const int g = a.num_heads / a.kv_heads;
    if (g > 16) return fail(KVP_EINVAL, "more than 16 query heads per kv head are not supported");
    if (g > 8 && D > 128) return fail(KVP_EINVAL, "head_dim 256 supports at most 8 query heads per kv head");
    if (a.block_size < 1 || a.max_blocks < 1 || a.num_seqs < 0) return fail(KVP_EINVAL, "bad block_size / max_blocks / num_seqs");
    pl.R = gcd_int(a.block_size, 16);
    pl.nruns = 16 / pl.R;
    pl.W = (D % 64 == 0) ? 64 : 32;
    pl.nch = D / pl.W;
    pl.per_head = pool_map_mode();
    const size_t rowb = static_cast<size_t>(pl.W) * 2;
    // kv heads per CTA: largest divisor of kv_heads <= 8 whose stage fits 64 KB (or the caller's choice).
    int kc = a.kv_heads_per_cta;
    if (kc <= 0 || kc > kvpd::kMaxKvhPerCta || a.kv_heads % kc != 0) {
        kc = 1;
        for (int d = 1; d <= std::min(a.kv_heads, kvpd::kMaxKvhPerCta); ++d)
            if (a.kv_heads % d == 0 && static_cast<size_t>(d) * 16 * D * 2 * 2 <= (64u << 10)) kc = d;
    }
    pl.kvh_cta = kc;
    pl.groups = a.kv_heads / kc;
    if (!pl.per_head) {
        pl.head_stride = static_cast<uint32_t>(pl.R * rowb);
        pl.box_slot = static_cast<uint32_t>(round_up(static_cast<size_t>(kc) * pl.R * rowb, 1024));
    } else {
        pl.head_stride = static_cast<uint32_t>(round_up(pl.R * rowb, 1024));
        pl.box_slot = static_cast<uint32_t>(kc) * pl.head_stride;
    }
    pl.box_tx = static_cast<uint32_t>(static_cast<size_t>(kc) * pl.R * rowb);
    pl.stage_half = static_cast<uint32_t>(pl.nruns) * pl.nch * pl.box_slot;
    pl.max_tiles = static_cast<int>((static_cast<long long>(a.max_blocks) * a.block_size + 15) / 16);

    // Schedule: stream-K when splitting is automatic and a workspace is available; otherwise fixed splits.
    pl.streamk = (a.split_tiles == 0 && have_workspace && a.num_seqs > 0 && a.num_seqs <= kvpd::kMaxStreamSeqs) ? 1 : 0;
    // Consumer warps per kv head: fill 8 consumer warps per CTA, so small groups still have enough warps in
    // flight to hide the per-tile latency -- as many as the shared memory of the smallest ring allows.
    const size_t qelem = a.q_dtype == KVP_DTYPE_F32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(a.q) & 15u) == 0)
        pl.q_area = static_cast<uint32_t>(round_up(static_cast<size_t>(kc) * g * D * qelem, 128));
    pl.stage_bytes = 2u * pl.stage_half;
    const size_t stage = pl.stage_bytes;
    const int NT = g <= 8 ? 1 : 2;
    const size_t pre = pl.streamk ? round_up((static_cast<size_t>(a.num_seqs) + 1) * 4 + a.num_seqs, 128) : 0;
    const size_t smem_cap = kDynSmemCap;
    size_t comb = 0;
    auto total = [&](int wph, int k) {
        comb = static_cast<size_t>(wph - 1) * kc * 32 * (NT * (D / 16) * 4 + NT * 4) * sizeof(float);
        return round_up(stage * wph * k, 128) + 2 * static_cast<size_t>(pl.q_area) + round_up(comb, 16) + pre + 1024;
    };
    auto min_per = [](int wph) { return wph == 1 ? 2 : 1; };
    // Measured on B200: two warps per kv head help when a CTA serves at most two kv heads, one is best otherwise.
    pl.wph = kc <= 2 ? 2 : 1;
    if (a.warps_per_kv_head > 0) pl.wph = std::min(a.warps_per_kv_head, std::max(1, kvpd::kMaxConsumerWarps / kc));
    while (pl.wph > 1 && total(pl.wph, min_per(pl.wph)) > smem_cap) --pl.wph;
    if (total(pl.wph, min_per(pl.wph)) > smem_cap) {
        if (total(1, 1) > smem_cap) return fail(KVP_EINVAL, "shape needs more shared memory than a CTA has");
    }
    // Stages: a multiple of wph (each stage keeps the same consumers); a ring of about 192 KB for large stages
    // (three 64 KB stages measured best for 8 kv heads x D=128, one CTA per SM) and about 96 KB for small ones
    // (two CTAs per SM measured better than a deeper ring); at least two per consumer when one warp serves
    // each head (when the shared memory allows).
    const size_t ring = stage >= (48u << 10) ? (192u << 10) : (96u << 10);  // small stages: 2 CTAs per SM
    int per = a.stages > 0 ? std::max(1, a.stages / pl.wph)
                           : static_cast<int>(std::max<size_t>(min_per(pl.wph), ring / (stage * pl.wph)));
    per = std::min(per, kvpd::kMaxStages / pl.wph);
    while (per > 1 && total(pl.wph, per) > smem_cap) --per;
    if (total(pl.wph, per) > smem_cap) return fail(KVP_EINVAL, "shape needs more shared memory than a CTA has");
    pl.smem = total(pl.wph, per);
    pl.stages = per * pl.wph;
    pl.q_off = static_cast<uint32_t>(round_up(stage * pl.stages, 128));
    pl.comb_off = pl.q_off + 2 * pl.q_area;
    pl.pre_off = static_cast<uint32_t>(pl.comb_off + round_up(comb, 16));

    if (pl.streamk) {
        const void* fn = pick_kernel(a.kv_dtype, a.q_dtype, D, g, true);
        pl.G = sm_count() * streamk_ctas_per_sm(fn, (kc * pl.wph + 1) * 32, pl.smem);
        // The partition of a step depends on the grid once a step has more units than CTAs.  Block sizes that
        // are not multiples of 16 pad their stages (more shared memory, fewer resident CTAs), so they take the
        // grid of the 16-token layout: the same contexts give the same partition -- and bit-identical results
        // -- in every block size.  CTAs beyond residency simply start later (no CTA waits on another).
        if (pl.R != 16) {
            kvp_attn_args b = a;
            b.block_size = 16;
            b.max_blocks = pl.max_tiles;
            AttnPlan p16;
            if (plan_attention(b, have_workspace, &p16) == KVP_OK && p16.streamk) pl.G = p16.G;
        }
        // A sequence switch (query load, state reset, segment epilogue, and with two warps per kv head their
        // state combine) costs a CTA about 3.8 us, 6.8 us with two warps per head (the optima of start-cost
        // sweeps on B200 for the Qwen2.5-0.5B, TinyLlama and Llama-3-8B shapes, with each launch's successor
        // scheduled from its start); charge it in tiles: a tile's
        // time at the full bandwidth shared by the CTAs of one SM.  Only quantities independent of the block
        // size enter (the tile's K/V bytes, one CTA per SM for 48 KB tiles or more, else two), so every block
        // size and placement of the same contexts gets the same partition -- and bit-identical results.
        if (a.seq_start_tiles > 0) {
            pl.seq_units = std::min(a.seq_start_tiles, 1024);
        } else if (a.seq_start_tiles == 0) {
            const double tile_bytes = 16.0 * kc * D * 2 * 2;
            const double ctas = static_cast<double>(sm_count()) * (tile_bytes >= (48 << 10) ? 1 : 2);
            const double switch_us = pl.wph > 1 ? 6.8 : 3.8;
            const double tile_us = tile_bytes * ctas / 6.4e6;
            pl.seq_units = static_cast<int>(std::min(32.0, std::max(0.0, std::round(switch_us / tile_us))));
        }
        // Back-to-back launches (a step's layers) see their last-dispatched CTAs start late: they get the SM slots
        // the previous grid frees last and run their whole prologue after it ends.  A per-CTA timeline of
        // graph-replayed steps on B200 (Qwen2.5-0.5B and TinyLlama shapes, 296 CTAs) put the CTAs from about the
        // last sixth of the index range behind, by 1 to 5 us at their first tile.  Those CTAs get about 3 us worth
        // of tiles fewer each (tile time as for the start cost above), spread over all CTAs; linear ramps from
        // 3 to 8 us and over a tenth to a quarter of the grid measured the same.  Applied to every balanced
        // launch, so the partition -- and the result, bit for bit -- depends only on the lengths and the head
        // shape, not on how the launch is ordered against its neighbours.
        {
            const double tile_bytes = 16.0 * kc * D * 2 * 2;
            const double ctas = static_cast<double>(sm_count()) * (tile_bytes >= (48 << 10) ? 1 : 2);
            const double tile_us = tile_bytes * ctas / 6.4e6;
            pl.taper_m = std::max(1, static_cast<int>(std::lround(pl.G / 6.0)));
            pl.taper_d = static_cast<int>(std::lround(3.0 / tile_us));
        }
        pl.split_tiles = pl.max_tiles;
        pl.max_splits = 1;
        // The merge counters come first, in a region sized for the most sequences a call may have, so their
        // place does not depend on num_seqs: a workspace left clean by one call is clean for the next call of
        // the same head shape whatever its batch size (the partials behind them need no initial value).
        const size_t rows = (static_cast<size_t>(pl.G) + a.num_seqs) * a.num_heads;
        pl.ws_cnt_off = 0;
        pl.ws_ml_off = round_up(static_cast<size_t>(kvpd::kMaxStreamSeqs) * pl.groups * 4, 256);
        pl.ws_o_off = pl.ws_ml_off + round_up(rows * sizeof(float2), 256);
        pl.ws_bytes = pl.ws_o_off + round_up(rows * static_cast<size_t>(D) * sizeof(float), 256);
        *out = pl;
        return KVP_OK;
    }
    int split = pl.max_tiles;
    if (a.split_tiles > 0) split = std::min(a.split_tiles, pl.max_tiles);
    pl.split_tiles = std::max(1, split);
    pl.max_splits = (pl.max_tiles + pl.split_tiles - 1) / pl.split_tiles;
    if (pl.max_splits > 65535) return fail(KVP_EINVAL, "too many context splits; raise split_tiles");
    pl.ws_bytes = 0;
    if (pl.max_splits > 1) {
        const size_t rows = static_cast<size_t>(a.num_seqs) * pl.max_splits * a.num_heads;
        pl.ws_o_off = round_up(rows * sizeof(float2), 256);
        pl.ws_bytes = pl.ws_o_off + rows * static_cast<size_t>(D) * sizeof(float);
    }
    *out = pl;
    return KVP_OK;
}

}  // namespace kvpi

extern "C" KVP_API size_t kvp_attention_workspace_size(const kvp_attn_args* a) {
    if (!a || a->kv_dtype == KVP_DTYPE_F32) return 0;
    kvpi::AttnPlan pl;
    if (kvpi::plan_attention(*a, true, &pl) != KVP_OK) return 0;
    return pl.ws_bytes;
}

namespace {

// kvp_paged_attention with every pipeline wait limited to `wait_limit` clock cycles; `stall` arms the first stage
// of the CTAs in the grid's first row for a copy that is never issued (kvp_attention_wait_test only).
int attention_call(const kvp_attn_args* a, void* stream, long long wait_limit, int stall) {
    using namespace kvpi;
    clear_error();
    if (!a) return fail(KVP_EINVAL, "null arguments");
    if (!valid_dtype(a->q_dtype) || !valid_dtype(a->out_dtype) || !valid_dtype(a->kv_dtype))
        return fail(KVP_EINVAL, "unsupported dtype");
    if (a->num_seqs > 0 && (!a->q || !a->k_cache || !a->v_cache || !a->block_tables || !a->seq_lens || !a->out))
        return fail(KVP_EINVAL, "null buffer");
    if (a->kv_dtype == KVP_DTYPE_F32) return launch_attention_f32(*a, static_cast<cudaStream_t>(stream));
    if (!aligned16(a->k_cache) || !aligned16(a->v_cache)) return fail(KVP_EINVAL, "K/V pools must be 16-byte aligned");
    if ((a->k_new == nullptr) != (a->v_new == nullptr)) return fail(KVP_EINVAL, "k_new and v_new go together");
    if (a->k_new) {
        if (!aligned16(a->k_new) || !aligned16(a->v_new)) return fail(KVP_EINVAL, "k_new / v_new must be 16-byte aligned");
        if (a->num_blocks <= 0) return fail(KVP_EINVAL, "the fused append needs num_blocks (it bounds the written slot)");
    }
    if ((reinterpret_cast<uintptr_t>(a->inputs_ready) | reinterpret_cast<uintptr_t>(a->inputs_epoch)) & 3u)
        return fail(KVP_EINVAL, "inputs_ready / inputs_epoch must be 4-byte aligned");
    AttnPlan pl;
    int rc = plan_attention(*a, a->workspace != nullptr, &pl);
    if (rc != KVP_OK) return rc;
    if (pl.ws_bytes > 0) {
        if (!a->workspace || a->workspace_bytes < pl.ws_bytes)
            return fail(KVP_ENOSPACE, "workspace smaller than kvp_attention_workspace_size()");
        if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0) return fail(KVP_EINVAL, "workspace must be 256-byte aligned");
    }
    // Rows of the tensor map: the whole pool when its size is known (TMA then zero-fills anything
    // outside it); otherwise the largest extent a 32-bit row coordinate can address.
    long long rows;
    if (a->num_blocks > 0) {
        rows = a->num_blocks * static_cast<long long>(a->block_size);
        if (rows > 0x7fffffffLL) return fail(KVP_EINVAL, "num_blocks * block_size must stay below 2^31");
    } else {
        rows = 0x7fffffffLL / a->block_size * a->block_size;
    }
    alignas(64) CUtensorMap km, vm;
    rc = encode_pool_map(&km, a->k_cache, a->kv_dtype, *a, pl, rows, pl.per_head);
    if (rc != KVP_OK) return rc;
    rc = encode_pool_map(&vm, a->v_cache, a->kv_dtype, *a, pl, rows, pl.per_head);
    if (rc != KVP_OK) return rc;

    kvpd::AttnParams prm;
    std::memset(&prm, 0, sizeof(prm));
    prm.q = a->q;
    prm.tables = a->block_tables;
    prm.lens = a->seq_lens;
    prm.out = a->out;
    if (pl.ws_bytes > 0) {
        char* ws = static_cast<char*>(a->workspace);
        prm.ws_ml = reinterpret_cast<float2*>(ws + pl.ws_ml_off);
        prm.ws_o = reinterpret_cast<float*>(ws + pl.ws_o_off);
        if (pl.streamk) {
            prm.counters = reinterpret_cast<int32_t*>(ws + pl.ws_cnt_off);
            // The counters must start at zero; every completed call leaves them zero again.
            if (!(a->flags & KVP_ATTN_WORKSPACE_CLEAN)) {
                const cudaError_t e = cudaMemsetAsync(prm.counters, 0, static_cast<size_t>(a->num_seqs) * pl.groups * 4,
                                                      static_cast<cudaStream_t>(stream));
                if (e != cudaSuccess) return cuda_status(e, "workspace counter reset");
            }
        }
    }
    prm.status = a->status;
    prm.num_blocks = a->num_blocks > 0 ? a->num_blocks : 0;
    prm.q_dtype = a->q_dtype;
    prm.out_dtype = a->out_dtype;
    prm.num_seqs = a->num_seqs;
    prm.nh = a->num_heads;
    prm.g = a->num_heads / a->kv_heads;
    prm.max_blocks = a->max_blocks;
    prm.B = a->block_size;
    prm.R = pl.R;
    prm.nruns = pl.nruns;
    prm.kvh_cta = pl.kvh_cta;
    prm.groups = pl.groups;
    prm.stages = pl.stages;
    prm.split_tiles = pl.split_tiles;
    prm.max_splits = pl.max_splits;
    prm.per_head = pl.per_head;
    prm.G = pl.G;
    prm.head_stride = pl.head_stride;
    prm.box_slot = pl.box_slot;
    prm.stage_half = pl.stage_half;
    prm.box_tx = pl.box_tx;
    prm.stage_bytes = pl.stage_bytes;
    prm.q_area = pl.q_area;
    prm.q_off = pl.q_off;
    prm.comb_off = pl.comb_off;
    prm.pre_off = pl.pre_off;
    prm.wph = pl.wph;
    prm.oob_row = static_cast<int>(std::min<long long>(rows, 0x7fffffffLL));
    prm.Bshift = -1;
    if ((a->block_size & (a->block_size - 1)) == 0)
        for (int b = 0; (1 << b) <= a->block_size; ++b)
            if ((1 << b) == a->block_size) prm.Bshift = b;
    prm.k_new = a->k_new;
    prm.v_new = a->v_new;
    prm.k_pool = const_cast<void*>(a->k_cache);
    prm.v_pool = const_cast<void*>(a->v_cache);
    prm.kvh = a->kv_heads;
    prm.early_load = (a->flags & KVP_ATTN_EARLY_LOAD) ? 1 : 0;
    prm.seq_units = pl.seq_units;
    prm.taper_m = pl.taper_m;
    prm.taper_d = pl.taper_d;
    prm.wait_limit = wait_limit;
    prm.stall_first_stage = stall;
    prm.inputs_ready = a->inputs_ready;
    prm.inputs_epoch = a->inputs_ready ? a->inputs_epoch : nullptr;
    const float scale = a->scale > 0.f ? a->scale : 1.0f / std::sqrt(static_cast<float>(a->head_dim));
    prm.sl2 = scale * 1.4426950408889634f;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool qres = a->q_dtype != a->kv_dtype;
    if (a->kv_dtype == KVP_DTYPE_F16)
        return qres ? kvpd::launch_f16_qres(*a, pl, prm, km, vm, s) : kvpd::launch_f16(*a, pl, prm, km, vm, s);
    return qres ? kvpd::launch_bf16_qres(*a, pl, prm, km, vm, s) : kvpd::launch_bf16(*a, pl, prm, km, vm, s);
}

}  // namespace

extern "C" KVP_API int kvp_paged_attention(const kvp_attn_args* a, void* stream) {
    return attention_call(a, stream, kvpd::kWaitLimitCycles, 0);
}

extern "C" KVP_API int kvp_attention_wait_test(const kvp_attn_args* a, void* stream, int64_t wait_limit_cycles,
                                               int32_t stall_first_stage) {
    if (wait_limit_cycles < 1 || wait_limit_cycles > kvpd::kWaitLimitCycles || stall_first_stage < 0 ||
        stall_first_stage > 1) {
        kvpi::clear_error();
        return kvpi::fail(KVP_EINVAL, "wait limit must be in [1, 2e9] cycles and stall_first_stage 0 or 1");
    }
    return attention_call(a, stream, wait_limit_cycles, stall_first_stage);
}
