// Device helpers shared by the kernels: mbarrier pipeline primitives with bounded waits, TMA tiled and
// bulk copies (each CTA loads only into its own shared memory), warp-level tensor-core fragments (ldmatrix / movmatrix /
// mma.sync m16n8k16 with fp32 accumulate), and 16-bit float conversions.  sm_100a only.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "kvp_b200.h"

namespace kvpd {

// ---------------------------------------------------------------- 16-bit storage types
template <class T>
struct F16Traits;
template <>
struct F16Traits<__half> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float unpack_lo(uint32_t v) {
        return __low2float(*reinterpret_cast<__half2*>(&v));
    }
    static __device__ __forceinline__ float unpack_hi(uint32_t v) {
        return __high2float(*reinterpret_cast<__half2*>(&v));
    }
    static __device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};
template <>
struct F16Traits<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float unpack_lo(uint32_t v) {
        return __low2float(*reinterpret_cast<__nv_bfloat162*>(&v));
    }
    static __device__ __forceinline__ float unpack_hi(uint32_t v) {
        return __high2float(*reinterpret_cast<__nv_bfloat162*>(&v));
    }
    static __device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

// Loads element i of a q/out style buffer of runtime dtype as float.
__device__ __forceinline__ float load_any(const void* p, size_t i, int dtype) {
    if (dtype == KVP_DTYPE_F32) return reinterpret_cast<const float*>(p)[i];
    if (dtype == KVP_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void store_any(void* p, size_t i, int dtype, float x) {
    if (dtype == KVP_DTYPE_F32)
        reinterpret_cast<float*>(p)[i] = x;
    else if (dtype == KVP_DTYPE_F16)
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
    else
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void report(int32_t* status, int bits) {
    if (status) atomicOr(status, bits);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Device-scope fetch-and-add with acquire-release semantics: releases the writes ordered before it (other
// threads' writes included when a CTA barrier orders them before it) and acquires those released by the
// earlier adders.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* addr, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
    return old;
}

// Programmatic dependent launch.  griddep_wait: blocks until the previous kernel on the stream has completed
// and its memory is visible (returns at once when the kernel was launched without the programmatic
// serialization attribute).  griddep_launch_dependents: lets the next kernel on the stream start its own
// prologue once every CTA of this grid has called it or exited (its griddep_wait still waits for this grid).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Orders this thread's generic-proxy global stores before later async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Bounded wait of a whole warp until *flag != 0 -- or, with `epoch`, until *flag - *epoch >= 0 as a signed
// 32-bit difference -- a word a copy on another stream writes after the data it guards: every lane's acquire
// load at GPU scope orders its own later reads, and the proxy fence the bulk copies issued next.  False when
// `limit` clock cycles passed first.
__device__ __forceinline__ bool warp_wait_flag(const int32_t* flag, const int32_t* epoch, long long limit) {
    const long long t0 = clock64();
    const uint32_t e = epoch ? static_cast<uint32_t>(__ldcg(epoch)) : 0u;
    for (unsigned ns = 32;; ns = ns < 1024 ? 2 * ns : ns) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        const bool ready = epoch ? static_cast<int32_t>(static_cast<uint32_t>(v) - e) >= 0 : v != 0;
        if (__all_sync(0xffffffffu, ready)) break;
        if (__any_sync(0xffffffffu, clock64() - t0 > limit)) return false;
        __nanosleep(ns);
    }
    fence_proxy_async_global();
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for phase `parity` of the barrier to complete.  Gives up after about `limit` clock cycles
// (kWaitLimitCycles: roughly a second at B200 clocks) and returns false, so a broken pipeline ends the kernel
// with an error status instead of hanging the GPU.
constexpr long long kWaitLimitCycles = 2000000000LL;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > limit) return false;
    }
}

// ---------------------------------------------------------------- TMA (destination: this CTA only)
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- warp MMA fragments
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// D += A * B, m16n8k16, fp32 accumulate.  A: 4 regs (row-major 16x16), B: 2 regs (col-major 16x8).
template <class T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace kvpd
