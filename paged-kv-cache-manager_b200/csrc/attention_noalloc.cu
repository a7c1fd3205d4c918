// Paged decode attention for callers that cannot allocate device memory.
//
// kvp_paged_attention keeps the per-split partial results of long contexts (m, l and the unnormalised
// output of every split) in a workspace the caller allocates.  Some callers have no way to do that: a
// serving engine whose memory manager reserves nearly all of HBM for the KV pool up front and offers
// libraries no allocation hook, or a plugin interface whose enqueue callback must not allocate (a
// cudaMalloc there can stall every stream on the device while the allocator synchronises).  For them,
// kvp_paged_attention_noalloc runs the same kernels with the partials in a fixed array compiled into this
// library, so the call itself allocates nothing.
//
// The array is KVP_NOALLOC_SCRATCH_BYTES (32 MiB) of device memory that every GPU which loads the library
// holds until the process exits.  Its device address is looked up on the first call made in each CUDA context
// (the first call on a device, and again after cudaDeviceReset or a re-created primary context gives the
// device a new context, where the module -- and the array -- may sit at a new address), so that first call
// should come before any stream capture.  All calls share the
// array and it keeps whatever the last call left there: the only words that must start at zero, the merge
// counters of the balanced schedule, are cleared on the stream by every call (every split writes its partials
// before the merge reads them), and two calls that overlap on the GPU -- on different streams, or from
// different threads -- race on it and must be serialised by the caller.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "kvp_b200.h"
#include "kvp_internal.h"

namespace {

constexpr size_t kScratchBytes = KVP_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Split-K partials of kvp_paged_attention_noalloc.  In host code this name is only a stand-in for the
// device symbol: it is never dereferenced or passed to a kernel directly; the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_split_scratch[kScratchBytes];

// The scratch address found for a device, and the unique id of the context it was found in.
struct ScratchEntry {
    unsigned long long ctx_id = 0;
    void* addr = nullptr;
};
ScratchEntry g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the current context (0 when there is none yet, or the driver cannot say).
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(f);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(f);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS) return id;
    return 0;
}

// Device address of the scratch array in the current context: looked up on the first call in each context
// (without a context id from the driver, on every call).
int scratch_address(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return kvpi::cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return kvpi::fail(KVP_EINVAL, "device index outside the supported range");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    unsigned long long id = current_context_id();
    if (id == 0 || g_scratch[dev].ctx_id != id || !g_scratch[dev].addr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_split_scratch);  // also makes the device's primary context current
        if (e != cudaSuccess) return kvpi::cuda_status(e, "cudaGetSymbolAddress(split scratch)");
        if (id == 0) id = current_context_id();
        g_scratch[dev].ctx_id = id;
        g_scratch[dev].addr = p;
    }
    *out = g_scratch[dev].addr;
    return KVP_OK;
}

}  // namespace

extern "C" KVP_API int kvp_paged_attention_noalloc(const kvp_attn_args* a, void* stream) {
    kvpi::clear_error();
    if (!a) return kvpi::fail(KVP_EINVAL, "null arguments");
    void* scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc != KVP_OK) return rc;
    kvp_attn_args b = *a;
    b.workspace = scratch;
    b.workspace_bytes = kScratchBytes;
    // The shared array may hold another call's partials where this call keeps its merge counters (a call with
    // fixed splits puts partials there), so the counters are always cleared on the stream, never assumed clean.
    b.flags &= ~KVP_ATTN_WORKSPACE_CLEAN;
    size_t need = kvp_attention_workspace_size(&b);
    if (need > kScratchBytes) {
        if (a->split_tiles != 0)
            return kvpi::fail(KVP_ENOSPACE, "split partials need " + std::to_string(need) +
                                                " bytes but the no-allocation scratch holds " +
                                                std::to_string(kScratchBytes) +
                                                "; raise split_tiles or pass fewer sequences per call");
        // Automatic splitting: coarsen the splits until their partials fit (one split per sequence
        // needs no scratch at all).
        for (int s = 16; need > kScratchBytes && s < (1 << 30); s *= 2) {
            b.split_tiles = s;
            need = kvp_attention_workspace_size(&b);
        }
    }
    return kvp_paged_attention(&b, stream);
}
