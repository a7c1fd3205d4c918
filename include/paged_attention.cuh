// Drop-in replacement for the reference's GPU entry point (cuda/paged_attention.cuh:16-19 of
// prathameshpranjale/paged-kv-cache-manager): same name, arguments and error behaviour.
//
// fp16 q / k_cache / v_cache / out, fp32 math; layouts as in kvpage/paged_attention.h.  head_dim must be
// one of 32, 64, 96, 128, 256; num_heads % kv_heads == 0; `warps` must be 1..8 (validated as the reference
// does; the B200 kernel chooses its own warp layout).  Returns cudaErrorInvalidValue for invalid
// arguments, otherwise the launch status.  Asynchronous on `stream`; no allocation: long contexts are split
// across CTAs (balanced schedule) with the partials in the library's fixed no-allocation scratch
// (kvp_paged_attention_noalloc), and calls on one device are ordered through an event so that calls on
// different streams never overlap on it.  Without a pool size the kernel cannot bounds-check table entries,
// exactly like the reference kernel.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

__attribute__((visibility("default"))) cudaError_t launch_paged_attention(const __half* q, const __half* k_cache, const __half* v_cache,
                                   const int* block_tables, const int* seq_lens, __half* out, int num_seqs,
                                   int num_heads, int kv_heads, int head_dim, int block_size, int max_blocks,
                                   int warps, cudaStream_t stream = 0);
