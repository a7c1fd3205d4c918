/*
 * kvp_b200.h -- C ABI of the B200 paged KV-cache data plane.
 *
 * Plain pointers and sizes only.  Device buffers are caller-owned and stay caller-owned; no entry point
 * allocates device memory.  Every function returns an int status (KVP_OK == 0) and never throws or aborts;
 * kvp_last_error() gives the message of the last failure on the calling thread.  Launch functions are
 * asynchronous on the given stream (a cudaStream_t passed as void*, NULL = legacy default stream) and do
 * not synchronize.  Problems that only device data can reveal (a block id outside the pool, a sequence
 * longer than its table row, a pipeline wait that gave up) cannot be returned synchronously: kernels OR a
 * KVP_STATUS_* bit into the optional caller-provided device word `status`.
 *
 * Cache layout, identical to the reference (include/kvpage/paged_attention.h:8-21 of
 * prathameshpranjale/paged-kv-cache-manager):
 *   q, out        [num_seqs][num_heads][head_dim]
 *   k/v pool      [num_blocks][block_size][kv_heads][head_dim]   (one pool per layer)
 *   block_tables  [num_seqs][max_blocks] int32; entries past a sequence are never read
 *   seq_lens      [num_seqs] int32 >= 1
 * Query head h uses kv head h / (num_heads / kv_heads).  Multi-layer calls address layer l's pool at
 * base + l * layer_stride elements (layer_stride 0 = num_blocks * block_size * kv_heads * head_dim, i.e.
 * a contiguous [layers][num_blocks][block_size][kv_heads][head_dim] array as in python/paged_model.py:25).
 */
#ifndef KVP_B200_H
#define KVP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KVP_API __attribute__((visibility("default")))
#else
#define KVP_API
#endif

/* ---- status codes returned by every entry point ---- */
#define KVP_OK 0
#define KVP_EINVAL 1   /* bad argument (the reference throws std::invalid_argument here) */
#define KVP_ECUDA 2    /* a CUDA runtime/driver call failed */
#define KVP_EBOUNDS 3  /* a host-visible id or size is outside its range */
#define KVP_ENOSPACE 4 /* caller-provided workspace or capacity too small */
#define KVP_ESTATE 5   /* host control-plane misuse (the reference throws std::logic_error here) */

/* ---- bits kernels OR into the optional device status word ---- */
#define KVP_STATUS_BAD_BLOCK 1 /* a table / slot / pair block id outside [0, num_blocks); access skipped */
#define KVP_STATUS_BAD_LEN 2   /* seq_len < 1 or ceil(seq_len / block_size) > max_blocks; sequence skipped */
#define KVP_STATUS_TIMEOUT 4   /* a pipeline wait gave up after ~1 s; the kernel returned early */

typedef enum kvp_dtype { KVP_DTYPE_F32 = 0, KVP_DTYPE_F16 = 1, KVP_DTYPE_BF16 = 2 } kvp_dtype;

/* Message of the last failure on this thread ("" if none). */
KVP_API const char* kvp_last_error(void);
/* Library version string. */
KVP_API const char* kvp_version(void);

/* ======================================================================== paged decode attention
 * Replaces the reference's GPU entry point launch_paged_attention (cuda/paged_attention.cuh:16-19) and is
 * the device form of paged_attention_cpu / reference_attention (include/kvpage/paged_attention.h:25-35,
 * src/paged_attention.cpp:25-114): one query token per sequence, softmax(q.K^T * scale) V over the
 * sequence's context, read in place through its block table.  fp32 accumulation; q and out fp32, fp16 or
 * bf16.  K/V fp16 or bf16 (16-byte aligned pools): the tensor-core kernel, with the split schedules below.
 * K/V fp32 (the reference's own float layout; 4-byte aligned pools): a CUDA-core kernel in fp32 arithmetic,
 * one CTA per (sequence, kv head), no workspace, no fused append, the tuning fields ignored.
 * Requirements: head_dim in {32, 64, 96, 128, 256}; num_heads % kv_heads == 0; num_heads / kv_heads <= 16
 * (<= 8 at head_dim 256); block_size >= 1. */
typedef struct kvp_attn_args {
    const void* q;
    int32_t q_dtype;
    const void* k_cache; /* this layer's pools */
    const void* v_cache;
    int32_t kv_dtype;
    int64_t num_blocks; /* blocks in each pool; bounds every table entry (0: unchecked) */
    const int32_t* block_tables;
    const int32_t* seq_lens;
    void* out;
    int32_t out_dtype;
    int32_t num_seqs, num_heads, kv_heads, head_dim, block_size, max_blocks;
    float scale;         /* <= 0: 1/sqrt(head_dim) */
    int32_t split_tiles; /* 16-token tiles per context split; 0: automatic; < 0: never split */
    int32_t kv_heads_per_cta; /* tuning, 0: automatic */
    int32_t stages;           /* tuning, 0: automatic */
    void* workspace;          /* split-K partials; kvp_attention_workspace_size() bytes, 256-B aligned */
    size_t workspace_bytes;
    int32_t* status; /* optional device word for KVP_STATUS_* bits */
    int32_t warps_per_kv_head; /* tuning, 0: automatic (consumer warps sharing one kv head's tiles) */
    int32_t flags;             /* KVP_ATTN_* bits */
    /* Fused append (both or neither; 16-byte aligned): [num_seqs][kv_heads][head_dim] in the pool dtype, the
     * K/V of each sequence's newest token -- position seq_lens[s] - 1, slot table[(len-1)/B]*B + (len-1)%B.
     * The kernel writes them into the pools (which must then be writable) before it attends over them, so a
     * decode step needs no separate kvp_append_scatter for this layer.  No other sequence of the call may
     * read those slots: true after KVManager::append_token (the written block is never shared), not for
     * several prompt positions of one request in one call. */
    const void* k_new;
    const void* v_new;
    /* tuning (balanced schedule), 0: automatic: a sequence's start cost, in 16-token tiles, charged to the CTA
     * that starts it when the step's tiles are divided between CTAs; < 0: none */
    int32_t seq_start_tiles;
    /* Inputs written by a copy on another stream (null: none; fp16/bf16 pools): the kernel reads q, k_new and
     * v_new only once this device word is non-zero -- the copy stream writes it after the data -- so the
     * launch needs no stream wait on that copy, which would keep it from starting during the previous kernel
     * (KVP_ATTN_EARLY_START / EARLY_LOAD).  The inputs are then the copy's, not the previous kernel's: with
     * KVP_ATTN_EARLY_LOAD the queries are loaded, and the first ring of tiles attended, before the kernel waits
     * for the previous one (every global write still waits for it).  With inputs_epoch (a device word, set before the launch) the
     * condition is instead (*inputs_ready - *inputs_epoch) >= 0 as a signed 32-bit difference, so a flag
     * that a copy sets to each step's epoch needs no reset between steps.  The wait is bounded
     * (KVP_STATUS_TIMEOUT).  Both 4-byte aligned. */
    const int32_t* inputs_ready;
    const int32_t* inputs_epoch;
} kvp_attn_args;

/* The caller guarantees the workspace's counter words are zero, so the call skips resetting them: true for
 * workspace memory that was zero-filled once and has since only been used by completed calls with the same
 * num_heads, kv_heads, head_dim and kv_heads_per_cta (each call leaves the counters zero; they sit at the
 * start of the workspace in a region whose size does not depend on num_seqs, so the batch size may change
 * from call to call).  Without it every balanced-schedule call first clears them on the stream. */
#define KVP_ATTN_WORKSPACE_CLEAN 1
/* Early start (programmatic dependent launch; balanced schedule only): the kernel may begin while the previous
 * kernel on the stream is still running.  Its prologue (tile prefix sums, barrier setup) reads seq_lens --
 * which that previous kernel therefore must not write -- and everything else waits for it to complete, so
 * back-to-back launches (one per layer) hide each other's start-up. */
#define KVP_ATTN_EARLY_START 2
/* Early load (implies early start): additionally the previous kernel on the stream writes neither block_tables
 * nor this call's K/V pools, so each CTA may load its first K/V tiles before waiting for it.  True between the
 * per-layer launches of a decode step (a layer's kernel writes only its own layer's pool). */
#define KVP_ATTN_EARLY_LOAD 4

/* Bytes of workspace kvp_paged_attention needs for these arguments (0 when no context is split).  With
 * split_tiles == 0 and a workspace the balanced persistent schedule is used: the step's tiles are divided
 * evenly between as many CTAs as fit on the GPU, and contexts split between CTAs are merged in the same
 * kernel. */
KVP_API size_t kvp_attention_workspace_size(const kvp_attn_args* a);
KVP_API int kvp_paged_attention(const kvp_attn_args* a, void* stream);

/* Host-buffer attention with the parameter list of the reference's CPU entry points, reference_attention and
 * paged_attention_cpu (include/kvpage/paged_attention.h:25-35 of the reference; their callers are
 * tests/test_attention.cpp and the Python binding python/kvpage_py.cpp:43-66).  Host pointers: fp32 q and out
 * [num_seqs][num_heads][head_dim]; fp32 k_cache / v_cache [num_blocks][block_size][kv_heads][head_dim], of which
 * the blocks up to the largest id the sequences' table entries use are read; int32 block_tables
 * [num_seqs][max_blocks] and seq_lens [num_seqs].  The reference's checks give KVP_EINVAL with its messages
 * (num_heads % kv_heads != 0; a seq_len < 1 or longer than max_blocks blocks; partitions < 1), a negative
 * block id KVP_EBOUNDS.  The computation runs on the current device -- the fp32 CUDA-core kernel, no CPU
 * path: the inputs are copied in, the outputs copied back, and the call returns once `out` is written
 * (synchronous, like the reference).  Unlike the device entry points it allocates the device buffers it
 * needs and frees them before returning.  `partitions` is the reference's parameter (checked >= 1); the
 * kernel's own split of the context does not depend on it. */
KVP_API int kvp_paged_attention_host(int32_t num_heads, int32_t kv_heads, int32_t head_dim, int32_t block_size,
                                     int32_t num_seqs, int32_t max_blocks, const float* q, const float* k_cache,
                                     const float* v_cache, const int32_t* block_tables, const int32_t* seq_lens,
                                     float* out, int32_t partitions);

/* Failure-detection test hook (no counterpart in the reference, whose nearest analogue is the simulator's
 * livelock guard, src/simulator.cpp:136).  Every pipeline wait of the attention kernel is bounded; no valid
 * input makes one run out, so this entry point exists to test that path without a GPU fault: it is
 * kvp_paged_attention with each wait limited to wait_limit_cycles clock cycles (1 .. 2e9; the normal entry
 * point uses 2e9, about a second) and, with stall_first_stage == 1, in every CTA of the grid's first row (kv-head
 * group 0 of the balanced schedule, split 0 of the fixed splits) pipeline stage 0 armed for 16 bytes of a copy
 * that is never issued -- a flag nothing sets -- and the tiles issued from stage 1 on.  Those CTAs' consumers,
 * which expect the first tile in stage 0, give up after the limit, their
 * producers stop issuing and wait (bounded) for the copies they did issue, the kernel ORs KVP_STATUS_TIMEOUT
 * into `status` and returns; no copy is left in flight and the context stays usable.
 * After KVP_STATUS_TIMEOUT from any entry point the outputs of the affected sequences are undefined and the
 * workspace's merge counters may be nonzero: the next call on that workspace must not pass
 * KVP_ATTN_WORKSPACE_CLEAN (without it the call clears them). */
KVP_API int kvp_attention_wait_test(const kvp_attn_args* a, void* stream, int64_t wait_limit_cycles,
                                    int32_t stall_first_stage);

/* The same attention for callers that cannot allocate device memory -- e.g. a serving engine whose memory
 * manager reserves nearly all HBM for the KV pool and gives libraries no allocation hook, or a plugin whose
 * enqueue callback must not allocate.  This entry point has no counterpart in the reference.  It ignores
 * a->workspace and keeps the split partials in a fixed KVP_NOALLOC_SCRATCH_BYTES device array built into the
 * library (held by every GPU that loads it, until exit); it calls no allocator.  The array's device address
 * is looked up on the first call made in each CUDA context (the first call on a device, and again after a
 * cudaDeviceReset gives the device a new context), so make that first call before any stream capture.
 * With split_tiles == 0 the balanced schedule is used while its partials fit -- they need
 * 8192 * (kv_heads / kv_heads_per_cta) * 4 B of counters plus (SMs * CTAs per SM + num_seqs) * num_heads *
 * (head_dim + 2) * 4 B, rounded up to 256 B each -- and beyond that the call switches to fixed splits of 16,
 * 32, 64, ... tiles until their partials fit (at the Llama-3-8B head shape, 32/8 heads of 128, from about
 * 1,900 sequences per call); an explicit split_tiles whose partials exceed the array returns KVP_ENOSPACE.  KVP_ATTN_WORKSPACE_CLEAN is ignored: every call clears the
 * merge counters it uses.  All calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller. */
#define KVP_NOALLOC_SCRATCH_BYTES (32u << 20)
KVP_API int kvp_paged_attention_noalloc(const kvp_attn_args* a, void* stream);

/* ======================================================================== KV-cache mutations
 * The device data plane of the reference's KVManager decisions (src/kv_manager.cpp:211-242), whose bytes
 * the reference moves only in Python (python/paged_model.py:54-55, 92-95, 113-117, 145-146). */

/* Append scatter: writes each sequence's new token K/V, for every layer, into its slot
 * (slot = block * block_size + offset, i.e. (table[pos / B], pos % B) for pos = tokens before the append;
 * a negative slot skips the sequence).  k_new / v_new: [num_layers][num_seqs][kv_heads][head_dim] in the
 * pool dtype.  Slots must be distinct. */
typedef struct kvp_append_args {
    const void* k_new;
    const void* v_new;
    void* k_cache;
    void* v_cache;
    int64_t layer_stride; /* elements between layer pools; 0: contiguous */
    const int32_t* slots; /* [num_seqs] device */
    int32_t kv_dtype, num_layers, num_seqs, kv_heads, head_dim, block_size;
    int64_t num_blocks;
    int32_t* status;
} kvp_append_args;
KVP_API int kvp_append_scatter(const kvp_append_args* a, void* stream);

/* Copy-on-write: for each (src, dst) pair copies the whole block, every layer, K and V
 * (python/paged_model.py:92-95).  pairs: device int32 [n_pairs][2].  All pairs of one call run
 * concurrently, so no dst may equal another pair's src or dst. */
typedef struct kvp_cow_args {
    void* k_cache;
    void* v_cache;
    int64_t layer_stride; /* elements; 0: contiguous */
    const int32_t* pairs;
    int32_t n_pairs, kv_dtype, num_layers, kv_heads, head_dim, block_size;
    int64_t num_blocks;
    int32_t* status;
} kvp_cow_args;
KVP_API int kvp_cow_copy(const kvp_cow_args* a, void* stream);

/* Migration between shards: for each (src, dst) pair copies the whole block, every layer, K and V, from one
 * shard's pools into another's -- on the same GPU, or from a peer GPU over NVLink with plain peer loads into
 * the destination GPU's own memory.  Launch on the destination pools' device (the current device); peer
 * access to the source device is enabled on first use (kvp_enable_peer_access).  pairs: device int32
 * [n_pairs][2] on the destination device; destinations distinct.  The host side of migrating a request is
 * the reference's swap semantics without the host round trip (src/simulator.cpp:117-133, 193, 231-241):
 * admit it on the destination KVManager (fresh ids, no sharing), pair the source table with the new table
 * entry by entry, copy, and free it on the source KVManager once the copy is ordered before any later
 * source-side write (an event the source stream waits for). */
typedef struct kvp_migrate_args {
    const void* src_k_cache;
    const void* src_v_cache;
    int64_t src_layer_stride; /* elements; 0: contiguous */
    int64_t src_num_blocks;
    void* dst_k_cache;
    void* dst_v_cache;
    int64_t dst_layer_stride;
    int64_t dst_num_blocks;
    const int32_t* pairs;
    int32_t n_pairs, kv_dtype, num_layers, kv_heads, head_dim, block_size;
    int32_t* status;
} kvp_migrate_args;
KVP_API int kvp_migrate_blocks(const kvp_migrate_args* a, void* stream);
/* Lets the current device read peer_device's memory (idempotent; KVP_EINVAL if the pair has no P2P path). */
KVP_API int kvp_enable_peer_access(int32_t peer_device);

/* Swap between the device pools and a pinned host pool.  A host slot holds one block of every layer:
 * [K: num_layers x block_bytes][V: num_layers x block_bytes], block_bytes = block_size*kv_heads*head_dim*elem.
 * blocks / host_slots are HOST arrays of length n; host_pool is pinned (cudaHostAlloc / registered) memory
 * of at least (max slot + 1) * 2 * num_layers * block_bytes bytes.  Asynchronous on `stream`; the caller
 * orders it against compute with events.  Swap-out copies data only: the caller then frees the request in
 * its KVManager.  Swap-in copies into the fresh ids that re-admission returned (src/simulator.cpp:193, 231-241). */
typedef struct kvp_swap_args {
    void* k_cache;
    void* v_cache;
    int64_t layer_stride; /* elements; 0: contiguous */
    int32_t kv_dtype, num_layers, kv_heads, head_dim, block_size;
    int64_t num_blocks;
    const int32_t* blocks;     /* host */
    const int64_t* host_slots; /* host */
    int32_t n;
    void* host_pool;
    int64_t host_pool_slots; /* slots the host pool holds; every host_slots[i] must be below it */
} kvp_swap_args;
KVP_API int kvp_swap_out(const kvp_swap_args* a, void* stream);
KVP_API int kvp_swap_in(const kvp_swap_args* a, void* stream);

/* ======================================================================== host control plane
 * C view of kvp::KVManager (include/kvpage/kv_manager.h; reference include/kvpage/kv_manager.h:26-77).
 * Bool results come back as 1/0; a thrown std::logic_error becomes -KVP_ESTATE and std::invalid_argument
 * -KVP_EINVAL (message in kvp_last_error()). */
typedef struct kvp_mgr kvp_mgr;
KVP_API kvp_mgr* kvp_mgr_create(int32_t num_blocks, int32_t block_size);
KVP_API void kvp_mgr_destroy(kvp_mgr* m);
KVP_API void kvp_mgr_set_check_each_op(kvp_mgr* m, int32_t on);
KVP_API int kvp_mgr_admit(kvp_mgr* m, int64_t r, int32_t prompt_tokens);
KVP_API int kvp_mgr_admit_with_prefix(kvp_mgr* m, int64_t r, int64_t parent, int32_t shared_tokens,
                                      int32_t prompt_tokens);
KVP_API int kvp_mgr_fork(kvp_mgr* m, int64_t r, int64_t parent);
KVP_API int kvp_mgr_append_token(kvp_mgr* m, int64_t r);
KVP_API int kvp_mgr_free(kvp_mgr* m, int64_t r);
KVP_API int kvp_mgr_contains(kvp_mgr* m, int64_t r);
KVP_API int kvp_mgr_num_tokens(kvp_mgr* m, int64_t r);
/* Copies up to cap block ids of r into out; returns the table length. */
KVP_API int kvp_mgr_table(kvp_mgr* m, int64_t r, int32_t* out, int32_t cap);
KVP_API int kvp_mgr_refcount(kvp_mgr* m, int32_t block);
KVP_API int kvp_mgr_free_blocks(kvp_mgr* m);
KVP_API int kvp_mgr_total_blocks(kvp_mgr* m);
KVP_API int kvp_mgr_available_blocks(kvp_mgr* m);
KVP_API int kvp_mgr_can_admit(kvp_mgr* m, int32_t prompt_tokens);
KVP_API int kvp_mgr_blocks_needed_to_admit(kvp_mgr* m, int64_t parent, int32_t shared_tokens, int32_t prompt_tokens);
/* out[10] = requests, used_tokens, allocated_blocks, allocated_slots, internal_waste, logical_blocks,
 * blocks_saved, cow_copies, cached_blocks, cache_evictions. */
KVP_API void kvp_mgr_stats(kvp_mgr* m, int64_t* out);
KVP_API void kvp_mgr_recompute_stats(kvp_mgr* m, int64_t* out);
/* Writes validate()'s message ("" when consistent) into buf; returns its length. */
KVP_API int kvp_mgr_validate(kvp_mgr* m, char* buf, int32_t cap);
KVP_API int kvp_mgr_cache_prefix(kvp_mgr* m, int32_t key, int64_t owner, int32_t tokens);
KVP_API int kvp_mgr_has_cached_prefix(kvp_mgr* m, int32_t key);
KVP_API int kvp_mgr_cached_prefix_tokens(kvp_mgr* m, int32_t key);
KVP_API int kvp_mgr_blocks_needed_to_admit_cached(kvp_mgr* m, int32_t key, int32_t shared_tokens, int32_t prompt_tokens);
KVP_API int kvp_mgr_admit_with_cached_prefix(kvp_mgr* m, int64_t r, int32_t key, int32_t shared_tokens,
                                             int32_t prompt_tokens);
KVP_API int kvp_mgr_evictable_blocks(kvp_mgr* m, int32_t key, int32_t shared_blocks);
KVP_API int kvp_mgr_shared_blocks_with_cached(kvp_mgr* m, int32_t key, int32_t shared_tokens, int32_t prompt_tokens);
KVP_API int kvp_mgr_clear_cache(kvp_mgr* m);

/* Batched append for a decode step: append_token for rids[0..n) in order, as the reference's Python
 * harness does per request (python/paged_model.py:105-118).  For each i, slots[i] receives the write slot
 * (block * block_size + offset) of the new token; when the append was a copy-on-write, the pair
 * (old block, new block) goes to cow_pairs[2k], cow_pairs[2k+1] (k counts copies; total in *n_cow;
 * cow_pairs needs room for 2n ints).  Returns the number of successful appends: n on success; on the first
 * append that found no block the batch stops there, that request's slot is -1 and later slots are -1. */
KVP_API int kvp_mgr_append_batch(kvp_mgr* m, const int64_t* rids, int32_t n, int32_t* slots, int32_t* cow_pairs,
                                 int32_t* n_cow);
/* Dense table rows for a batch: row i = table of rids[i], padded with `pad` up to max_blocks; lens[i] =
 * tokens.  Returns KVP_EBOUNDS if a table is longer than max_blocks. */
KVP_API int kvp_mgr_dense_tables(kvp_mgr* m, const int64_t* rids, int32_t n, int32_t max_blocks, int32_t pad,
                                 int32_t* tables, int32_t* lens);

/* ======================================================================== decode-step runtime
 * One call per decode step for one GPU shard: the device form of the reference harness's decode_batch
 * (python/paged_model.py:105-154).  For the given requests, in order: KVManager::append_token (through the
 * caller's kvp_mgr), the copy-on-write copies those appends decided, then per layer one paged-attention
 * launch that writes the layer's new K/V into the appended slot (fused append) and attends over the updated
 * cache.  The host-buffer form copies each layer's inputs in and its output out on its own streams, so that
 * transfers overlap the attention of other layers, and returns once the outputs are in host memory (pinned
 * host buffers make the copies asynchronous).  With `graph` set, the per-layer launches of a step are
 * captured once into a CUDA graph and replayed while the batch size and buffers stay the same (a step whose
 * key repeats the previous step's is captured; a stream the caller is capturing is never captured into).
 * Device memory: the caller passes the pools and one workspace of kvp_decoder_workspace_size() bytes; the
 * decoder allocates no device memory (it allocates pinned host staging for tables and slots). */
typedef struct kvp_decoder_config {
    int32_t num_layers, num_heads, kv_heads, head_dim, block_size;
    int32_t kv_dtype, q_dtype, out_dtype;
    int64_t num_blocks;          /* blocks in each layer's pool */
    int64_t layer_stride;        /* elements between layer pools; 0: contiguous [L][num_blocks][B][kvh][D] */
    int32_t max_seqs;            /* most requests in one step */
    int32_t max_blocks_per_seq;  /* table row length */
    int32_t split_tiles;         /* 0: automatic from the step's context lengths; < 0: never split */
    void* k_cache;
    void* v_cache;
    void* workspace; /* device, 256-byte aligned */
    size_t workspace_bytes;
    int32_t graph;   /* 1: replay each step's per-layer launches as a CUDA graph (see above); 0: plain launches */
} kvp_decoder_config;
typedef struct kvp_decoder kvp_decoder;
KVP_API size_t kvp_decoder_workspace_size(const kvp_decoder_config* c);
KVP_API kvp_decoder* kvp_decoder_create(const kvp_decoder_config* c, kvp_mgr* mgr);
KVP_API void kvp_decoder_destroy(kvp_decoder* d);
/* q / out: [num_layers][n][num_heads][head_dim]; k_new / v_new: [num_layers][n][kv_heads][head_dim] (pool
 * dtype).  Host pointers.  Returns KVP_OK, or KVP_ENOSPACE when an append found no free block (the KVManager
 * state then reflects the appends that succeeded; nothing was launched). */
KVP_API int kvp_decoder_step(kvp_decoder* d, const int64_t* rids, int32_t n, const void* q, const void* k_new,
                             const void* v_new, void* out);
/* Same with device pointers (k_new / v_new 16-byte aligned), asynchronous on `stream` (only the host
 * bookkeeping and the small table upload are done before returning). */
KVP_API int kvp_decoder_step_device(kvp_decoder* d, const int64_t* rids, int32_t n, const void* q,
                                    const void* k_new, const void* v_new, void* out, void* stream);
/* Pipelined steps.  kvp_decoder_submit() is kvp_decoder_step() without the wait: it issues the step's copies
 * and launches and returns; kvp_decoder_wait() returns once the submitted step's outputs are in host memory
 * (a submit, step or step_device call waits for a submitted step first).  kvp_decoder_plan() does the NEXT
 * step's bookkeeping now -- its KVManager appends (the manager reflects them at once), copy-on-write pairs and
 * staged tables, in the staging buffer the submitted step does not use -- so that it overlaps the submitted
 * step on the device.  The next submit / step / step_device must then be for the same requests in the same
 * order (else KVP_EINVAL, and the planned appends stay in the manager); if the caller changed any table
 * between the plan and that call, the planned tables are re-read from the manager.  A second plan before that
 * call is KVP_ESTATE.  A serving loop: plan(batch); per step: submit(batch) -> plan(next batch) -> wait(). */
KVP_API int kvp_decoder_submit(kvp_decoder* d, const int64_t* rids, int32_t n, const void* q, const void* k_new,
                               const void* v_new, void* out);
/* Pinned host input buffers owned by the decoder, for callers that produce each step's inputs in place: for a
 * step of n requests, layer l's queries are at q + l * layer_stride bytes, its new K at k_new + l * layer_stride
 * and its new V at v_new + l * layer_stride (each [n][heads][head_dim] in the config's dtypes), so a layer's
 * three inputs are adjacent and a run of layers goes up in one copy instead of three.  A step given exactly
 * these pointers (same n) uses that layout; pointers into the buffer from another n are KVP_EINVAL (nothing is
 * done).  The buffer is shared by all n and lives as long as the decoder. */
KVP_API int kvp_decoder_host_inputs(kvp_decoder* d, int32_t n, void** q, void** k_new, void** v_new,
                                    size_t* layer_stride);
KVP_API int kvp_decoder_plan(kvp_decoder* d, const int64_t* rids, int32_t n);
KVP_API int kvp_decoder_wait(kvp_decoder* d);
/* OR of the KVP_STATUS_* bits the decoder's kernels reported so far (synchronises the decoder's streams). */
KVP_API int kvp_decoder_status(kvp_decoder* d);

#ifdef __cplusplus
}
#endif
#endif /* KVP_B200_H */
