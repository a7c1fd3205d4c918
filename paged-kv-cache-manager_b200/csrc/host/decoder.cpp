// Decode-step runtime: one call per step for one GPU shard (the device form of the reference harness's
// decode_batch, python/paged_model.py:105-154).
//
// Per step: host bookkeeping (KVManager::append_token per request -> copy-on-write pairs,
// dense table rows, lengths), one upload of that metadata, then on the compute stream: copy-on-write copies
// and one paged-attention launch per layer that first writes the layer's new K/V into the appended slot
// (fused append) and then attends over the context including it.  With host buffers, a copy-in
// stream feeds the new K/V and each layer's queries and a copy-out stream drains each layer's output as soon as
// its attention finishes, so transfers overlap the attention of other layers.  Once a step's key (batch size
// and buffers) repeats, that whole body -- copies and launches on the three streams -- is replayed from one
// CUDA graph, so a step costs the host a handful of runtime calls.  A step can be submitted without waiting for
// it (kvp_decoder_submit / kvp_decoder_wait) and the next step's bookkeeping planned while it runs
// (kvp_decoder_plan, into the second of two pinned staging buffers).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <stdexcept>
#include <unordered_set>
#include <vector>

#include "kvp_b200.h"
#include "kvp_internal.h"

namespace {

constexpr int kMaxSplitsCap = 64;  // most fixed splits per sequence the decoder reserves workspace for

size_t align256(size_t x) { return (x + 255) / 256 * 256; }
int elem(int dt) { return dt == KVP_DTYPE_F32 ? 4 : 2; }

struct Layout {
    size_t meta = 0;        // [tables max_seqs*max_blocks][lens][pairs 2*max_seqs] int32
    size_t flags = 0;       // int32 per layer: input-ready flags (one per copy-in group), 1 while the group is up
    size_t status = 0;      // int32
    size_t attn = 0;        // split partials
    size_t q = 0, k = 0, v = 0, out = 0;  // host-path staging
    size_t total = 0;
    size_t attn_bytes = 0;
};

Layout layout_of(const kvp_decoder_config& c) {
    Layout L;
    const size_t ns = static_cast<size_t>(c.max_seqs);
    size_t o = 0;
    L.meta = o;
    o = align256(o + sizeof(int32_t) * (ns * static_cast<size_t>(c.max_blocks_per_seq) + 3 * ns));
    L.flags = o;
    o = align256(o + sizeof(int32_t) * static_cast<size_t>(c.num_layers));
    L.status = o;
    o = align256(o + sizeof(int32_t));
    L.attn = o;
    if (c.split_tiles >= 0) {
        // The attention workspace of the largest step: the balanced (stream-K) schedule for split_tiles 0,
        // otherwise the fixed splits.
        kvp_attn_args a{};
        a.q_dtype = c.q_dtype;
        a.kv_dtype = c.kv_dtype;
        a.out_dtype = c.out_dtype;
        a.num_blocks = c.num_blocks;
        a.num_seqs = c.max_seqs;
        a.num_heads = c.num_heads;
        a.kv_heads = c.kv_heads;
        a.head_dim = c.head_dim;
        a.block_size = c.block_size;
        a.max_blocks = c.max_blocks_per_seq;
        a.split_tiles = c.split_tiles;
        L.attn_bytes = kvp_attention_workspace_size(&a);
    }
    o = align256(o + L.attn_bytes);
    const size_t per_q = ns * c.num_heads * c.head_dim, per_kv = ns * c.kv_heads * c.head_dim;
    L.q = o;
    o = align256(o + static_cast<size_t>(c.num_layers) * per_q * elem(c.q_dtype));
    L.k = o;
    o = align256(o + static_cast<size_t>(c.num_layers) * per_kv * elem(c.kv_dtype));
    L.v = o;
    o = align256(o + static_cast<size_t>(c.num_layers) * per_kv * elem(c.kv_dtype));
    L.out = o;
    o = align256(o + static_cast<size_t>(c.num_layers) * per_q * elem(c.out_dtype));
    L.total = o;
    return L;
}

int check_config(const kvp_decoder_config* c) {
    using kvpi::fail;
    if (!c) return fail(KVP_EINVAL, "null config");
    if (c->num_layers < 1 || c->num_heads < 1 || c->kv_heads < 1 || c->head_dim < 1 || c->block_size < 1 ||
        c->max_seqs < 1 || c->max_blocks_per_seq < 1 || c->num_blocks < 1)
        return fail(KVP_EINVAL, "bad decoder shape");
    if (!(c->kv_dtype == KVP_DTYPE_F16 || c->kv_dtype == KVP_DTYPE_BF16) || !kvpi::valid_dtype(c->q_dtype) ||
        !kvpi::valid_dtype(c->out_dtype))
        return fail(KVP_EINVAL, "bad decoder dtype");
    return KVP_OK;
}

}  // namespace

// What a captured step depends on besides the device-resident metadata: the batch size (it fixes the
// metadata layout and the kernels' parameters) and the per-layer buffers (device or host).
struct GraphKey {
    int n = -1;
    const void *q = nullptr, *k = nullptr, *v = nullptr, *out = nullptr;
    bool operator==(const GraphKey& o) const { return n == o.n && q == o.q && k == o.k && v == o.v && out == o.out; }
};

// One of the two pinned staging buffers of step metadata (same layout as the device meta region), and what its
// table rows hold: row i is request rids[i]'s table with sizes[i] entries, as of the manager's table_changes()
// count `changes`, when the decoder's own appends had reached `ours` (valid: a step's bookkeeping completed
// since the rows were last fully written).
struct Staging {
    int32_t* h = nullptr;  // pinned: tables, lengths, pairs
    cudaEvent_t ev = nullptr;  // after the latest upload from `h` (it is writable again)
    std::vector<int32_t> pairs;  // the copy-on-write pairs of the step staged here (src, dst, ...)
    bool valid = false;
    uint64_t changes = 0, ours = 0;
    std::vector<int64_t> rids;
    std::vector<int32_t> sizes;
};

struct kvp_decoder {
    kvp_decoder_config cfg{};
    kvp_mgr* mgr = nullptr;
    Layout lay;
    char* ws = nullptr;
    // Double-buffered staging: a step's bookkeeping (or the next step's, planned while this one runs) writes
    // one buffer while the other may still be read by an upload in flight.
    Staging stg[2];
    int next = 0;                // the buffer the next step's bookkeeping writes
    uint64_t our_appends = 0;    // appends this decoder made through the manager
    // A planned step (kvp_decoder_plan): its bookkeeping is done and staged in stg[plan_buf].
    bool planned = false;
    int plan_buf = 0;
    uint64_t plan_changes = 0;
    bool submitted = false;      // a host-buffer step was submitted and not yet waited for
    // Input-ready flags are set by a stream memory operation (cuStreamWriteValue32: no copy-engine work) where the
    // driver offers it inside graphs, else by a 4-byte copy from the pinned word h_one.
    using WriteValueFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
    WriteValueFn write_value = nullptr;
    int32_t* h_one = nullptr;
    char* h_in = nullptr;  // pinned packed input buffer (kvp_decoder_host_inputs), allocated on first use
    size_t h_in_bytes = 0;
    size_t meta_bytes = 0;
    int64_t layer_stride = 0;   // elements
    cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join_in = nullptr, ev_join_out = nullptr;
    std::vector<cudaEvent_t> ev_att;
    int device = 0;
    GraphKey last_key, exec_key;  // the previous step's key; the key the instantiated graph was captured for
    cudaGraphExec_t exec = nullptr;
    GraphKey last_full, full_key;  // the same for the whole host-buffer step (copies included)
    cudaGraphExec_t exec_full = nullptr;
    bool graph_off = false;       // set when a capture failed: plain launches from then on

    ~kvp_decoder() {
        if (exec) cudaGraphExecDestroy(exec);
        if (exec_full) cudaGraphExecDestroy(exec_full);
        if (h_one) cudaFreeHost(h_one);
        if (h_in) cudaFreeHost(h_in);
        for (Staging& b : stg) {
            if (b.h) cudaFreeHost(b.h);
            if (b.ev) cudaEventDestroy(b.ev);
        }
        for (auto e : ev_att) cudaEventDestroy(e);
        for (auto e : {ev_fork, ev_join_in, ev_join_out})
            if (e) cudaEventDestroy(e);
        for (auto s : {s_in, s_comp, s_out})
            if (s) cudaStreamDestroy(s);
    }

    int32_t* d_meta() const { return reinterpret_cast<int32_t*>(ws + lay.meta); }
    int32_t* d_flags() const { return reinterpret_cast<int32_t*>(ws + lay.flags); }
    int32_t* d_status() const { return reinterpret_cast<int32_t*>(ws + lay.status); }
};

namespace {

// Host bookkeeping of a step into staging buffer `buf`: appends, copy-on-write pairs, table rows and lengths
// (the fused append derives each written slot from the table row and the length).  When the buffer last
// staged the same batch, in the same order, and every table change since then was one of this decoder's own
// appends (the manager's change count against the decoder's append count), a row can only have changed from
// its last staged entry on -- appends add entries and copy-on-write replaces the last one -- so only those
// entries are written (a full row rewrite cost about 40 us per step for 256 requests of 1,100 tokens, 190 us
// at 4,400).  Returns KVP_OK or KVP_ENOSPACE (an append found no block).
int host_step(kvp_decoder* d, const int64_t* rids, int n, int buf) {
    kvp::KVManager& m = d->mgr->m;
    const kvp_decoder_config& c = d->cfg;
    const int B = c.block_size, MB = c.max_blocks_per_seq;
    Staging& st = d->stg[buf];
    int32_t* tables = st.h;
    int32_t* lens = tables + static_cast<size_t>(n) * MB;
    const bool incremental = st.valid && m.table_changes() - st.changes == d->our_appends - st.ours &&
                             st.rids.size() == static_cast<size_t>(n) &&
                             std::memcmp(st.rids.data(), rids, sizeof(int64_t) * static_cast<size_t>(n)) == 0;
    st.valid = false;  // until this step's bookkeeping completes
    st.pairs.clear();
    st.sizes.resize(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
        const kvp::BlockTable& t = m.table(rids[i]);
        const int pos = t.tokens;
        const kvp::BlockId old_last = t.blocks.empty() ? kvp::kNoBlock : t.blocks.back();
        if (!m.append_token(rids[i])) return kvpi::fail(KVP_ENOSPACE, "no free block for request " + std::to_string(rids[i]));
        ++d->our_appends;
        if (pos % B != 0 && t.blocks.back() != old_last) {
            st.pairs.push_back(old_last);
            st.pairs.push_back(t.blocks.back());
        }
        const int size = static_cast<int>(t.blocks.size());
        if (size > MB)
            return kvpi::fail(KVP_EBOUNDS, "request " + std::to_string(rids[i]) + " outgrew max_blocks_per_seq");
        lens[i] = t.tokens;
        int32_t* row = tables + static_cast<size_t>(i) * MB;
        const int from = incremental ? std::max(0, std::min(st.sizes[static_cast<size_t>(i)], size) - 1) : 0;
        std::memcpy(row + from, t.blocks.data() + from, sizeof(int32_t) * static_cast<size_t>(size - from));
        st.sizes[static_cast<size_t>(i)] = size;
    }
    std::memcpy(lens + n, st.pairs.data(), sizeof(int32_t) * st.pairs.size());
    st.rids.assign(rids, rids + n);
    st.changes = m.table_changes();
    st.ours = d->our_appends;
    st.valid = true;
    return KVP_OK;
}

// Rewrites the rows and lengths of staging buffer `buf` from the manager (no appends): a planned step whose
// tables the caller changed between the plan and the submit.  Its copy-on-write pairs stay as planned.
int restage(kvp_decoder* d, const int64_t* rids, int n, int buf) {
    kvp::KVManager& m = d->mgr->m;
    const int MB = d->cfg.max_blocks_per_seq;
    Staging& st = d->stg[buf];
    int32_t* lens = st.h + static_cast<size_t>(n) * MB;
    st.valid = false;
    for (int i = 0; i < n; ++i) {
        const kvp::BlockTable& t = m.table(rids[i]);
        const int size = static_cast<int>(t.blocks.size());
        if (size > MB)
            return kvpi::fail(KVP_EBOUNDS, "request " + std::to_string(rids[i]) + " outgrew max_blocks_per_seq");
        std::memcpy(st.h + static_cast<size_t>(i) * MB, t.blocks.data(), sizeof(int32_t) * static_cast<size_t>(size));
        st.sizes[static_cast<size_t>(i)] = size;
        lens[i] = t.tokens;
    }
    st.changes = m.table_changes();
    st.ours = d->our_appends;
    st.valid = true;
    return KVP_OK;
}


// Copy-on-write launches in order-preserving chunks: a pair whose destination is the source of an earlier
// pair of the chunk starts a new chunk, so every block is read before it is overwritten.
int launch_cow(kvp_decoder* d, const int32_t* d_pairs, cudaStream_t s, int buf) {
    const kvp_decoder_config& c = d->cfg;
    const std::vector<int32_t>& pairs = d->stg[buf].pairs;
    const int npairs = static_cast<int>(pairs.size() / 2);
    int start = 0;
    std::unordered_set<int32_t> srcs;
    auto flush = [&](int end) {
        if (end <= start) return KVP_OK;
        kvp_cow_args a{};
        a.k_cache = c.k_cache;
        a.v_cache = c.v_cache;
        a.layer_stride = d->layer_stride;
        a.pairs = d_pairs + 2 * start;
        a.n_pairs = end - start;
        a.kv_dtype = c.kv_dtype;
        a.num_layers = c.num_layers;
        a.kv_heads = c.kv_heads;
        a.head_dim = c.head_dim;
        a.block_size = c.block_size;
        a.num_blocks = c.num_blocks;
        a.status = d->d_status();
        return kvp_cow_copy(&a, s);
    };
    for (int k = 0; k < npairs; ++k) {
        if (srcs.count(pairs[2 * k + 1])) {
            int rc = flush(k);
            if (rc != KVP_OK) return rc;
            start = k;
            srcs.clear();
        }
        srcs.insert(pairs[2 * k]);
    }
    return flush(npairs);
}

// Where a step's inputs are: layer l's queries at q + l * q_stride bytes, its new K at k + l * kv_stride and its
// new V at v + l * kv_stride.  Separate arrays [L][n][...]: each stride is one layer of that array.  Packed (the
// decoder's own pinned input buffer and its device mirror): a layer's queries, new K and new V are adjacent and
// both strides are their sum, so a run of layers is one contiguous range -- one copy.
struct Inputs {
    const char *q = nullptr, *k = nullptr, *v = nullptr;
    size_t q_stride = 0, kv_stride = 0;
    bool packed = false;
};

size_t q_layer_bytes(const kvp_decoder_config& c, int n) {
    return static_cast<size_t>(n) * c.num_heads * c.head_dim * elem(c.q_dtype);
}
size_t kv_layer_bytes(const kvp_decoder_config& c, int n) {
    return static_cast<size_t>(n) * c.kv_heads * c.head_dim * elem(c.kv_dtype);
}

Inputs separate_inputs(const kvp_decoder_config& c, int n, const void* q, const void* k, const void* v) {
    Inputs in;
    in.q = static_cast<const char*>(q);
    in.k = static_cast<const char*>(k);
    in.v = static_cast<const char*>(v);
    in.q_stride = q_layer_bytes(c, n);
    in.kv_stride = kv_layer_bytes(c, n);
    return in;
}

Inputs packed_inputs(const kvp_decoder_config& c, int n, const void* base) {
    Inputs in;
    in.q = static_cast<const char*>(base);
    in.k = in.q + q_layer_bytes(c, n);
    in.v = in.k + kv_layer_bytes(c, n);
    in.q_stride = in.kv_stride = q_layer_bytes(c, n) + 2 * kv_layer_bytes(c, n);
    in.packed = true;
    return in;
}

// Layer l's attention launch (fused append of its new token) on stream s, its inputs as `in` places them (device
// memory) and its output at out + l * one layer's output; `ready`: the input-ready flag of the layer's copy-in
// group (null: its inputs are in place before the launch).
int launch_layer(kvp_decoder* d, int n, int l, const Inputs& in, void* out, cudaStream_t s,
                 const int32_t* ready = nullptr) {
    const kvp_decoder_config& c = d->cfg;
    const int32_t* meta = d->d_meta();
    const size_t L = static_cast<size_t>(l);
    const size_t kv_layer_bytes = static_cast<size_t>(d->layer_stride) * 2;
    const size_t q_layer = static_cast<size_t>(n) * c.num_heads * c.head_dim;
    kvp_attn_args a{};
    a.q = in.q + in.q_stride * L;
    a.q_dtype = c.q_dtype;
    a.k_cache = static_cast<const char*>(c.k_cache) + kv_layer_bytes * L;
    a.v_cache = static_cast<const char*>(c.v_cache) + kv_layer_bytes * L;
    a.kv_dtype = c.kv_dtype;
    a.num_blocks = c.num_blocks;
    a.block_tables = meta;                                              // [n][max_blocks_per_seq]
    a.seq_lens = meta + static_cast<size_t>(n) * c.max_blocks_per_seq;  // [n]
    a.out = static_cast<char*>(out) + q_layer * elem(c.out_dtype) * L;
    a.out_dtype = c.out_dtype;
    a.num_seqs = n;
    a.num_heads = c.num_heads;
    a.kv_heads = c.kv_heads;
    a.head_dim = c.head_dim;
    a.block_size = c.block_size;
    a.max_blocks = c.max_blocks_per_seq;
    a.split_tiles = c.split_tiles;  // 0: balanced schedule over the step's real context lengths
    a.workspace = d->lay.attn_bytes ? d->ws + d->lay.attn : nullptr;
    a.workspace_bytes = d->lay.attn_bytes;
    a.status = d->d_status();
    // lengths and tables are uploaded before the step's first launch and no kernel writes them: each layer's
    // launch may start during the previous one, and from the second layer on (the previous kernel then writes
    // only its own layer's pool) also load K/V before it ends
    a.flags = KVP_ATTN_WORKSPACE_CLEAN | (l > 0 ? KVP_ATTN_EARLY_LOAD : KVP_ATTN_EARLY_START);
    a.k_new = in.k + in.kv_stride * L;  // fused append of this layer's new token
    a.v_new = in.v + in.kv_stride * L;
    a.inputs_ready = ready;
    return kvp_paged_attention(&a, s);
}

// Every layer's launch, in order on stream s (device buffers).
int enqueue_layers(kvp_decoder* d, int n, const void* q, const void* knew, const void* vnew, void* out,
                   cudaStream_t s) {
    const Inputs in = separate_inputs(d->cfg, n, q, knew, vnew);
    for (int l = 0; l < d->cfg.num_layers; ++l) {
        const int rc = launch_layer(d, n, l, in, out, s);
        if (rc != KVP_OK) return rc;
    }
    return KVP_OK;
}

// Layers per output copy: enough consecutive layers that each copy moves at least ~512 KB (small copies pay a
// fixed cost each on the copy engines); the last layer is copied on its own (nothing overlaps that copy).
int layers_per_copy(const kvp_decoder_config& c, int n) {
    const size_t q_layer = static_cast<size_t>(n) * c.num_heads * c.head_dim * elem(c.q_dtype);
    const size_t want = size_t(512) << 10;
    return static_cast<int>(std::min<size_t>(static_cast<size_t>(c.num_layers), std::max<size_t>(1, (want + q_layer - 1) / q_layer)));
}

// Sets an input-ready flag to 1 on stream s once the work before it in s is done.
cudaError_t set_flag(kvp_decoder* d, int32_t* flag, cudaStream_t s) {
    if (d->write_value)
        return d->write_value(s, reinterpret_cast<CUdeviceptr>(flag), 1u, 0u) == CUDA_SUCCESS ? cudaSuccess
                                                                                              : cudaErrorUnknown;
    return cudaMemcpyAsync(flag, d->h_one, sizeof(int32_t), cudaMemcpyHostToDevice, s);
}

// The device copy of a step's host inputs: the workspace's input region, laid out as the host inputs are.
Inputs device_inputs(kvp_decoder* d, int n, const Inputs& host) {
    char* base = d->ws + d->lay.q;  // the q, k and v regions follow one another: room for either layout
    return host.packed ? packed_inputs(d->cfg, n, base)
                       : separate_inputs(d->cfg, n, base, d->ws + d->lay.k, d->ws + d->lay.v);
}

// The step's host inputs as the caller passed them: the decoder's own packed buffer (kvp_decoder_host_inputs) or
// separate arrays.
Inputs host_inputs_of(kvp_decoder* d, int n, const void* q, const void* k, const void* v) {
    if (d->h_in && q == d->h_in) {
        const Inputs p = packed_inputs(d->cfg, n, d->h_in);
        if (k == p.k && v == p.v) return p;
    }
    return separate_inputs(d->cfg, n, q, k, v);
}

// Layers [l0, l0 + G) of the step's inputs up on stream s: one copy when packed, else one per array.
cudaError_t copy_layers(const Inputs& dev, const Inputs& host, int l0, int G, cudaStream_t s) {
    const size_t L0 = static_cast<size_t>(l0), n = static_cast<size_t>(G);
    const auto up = [&](const char* dst, const char* src, size_t stride) {
        return cudaMemcpyAsync(const_cast<char*>(dst) + stride * L0, src + stride * L0, stride * n,
                               cudaMemcpyHostToDevice, s);
    };
    if (host.packed) return up(dev.q, host.q, host.q_stride);
    cudaError_t e = up(dev.q, host.q, host.q_stride);
    if (e == cudaSuccess) e = up(dev.k, host.k, host.kv_stride);
    if (e == cudaSuccess) e = up(dev.v, host.v, host.kv_stride);
    return e;
}

// Layer 0's inputs, copied up on the copy-in stream before the step's bookkeeping (they do not depend on it), so
// the copy overlaps the host work, then layer 0's input-ready flag.
int copy_first_layer(kvp_decoder* d, int n, const Inputs& host) {
    cudaError_t e = copy_layers(device_inputs(d, n, host), host, 0, 1, d->s_in);
    if (e == cudaSuccess) e = set_flag(d, d->d_flags(), d->s_in);
    return kvpi::cuda_status(e, "decoder first-layer copy");
}

// The host-buffer step's device work after the metadata upload and the copy-on-write copies, forked from and
// joined back into the compute stream.  Layer 0's inputs are already on their way (copy_first_layer); the rest
// go up on the copy-in stream in groups of 2, 4, ... layers, which land while earlier layers compute with few
// copies (per-layer copies of a few hundred KB each fell behind the attention at the TinyLlama shape: 1.49 ms
// per step against 1.34 ms with doubling groups on B200).  After each group the copy-in stream copies the
// group's input-ready flag to 1, and the group's layers wait for it inside the kernel (kvp_attn_args.inputs_ready)
// rather than on the stream: a stream wait on another stream's copy ends the early start of the launch after it,
// which cost 13-27 us per group on B200 (Qwen2.5-0.5B / TinyLlama shapes).  The flags are set by stream memory
// operations where the driver allows them in graphs: a copy engine spends ~7 us on even a 4-byte copy (B200),
// time the step's input copies wait for.  Once the last layer is done, the copy-in stream clears the flags for
// the next step.  Outputs go back on the copy-out stream in groups of layers_per_copy() layers once their last
// launch is done.  The same calls are captured into one graph when a step's key repeats.
int enqueue_host_body(kvp_decoder* d, int n, const Inputs& host, char* hout) {
    const kvp_decoder_config& c = d->cfg;
    const size_t o_layer = static_cast<size_t>(n) * c.num_heads * c.head_dim * elem(c.out_dtype);
    const Inputs dev = device_inputs(d, n, host);
    char* dout = d->ws + d->lay.out;
    const int L = c.num_layers;
    const int per = layers_per_copy(c, n);
    cudaError_t e = cudaEventRecord(d->ev_fork, d->s_comp);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->s_in, d->ev_fork, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->s_out, d->ev_fork, 0);
    // copy-in groups [in0, in0 + g) with g = 1, 2, 4, ..., group gi's flag in word gi (fewer groups than layers);
    // the first (layer 0) was issued before the bookkeeping and has been waited for
    size_t gi = 1;
    for (int in0 = 1, g = 2; e == cudaSuccess && in0 < L; in0 += g, g *= 2, ++gi) {
        e = copy_layers(dev, host, in0, std::min(g, L - in0), d->s_in);
        if (e == cudaSuccess) e = set_flag(d, d->d_flags() + gi, d->s_in);
    }
    gi = 0;
    size_t oi = 0;
    for (int l = 0, next_in = 0, g = 1, out0 = 0; e == cudaSuccess && l < L; ++l) {
        if (l == next_in) {  // the first layer of the next copy-in group
            ++gi;
            next_in += g;
            g *= 2;
        }
        const int rc = launch_layer(d, n, l, dev, dout, d->s_comp, d->d_flags() + (gi - 1));
        if (rc != KVP_OK) return rc;
        // An output group is complete -- the last layer always gets its own, since nothing overlaps its copy.
        if (l + 1 - out0 == per || l + 1 == L || l + 2 == L) {
            const size_t L0 = static_cast<size_t>(out0), G = static_cast<size_t>(l + 1 - out0);
            e = cudaEventRecord(d->ev_att[oi], d->s_comp);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(d->s_out, d->ev_att[oi], 0);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(hout + o_layer * L0, dout + o_layer * L0, o_layer * G, cudaMemcpyDeviceToHost,
                                    d->s_out);
            ++oi;
            out0 = l + 1;
        }
    }
    // every layer is done with the flags: clear them for the next step (beside the last output copy)
    if (e == cudaSuccess && oi > 0) e = cudaStreamWaitEvent(d->s_in, d->ev_att[oi - 1], 0);
    if (e == cudaSuccess) e = cudaMemsetAsync(d->d_flags(), 0, sizeof(int32_t) * gi, d->s_in);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev_join_in, d->s_in);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev_join_out, d->s_out);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->s_comp, d->ev_join_in, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->s_comp, d->ev_join_out, 0);
    return kvpi::cuda_status(e, "decoder step copies");
}

// Ends a capture on s and instantiates its graph into *out (replacing any previous one).  Returns false, with
// the error state cleared, if the capture or the instantiation failed.
bool finish_capture(cudaStream_t s, int rc, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    cudaGraphExec_t ex = nullptr;
    const bool ok = rc == KVP_OK && e == cudaSuccess && g && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess;
    if (g) cudaGraphDestroy(g);
    if (!ok) {
        if (ex) cudaGraphExecDestroy(ex);
        cudaGetLastError();
        kvpi::clear_error();
        return false;
    }
    if (*out) cudaGraphExecDestroy(*out);
    *out = ex;
    return true;
}

// Captures the per-layer launches (device buffers) into a graph and instantiates it.  Returns false if
// anything failed; the caller then launches them directly.
bool capture_layers(kvp_decoder* d, const GraphKey& key, cudaStream_t s) {
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const int rc = enqueue_layers(d, key.n, key.q, key.k, key.v, const_cast<void*>(key.out), s);
    if (!finish_capture(s, rc, &d->exec)) return false;
    d->exec_key = key;
    return true;
}

// The same for the whole host-buffer step body (copies included), captured from the compute stream.
bool capture_host_body(kvp_decoder* d, const GraphKey& key) {
    if (cudaStreamBeginCapture(d->s_comp, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const int rc = enqueue_host_body(d, key.n, host_inputs_of(d, key.n, key.q, key.k, key.v),
                                     static_cast<char*>(const_cast<void*>(key.out)));
    if (!finish_capture(d->s_comp, rc, &d->exec_full)) return false;
    d->full_key = key;
    return true;
}

// Device-buffer step after the metadata upload: copy-on-write copies, then the layer launches (replayed from
// a graph once the key repeats, unless the caller is capturing the stream itself).
int enqueue_device(kvp_decoder* d, int n, const void* q, const void* knew, const void* vnew, void* out,
                   cudaStream_t s_comp, int buf) {
    const kvp_decoder_config& c = d->cfg;
    const int32_t* d_pairs = d->d_meta() + static_cast<size_t>(n) * c.max_blocks_per_seq + n;
    int rc = launch_cow(d, d_pairs, s_comp, buf);
    if (rc != KVP_OK) return rc;
    if (c.graph && !d->graph_off) {
        GraphKey key;
        key.n = n;
        key.q = q;
        key.k = knew;
        key.v = vnew;
        key.out = out;
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        // The legacy default stream cannot be captured; a stream the caller is capturing records our launches.
        const bool capturable = s_comp != nullptr && cudaStreamIsCapturing(s_comp, &cs) == cudaSuccess &&
                                cs == cudaStreamCaptureStatusNone;
        if (capturable) {
            const bool repeat = key == d->last_key;
            d->last_key = key;
            if (!(d->exec && d->exec_key == key) && repeat && !capture_layers(d, key, s_comp)) d->graph_off = true;
            if (d->exec && d->exec_key == key)
                return kvpi::cuda_status(cudaGraphLaunch(d->exec, s_comp), "decoder graph launch");
        }
    }
    return enqueue_layers(d, n, q, knew, vnew, out, s_comp);
}

// Uploads staging buffer `buf` into the device meta region on stream s; the buffer is the next one's to write.
int upload_meta(kvp_decoder* d, int n, cudaStream_t s, int buf) {
    Staging& st = d->stg[buf];
    const size_t ints = static_cast<size_t>(n) * d->cfg.max_blocks_per_seq + static_cast<size_t>(n) + st.pairs.size();
    cudaError_t e = cudaMemcpyAsync(d->d_meta(), st.h, ints * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return kvpi::cuda_status(e, "decoder metadata upload");
    e = cudaEventRecord(st.ev, s);
    d->next = 1 - buf;
    return kvpi::cuda_status(e, "decoder record");
}

// Staging buffer `buf` may still be read by an earlier step's upload.
int wait_staging(kvp_decoder* d, int buf) {
    return kvpi::cuda_status(cudaEventSynchronize(d->stg[buf].ev), "decoder staging wait");
}

// The staged metadata of a step over `rids`: the planned step's (which must be this batch), re-read from the
// manager if the caller changed any table since the plan, or else this step's bookkeeping now.  Sets *buf.
int stage_step(kvp_decoder* d, const int64_t* rids, int n, int* buf) {
    if (d->planned) {
        d->planned = false;
        const Staging& st = d->stg[d->plan_buf];
        if (st.rids.size() != static_cast<size_t>(n) ||
            std::memcmp(st.rids.data(), rids, sizeof(int64_t) * static_cast<size_t>(n)) != 0)
            return kvpi::fail(KVP_EINVAL, "the step's batch differs from the planned batch (same requests, same order)");
        *buf = d->plan_buf;
        return d->mgr->m.table_changes() == d->plan_changes ? KVP_OK : restage(d, rids, n, *buf);
    }
    *buf = d->next;
    const int rc = wait_staging(d, *buf);
    return rc != KVP_OK ? rc : host_step(d, rids, n, *buf);
}

// Makes the decoder's device current for the scope of a call (its streams, events and launches belong to it).
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <class F>
int guarded(F&& f) {
    kvpi::clear_error();
    try {
        return f();
    } catch (const std::invalid_argument& e) {
        return kvpi::fail(KVP_EINVAL, e.what());
    } catch (const std::exception& e) {
        return kvpi::fail(KVP_ESTATE, e.what());
    }
}

// Uses stream memory operations for the input-ready flags if the driver has cuStreamWriteValue32 and it works
// both directly and captured in a graph (probed once on the decoder's first flag word, left zero); otherwise the
// flags are set by copies.
void probe_write_value(kvp_decoder* d) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !f) {
        cudaGetLastError();
        return;
    }
    const auto fn = reinterpret_cast<kvp_decoder::WriteValueFn>(f);
    const CUdeviceptr flag = reinterpret_cast<CUdeviceptr>(d->d_flags());
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ex = nullptr;
    int32_t v = 0;
    bool ok = cudaStreamBeginCapture(d->s_comp, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (ok) {
        const bool wrote = fn(d->s_comp, flag, 1u, 0u) == CUDA_SUCCESS;
        ok = cudaStreamEndCapture(d->s_comp, &g) == cudaSuccess && wrote && g;
    }
    ok = ok && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess && cudaGraphLaunch(ex, d->s_comp) == cudaSuccess &&
         cudaMemcpyAsync(&v, d->d_flags(), sizeof(v), cudaMemcpyDeviceToHost, d->s_comp) == cudaSuccess &&
         cudaStreamSynchronize(d->s_comp) == cudaSuccess && v == 1;
    ok = ok && cudaMemsetAsync(d->d_flags(), 0, sizeof(int32_t), d->s_comp) == cudaSuccess &&
         fn(d->s_comp, flag, 1u, 0u) == CUDA_SUCCESS &&
         cudaMemcpyAsync(&v, d->d_flags(), sizeof(v), cudaMemcpyDeviceToHost, d->s_comp) == cudaSuccess &&
         cudaStreamSynchronize(d->s_comp) == cudaSuccess && v == 1;
    if (ex) cudaGraphExecDestroy(ex);
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    cudaMemsetAsync(d->d_flags(), 0, sizeof(int32_t), d->s_comp);
    cudaStreamSynchronize(d->s_comp);
    cudaGetLastError();
    if (ok) d->write_value = fn;
}

}  // namespace

extern "C" {

KVP_API size_t kvp_decoder_workspace_size(const kvp_decoder_config* c) {
    if (check_config(c) != KVP_OK) return 0;
    return layout_of(*c).total;
}

KVP_API kvp_decoder* kvp_decoder_create(const kvp_decoder_config* c, kvp_mgr* mgr) {
    kvpi::clear_error();
    if (check_config(c) != KVP_OK) return nullptr;
    if (!mgr || !c->k_cache || !c->v_cache || !c->workspace) {
        kvpi::fail(KVP_EINVAL, "null manager, pool or workspace");
        return nullptr;
    }
    if (mgr->m.block_size() != c->block_size || mgr->m.total_blocks() > c->num_blocks) {
        kvpi::fail(KVP_EINVAL, "manager block size / pool size differ from the decoder's");
        return nullptr;
    }
    if (c->split_tiles > 0) {
        const long long max_tiles = (static_cast<long long>(c->max_blocks_per_seq) * c->block_size + 15) / 16;
        if ((max_tiles + c->split_tiles - 1) / c->split_tiles > kMaxSplitsCap) {
            kvpi::fail(KVP_EINVAL, "split_tiles gives more than 64 splits per sequence; raise it or pass 0");
            return nullptr;
        }
    }
    {
        int cur = -1;
        cudaPointerAttributes at{};
        const bool ok_dev = cudaGetDevice(&cur) == cudaSuccess && cudaPointerGetAttributes(&at, c->k_cache) == cudaSuccess &&
                            at.type == cudaMemoryTypeDevice && at.device == cur;
        if (!ok_dev) {
            cudaGetLastError();
            kvpi::fail(KVP_EINVAL, "the pools must be device memory of the current device");
            return nullptr;
        }
    }
    Layout lay = layout_of(*c);
    if (c->workspace_bytes < lay.total || (reinterpret_cast<uintptr_t>(c->workspace) & 255u)) {
        kvpi::fail(KVP_ENOSPACE, "decoder workspace smaller than kvp_decoder_workspace_size() or not 256-byte aligned");
        return nullptr;
    }
    auto* d = new (std::nothrow) kvp_decoder();
    if (!d) {
        kvpi::fail(KVP_ESTATE, "out of host memory");
        return nullptr;
    }
    d->cfg = *c;
    d->mgr = mgr;
    d->lay = lay;
    d->ws = static_cast<char*>(c->workspace);
    d->layer_stride = c->layer_stride > 0 ? c->layer_stride
                                          : c->num_blocks * c->block_size * static_cast<int64_t>(c->kv_heads) * c->head_dim;
    d->meta_bytes = lay.status - lay.meta;
    cudaGetDevice(&d->device);
    bool ok = true;
    for (Staging& b : d->stg) {
        ok = ok && cudaHostAlloc(reinterpret_cast<void**>(&b.h), d->meta_bytes, cudaHostAllocDefault) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&b.ev, cudaEventDisableTiming) == cudaSuccess;
    }
    ok = ok && cudaHostAlloc(reinterpret_cast<void**>(&d->h_one), sizeof(int32_t), cudaHostAllocDefault) == cudaSuccess;
    if (ok) *d->h_one = 1;
    ok = ok && cudaStreamCreateWithFlags(&d->s_in, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&d->s_comp, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&d->s_out, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&d->ev_fork, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&d->ev_join_in, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&d->ev_join_out, cudaEventDisableTiming) == cudaSuccess;
    d->ev_att.resize(static_cast<size_t>(c->num_layers));
    for (int l = 0; ok && l < c->num_layers; ++l)
        ok = cudaEventCreateWithFlags(&d->ev_att[static_cast<size_t>(l)], cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaMemsetAsync(d->d_status(), 0, sizeof(int32_t), d->s_comp) == cudaSuccess;
    ok = ok && cudaMemsetAsync(d->d_flags(), 0, sizeof(int32_t) * static_cast<size_t>(c->num_layers), d->s_comp) == cudaSuccess;
    // The attention workspace's merge counters start at zero and every completed call leaves them zero.
    if (lay.attn_bytes) ok = ok && cudaMemsetAsync(d->ws + lay.attn, 0, lay.attn_bytes, d->s_comp) == cudaSuccess;
    for (Staging& b : d->stg) ok = ok && cudaEventRecord(b.ev, d->s_in) == cudaSuccess;
    ok = ok && cudaStreamSynchronize(d->s_comp) == cudaSuccess;
    if (ok) probe_write_value(d);
    if (!ok) {
        kvpi::fail(KVP_ECUDA, std::string("decoder setup: ") + cudaGetErrorString(cudaGetLastError()));
        delete d;
        return nullptr;
    }
    return d;
}

KVP_API void kvp_decoder_destroy(kvp_decoder* d) {
    if (!d) return;
    DeviceScope scope(d->device);
    cudaStreamSynchronize(d->s_in);
    cudaStreamSynchronize(d->s_comp);
    cudaStreamSynchronize(d->s_out);
    delete d;
}

KVP_API int kvp_decoder_step_device(kvp_decoder* d, const int64_t* rids, int32_t n, const void* q, const void* k_new,
                                    const void* v_new, void* out, void* stream) {
    return guarded([&] {
        if (!d || (n > 0 && (!rids || !q || !k_new || !v_new || !out))) return kvpi::fail(KVP_EINVAL, "null argument");
        if (n < 0 || n > d->cfg.max_seqs) return kvpi::fail(KVP_EINVAL, "n outside [0, max_seqs]");
        if (n == 0) return KVP_OK;
        DeviceScope scope(d->device);
        if (!kvpi::aligned16(k_new) || !kvpi::aligned16(v_new)) return kvpi::fail(KVP_EINVAL, "k_new / v_new must be 16-byte aligned");
        if (d->submitted) {  // a host-buffer step in flight on the decoder's streams reads the same meta region
            const int rw = kvp_decoder_wait(d);
            if (rw != KVP_OK) return rw;
        }
        int buf = 0;
        int rc = stage_step(d, rids, n, &buf);
        if (rc != KVP_OK) return rc;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        rc = upload_meta(d, n, s, buf);
        if (rc != KVP_OK) return rc;
        return enqueue_device(d, n, q, k_new, v_new, out, s, buf);
    });
}

KVP_API int kvp_decoder_host_inputs(kvp_decoder* d, int32_t n, void** q, void** k_new, void** v_new,
                                    size_t* layer_stride) {
    return guarded([&] {
        if (!d || !q || !k_new || !v_new || !layer_stride) return kvpi::fail(KVP_EINVAL, "null argument");
        if (n < 1 || n > d->cfg.max_seqs) return kvpi::fail(KVP_EINVAL, "n outside [1, max_seqs]");
        const kvp_decoder_config& c = d->cfg;
        if ((q_layer_bytes(c, n) | kv_layer_bytes(c, n)) & 15u)
            return kvpi::fail(KVP_EINVAL, "packed inputs need rows of a multiple of 16 bytes");
        if (!d->h_in) {
            DeviceScope scope(d->device);
            const size_t bytes = static_cast<size_t>(c.num_layers) *
                                 (q_layer_bytes(c, c.max_seqs) + 2 * kv_layer_bytes(c, c.max_seqs));
            if (cudaHostAlloc(reinterpret_cast<void**>(&d->h_in), bytes, cudaHostAllocDefault) != cudaSuccess) {
                d->h_in = nullptr;
                return kvpi::cuda_status(cudaGetLastError(), "pinned input buffer");
            }
            d->h_in_bytes = bytes;
        }
        const Inputs in = packed_inputs(c, n, d->h_in);
        *q = const_cast<char*>(in.q);
        *k_new = const_cast<char*>(in.k);
        *v_new = const_cast<char*>(in.v);
        *layer_stride = in.q_stride;
        return KVP_OK;
    });
}

KVP_API int kvp_decoder_plan(kvp_decoder* d, const int64_t* rids, int32_t n) {
    return guarded([&] {
        if (!d || (n > 0 && !rids)) return kvpi::fail(KVP_EINVAL, "null argument");
        if (n < 0 || n > d->cfg.max_seqs) return kvpi::fail(KVP_EINVAL, "n outside [0, max_seqs]");
        if (d->planned) return kvpi::fail(KVP_ESTATE, "a step is already planned (submit it first)");
        if (n == 0) return KVP_OK;
        DeviceScope scope(d->device);
        // The buffer the submitted step uploaded from may still be in flight; the other one is free once the
        // upload before it completed (a step ago).
        const int buf = d->next;
        int rc = wait_staging(d, buf);
        if (rc != KVP_OK) return rc;
        rc = host_step(d, rids, n, buf);
        if (rc != KVP_OK) return rc;
        d->planned = true;
        d->plan_buf = buf;
        d->plan_changes = d->mgr->m.table_changes();
        return KVP_OK;
    });
}

KVP_API int kvp_decoder_wait(kvp_decoder* d) {
    if (!d) return kvpi::fail(KVP_EINVAL, "null argument");
    kvpi::clear_error();
    DeviceScope scope(d->device);
    d->submitted = false;
    return kvpi::cuda_status(cudaStreamSynchronize(d->s_comp), "decoder step");  // outputs are in host memory
}

KVP_API int kvp_decoder_submit(kvp_decoder* d, const int64_t* rids, int32_t n, const void* q, const void* k_new,
                               const void* v_new, void* out) {
    return guarded([&] {
        if (!d || (n > 0 && (!rids || !q || !k_new || !v_new || !out))) return kvpi::fail(KVP_EINVAL, "null argument");
        if (n < 0 || n > d->cfg.max_seqs) return kvpi::fail(KVP_EINVAL, "n outside [0, max_seqs]");
        if (n == 0) return KVP_OK;
        DeviceScope scope(d->device);
        const kvp_decoder_config& c = d->cfg;
        // The device staging of a step's inputs is single: a step still in flight finishes first.
        if (d->submitted) {
            const int rw = kvp_decoder_wait(d);
            if (rw != KVP_OK) return rw;
        }
        const Inputs host = host_inputs_of(d, n, q, k_new, v_new);
        if (!host.packed && d->h_in) {  // pointers into the packed buffer, but not its layout for this n
            const auto inside = [&](const void* x) {
                return static_cast<const char*>(x) >= d->h_in && static_cast<const char*>(x) < d->h_in + d->h_in_bytes;
            };
            if (inside(q) || inside(k_new) || inside(v_new))
                return kvpi::fail(KVP_EINVAL, "inputs in the decoder's packed buffer must be kvp_decoder_host_inputs()'s "
                                              "pointers for this step's n");
        }
        const int rc = [&]() -> int {
            int rc = copy_first_layer(d, n, host);
            if (rc != KVP_OK) return rc;
            int buf = 0;
            rc = stage_step(d, rids, n, &buf);
            if (rc != KVP_OK) return rc;
            // compute stream: metadata, copy-on-write copies, then the step body (copies in, launches, copies out)
            rc = upload_meta(d, n, d->s_comp, buf);
            if (rc != KVP_OK) return rc;
            const int32_t* d_pairs = d->d_meta() + static_cast<size_t>(n) * c.max_blocks_per_seq + n;
            rc = launch_cow(d, d_pairs, d->s_comp, buf);
            if (rc != KVP_OK) return rc;
            bool launched = false;
            if (c.graph && !d->graph_off) {
                GraphKey key;
                key.n = n;
                key.q = q;
                key.k = k_new;
                key.v = v_new;
                key.out = out;
                const bool repeat = key == d->last_full;
                d->last_full = key;
                if (!(d->exec_full && d->full_key == key) && repeat && !capture_host_body(d, key)) d->graph_off = true;
                if (d->exec_full && d->full_key == key) {
                    const cudaError_t e = cudaGraphLaunch(d->exec_full, d->s_comp);
                    if (e != cudaSuccess) return kvpi::cuda_status(e, "decoder graph launch");
                    launched = true;
                }
            }
            if (!launched) {
                rc = enqueue_host_body(d, n, host, static_cast<char*>(out));
                if (rc != KVP_OK) return rc;
            }
            return KVP_OK;
        }();
        if (rc != KVP_OK) {
            // The step's copies read the caller's buffers and may have set input-ready flags: let them finish and
            // clear the flags before any later step.
            cudaStreamSynchronize(d->s_in);
            cudaStreamSynchronize(d->s_out);
            cudaStreamSynchronize(d->s_comp);
            cudaMemsetAsync(d->d_flags(), 0, sizeof(int32_t) * static_cast<size_t>(c.num_layers), d->s_comp);
            cudaStreamSynchronize(d->s_comp);
            return rc;
        }
        d->submitted = true;
        return KVP_OK;
    });
}

KVP_API int kvp_decoder_step(kvp_decoder* d, const int64_t* rids, int32_t n, const void* q, const void* k_new,
                             const void* v_new, void* out) {
    const int rc = kvp_decoder_submit(d, rids, n, q, k_new, v_new, out);
    return rc != KVP_OK || !d || n == 0 ? rc : kvp_decoder_wait(d);
}

KVP_API int kvp_decoder_status(kvp_decoder* d) {
    if (!d) return -KVP_EINVAL;
    DeviceScope scope(d->device);
    cudaStreamSynchronize(d->s_comp);
    int32_t v = 0;
    if (cudaMemcpy(&v, d->d_status(), sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return -KVP_ECUDA;
    return v;
}

}  // extern "C"
