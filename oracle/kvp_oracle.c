/*
 * ORACLE -- test infrastructure, not product code.
 *
 * A plain-C restatement of the reference's CPU decode attention over a paged KV cache
 * (prathameshpranjale/paged-kv-cache-manager, src/paged_attention.cpp).  Only the test suite,
 * the smoke check and the CPU-baseline leg of the benchmark load this file's library; the
 * product path never calls it.
 *
 * Layouts (row-major, contiguous), as the reference fixes them in include/kvpage/paged_attention.h:8-21:
 *   q, out        [num_seqs][num_heads][head_dim]                  float
 *   k, v          [num_blocks][block_size][kv_heads][head_dim]     float
 *   tables        [num_seqs][max_blocks]                           int32 (entries past a sequence ignored)
 *   lens          [num_seqs]                                       int32 (>= 1)
 * Query head h reads kv head h / (num_heads / kv_heads); scale = 1/sqrt(head_dim).
 *
 * Every entry point returns 0 on success and -1 where the reference throws std::invalid_argument.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORA_API __attribute__((visibility("default")))

/* Input validation: src/paged_attention.cpp:12-17 (kv_heads > 0, num_heads % kv_heads == 0,
 * every seq_len >= 1 and ceil(seq_len / block_size) <= max_blocks). */
static int ora_check(int nh, int kvh, int bs, int ns, int max_blocks, const int32_t* lens) {
    if (kvh <= 0 || nh % kvh != 0) return -1;
    for (int i = 0; i < ns; ++i) {
        if (lens[i] < 1) return -1;
        if ((lens[i] + bs - 1) / bs > max_blocks) return -1;
    }
    return 0;
}

/* Element offset of (block, slot, kv head): src/paged_attention.cpp:19-21. */
static inline size_t ora_kv_index(int kvh, int hd, int bs, int block, int off, int h) {
    return (((size_t)block * (size_t)bs + (size_t)off) * (size_t)kvh + (size_t)h) * (size_t)hd;
}

/* reference_attention (src/paged_attention.cpp:25-66): per sequence and query head, double-precision
 * scores in token order, max, exp(score - max), sum, then the weighted sum of V divided by the sum.
 * The reference first gathers K/V into a contiguous copy; reading through the table in the same
 * token order gives the same numbers, so the copy is skipped here. */
static void ora_reference_range(int nh, int kvh, int hd, int bs, int max_blocks, const float* q, const float* k,
                                const float* v, const int32_t* tables, const int32_t* lens, float* out, int s0,
                                int s1, double* sc) {
    const int group = nh / kvh;
    const double scale = 1.0 / sqrt((double)hd);
    for (int i = s0; i < s1; ++i) {
        const int n = lens[i];
        const int32_t* table = tables + (size_t)i * (size_t)max_blocks;
        for (int h = 0; h < nh; ++h) {
            const int kh = h / group;
            const float* qh = q + ((size_t)i * nh + h) * (size_t)hd;
            double mx = -INFINITY;
            for (int t = 0; t < n; ++t) {
                const float* kt = k + ora_kv_index(kvh, hd, bs, table[t / bs], t % bs, kh);
                double d = 0.0;
                for (int e = 0; e < hd; ++e) d += (double)qh[e] * (double)kt[e];
                sc[t] = d * scale;
                if (sc[t] > mx) mx = sc[t];
            }
            double sum = 0.0;
            for (int t = 0; t < n; ++t) {
                sc[t] = exp(sc[t] - mx);
                sum += sc[t];
            }
            float* oh = out + ((size_t)i * nh + h) * (size_t)hd;
            for (int e = 0; e < hd; ++e) {
                double acc = 0.0;
                for (int t = 0; t < n; ++t)
                    acc += sc[t] * (double)v[ora_kv_index(kvh, hd, bs, table[t / bs], t % bs, kh) + e];
                oh[e] = (float)(acc / sum);
            }
        }
    }
}

/* paged_attention_cpu (src/paged_attention.cpp:68-114): fp32 online softmax. The context is split into
 * `partitions` interleaved token groups (group p visits tokens p, p+P, ...), each keeping (m, l, acc);
 * the groups are merged at the end, skipping groups that saw no token. */
static void ora_paged_range(int nh, int kvh, int hd, int bs, int max_blocks, const float* q, const float* k,
                            const float* v, const int32_t* tables, const int32_t* lens, float* out, int partitions,
                            int s0, int s1, float* m, float* l, float* acc, float* o) {
    const int group = nh / kvh;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int i = s0; i < s1; ++i) {
        const int n = lens[i];
        const int32_t* table = tables + (size_t)i * (size_t)max_blocks;
        for (int h = 0; h < nh; ++h) {
            const int kh = h / group;
            const float* qh = q + ((size_t)i * nh + h) * (size_t)hd;
            for (int p = 0; p < partitions; ++p) {
                m[p] = -INFINITY;
                l[p] = 0.0f;
            }
            memset(acc, 0, sizeof(float) * (size_t)partitions * (size_t)hd);
            for (int p = 0; p < partitions; ++p) {
                float* ap = acc + (size_t)p * hd;
                for (int t = p; t < n; t += partitions) {
                    const size_t base = ora_kv_index(kvh, hd, bs, table[t / bs], t % bs, kh);
                    float d = 0.0f;
                    for (int e = 0; e < hd; ++e) d += qh[e] * k[base + e];
                    d *= scale;
                    const float m_new = m[p] > d ? m[p] : d;
                    const float corr = expf(m[p] - m_new);
                    const float w = expf(d - m_new);
                    l[p] = l[p] * corr + w;
                    for (int e = 0; e < hd; ++e) ap[e] = ap[e] * corr + w * v[base + e];
                    m[p] = m_new;
                }
            }
            float M = -INFINITY;
            for (int p = 0; p < partitions; ++p)
                if (m[p] > M) M = m[p];
            float L = 0.0f;
            memset(o, 0, sizeof(float) * (size_t)hd);
            for (int p = 0; p < partitions; ++p) {
                if (m[p] == -INFINITY) continue;
                const float c = expf(m[p] - M);
                L += l[p] * c;
                for (int e = 0; e < hd; ++e) o[e] += acc[(size_t)p * hd + e] * c;
            }
            float* oh = out + ((size_t)i * nh + h) * (size_t)hd;
            for (int e = 0; e < hd; ++e) oh[e] = o[e] / L;
        }
    }
}

ORA_API int ora_reference_attention(int nh, int kvh, int hd, int bs, int ns, int max_blocks, const float* q,
                                    const float* k, const float* v, const int32_t* tables, const int32_t* lens,
                                    float* out) {
    if (ora_check(nh, kvh, bs, ns, max_blocks, lens)) return -1;
    int longest = 1;
    for (int i = 0; i < ns; ++i)
        if (lens[i] > longest) longest = lens[i];
    double* sc = (double*)malloc(sizeof(double) * (size_t)longest);
    if (!sc) return -2;
    ora_reference_range(nh, kvh, hd, bs, max_blocks, q, k, v, tables, lens, out, 0, ns, sc);
    free(sc);
    return 0;
}

typedef struct {
    int nh, kvh, hd, bs, max_blocks, partitions, s0, s1, rc;
    const float *q, *k, *v;
    const int32_t *tables, *lens;
    float* out;
} ora_job;

static void* ora_paged_worker(void* arg) {
    ora_job* j = (ora_job*)arg;
    const size_t P = (size_t)j->partitions, D = (size_t)j->hd;
    float* buf = (float*)malloc(sizeof(float) * (2 * P + P * D + D));
    if (!buf) {
        j->rc = -2;
        return NULL;
    }
    ora_paged_range(j->nh, j->kvh, j->hd, j->bs, j->max_blocks, j->q, j->k, j->v, j->tables, j->lens, j->out,
                    j->partitions, j->s0, j->s1, buf, buf + P, buf + 2 * P, buf + 2 * P + P * D);
    free(buf);
    j->rc = 0;
    return NULL;
}

/* Same result as paged_attention_cpu; sequences are divided into `nthreads` contiguous slices that run on
 * separate host threads (the function is pure, so slices are independent). */
ORA_API int ora_paged_attention_cpu_mt(int nh, int kvh, int hd, int bs, int ns, int max_blocks, const float* q,
                                       const float* k, const float* v, const int32_t* tables, const int32_t* lens,
                                       float* out, int partitions, int nthreads) {
    if (ora_check(nh, kvh, bs, ns, max_blocks, lens)) return -1;
    if (partitions < 1) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > ns) nthreads = ns > 0 ? ns : 1;
    ora_job* jobs = (ora_job*)calloc((size_t)nthreads, sizeof(ora_job));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    if (!jobs || !th) {
        free(jobs);
        free(th);
        return -2;
    }
    for (int t = 0; t < nthreads; ++t) {
        ora_job* j = &jobs[t];
        j->nh = nh; j->kvh = kvh; j->hd = hd; j->bs = bs; j->max_blocks = max_blocks; j->partitions = partitions;
        j->s0 = (int)((int64_t)ns * t / nthreads);
        j->s1 = (int)((int64_t)ns * (t + 1) / nthreads);
        j->q = q; j->k = k; j->v = v; j->tables = tables; j->lens = lens; j->out = out;
        j->rc = -3;
    }
    int rc = 0;
    if (nthreads == 1) {
        ora_paged_worker(&jobs[0]);
    } else {
        for (int t = 0; t < nthreads; ++t) pthread_create(&th[t], NULL, ora_paged_worker, &jobs[t]);
        for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    }
    for (int t = 0; t < nthreads; ++t)
        if (jobs[t].rc) rc = jobs[t].rc;
    free(jobs);
    free(th);
    return rc;
}

ORA_API int ora_paged_attention_cpu(int nh, int kvh, int hd, int bs, int ns, int max_blocks, const float* q,
                                    const float* k, const float* v, const int32_t* tables, const int32_t* lens,
                                    float* out, int partitions) {
    return ora_paged_attention_cpu_mt(nh, kvh, hd, bs, ns, max_blocks, q, k, v, tables, lens, out, partitions, 1);
}

/* Round-to-nearest-even float -> bfloat16 bit pattern (NaN kept quiet). Used to build bf16 inputs whose
 * exact float values feed the attention oracle. */
ORA_API void ora_f32_to_bf16(const float* x, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
            y[i] = (uint16_t)((u >> 16) | 0x40u);
            continue;
        }
        const uint32_t lsb = (u >> 16) & 1u;
        u += 0x7fffu + lsb;
        y[i] = (uint16_t)(u >> 16);
    }
}

ORA_API void ora_bf16_to_f32(const uint16_t* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        const uint32_t u = (uint32_t)x[i] << 16;
        memcpy(&y[i], &u, 4);
    }
}
