/*
 * kvm_oracle.c -- TEST INFRASTRUCTURE ONLY (see kvm_oracle.h).
 *
 * Plain-C restatement of the reference's reselection path.  Every function
 * cites the reference file:line it follows (paths relative to the
 * CrKcel/kvmem-llama.cpp tree).  Build flags: -O2 -ffp-contract=off, no
 * -ffast-math, so float expressions are evaluated one IEEE operation at a
 * time exactly like the reference's x86-64 baseline build.
 */
#include "kvm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

/* Static-partition parallel for over [0, n) on n_threads pthreads; the
 * reference runs single-threaded, the all-core variant is a timing aid. */
typedef void (*ora_range_fn)(void *ctx, int64_t lo, int64_t hi);
typedef struct {
    ora_range_fn fn;
    void *ctx;
    int64_t lo, hi;
} ora_task;

static void *ora_task_run(void *arg)
{
    ora_task *t = (ora_task *)arg;
    t->fn(t->ctx, t->lo, t->hi);
    return NULL;
}

static void ora_parallel_for(int64_t n, int n_threads, ora_range_fn fn, void *ctx)
{
    if (n_threads <= 1 || n < 2) {
        fn(ctx, 0, n);
        return;
    }
    if (n_threads > 256) {
        n_threads = 256;
    }
    if ((int64_t)n_threads > n) {
        n_threads = (int)n;
    }
    pthread_t th[256];
    ora_task task[256];
    int started[256];
    for (int i = 0; i < n_threads; ++i) {
        task[i].fn = fn;
        task[i].ctx = ctx;
        task[i].lo = n * i / n_threads;
        task[i].hi = n * (i + 1) / n_threads;
        started[i] = pthread_create(&th[i], NULL, ora_task_run, &task[i]) == 0;
        if (!started[i]) {
            ora_task_run(&task[i]);
        }
    }
    for (int i = 0; i < n_threads; ++i) {
        if (started[i]) {
            pthread_join(th[i], NULL);
        }
    }
}

/* ---------------------------------------------------------------- F16 -- */

float ora_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal: shift the leading one up to the implicit bit */
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while (!(man & 0x400u));
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* IEEE binary32 -> binary16, round to nearest, ties to even. */
uint16_t ora_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) {            /* >= 65520: rounds to infinity */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) {             /* below 2^-14: f16 subnormal or 0 */
        if (ax < 0x33000000u) {         /* below 2^-25 */
            return (uint16_t)sign;
        }
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;    /* 14..24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) {
            ++q;
        }
        return (uint16_t)(sign | q);
    }
    const uint32_t e = (ax >> 23) - 112u;
    const uint32_t m = ax & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) {
        ++q;
    }
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------ quantizers --
 * Block formats: src/adapter/llama-kvmem-stagein.cu:19-30 (q8_0 = f16 d +
 * 32 int8, 34 B; q4_0 = f16 d + 16 nibble bytes, 18 B).  q5_0 = f16 d +
 * 32-bit high-bit mask + 16 nibble bytes, 22 B (ggml block_q5_0; the
 * reference repo has no q5_0 source, gguf-py 0.19.0 quants.Q5_0 is its
 * oracle).
 */

uint64_t ora_row_bytes(int type, uint32_t n_embd)
{
    switch (type) {
    case ORA_TYPE_F16:  return (uint64_t)n_embd * 2u;
    case ORA_TYPE_Q8_0: return (uint64_t)(n_embd / 32u) * 34u;
    case ORA_TYPE_Q4_0: return (uint64_t)(n_embd / 32u) * 18u;
    case ORA_TYPE_Q5_0: return (uint64_t)(n_embd / 32u) * 22u;
    default:            return 0;
    }
}

static void put_f16(uint8_t *p, float v)
{
    const uint16_t h = ora_f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xffu);
    p[1] = (uint8_t)(h >> 8);
}

/* q8_0: llama-kvmem-stagein.cu:180-198 (d = amax/127, id = d ? 1/d : 0,
 * q = roundf(x*id)), which mirrors ggml's quantize_row_q8_0_ref. */
void ora_quantize_q8_0(const float *x, int64_t n, uint8_t *y)
{
    const int64_t nb = n / 32;
    for (int64_t i = 0; i < nb; ++i) {
        const float *src = x + i * 32;
        uint8_t *blk = y + i * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(src[j]));   /* NaN-blind */
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        put_f16(blk, d);
        for (int j = 0; j < 32; ++j) {
            const float v = src[j] * id;
            blk[2 + j] = (uint8_t)(int8_t)roundf(v);
        }
    }
}

/* Signed value of the first element with the largest magnitude
 * (llama-kvmem-stagein.cu:207-214: strict `amax < fabsf(v)`). */
static float first_absmax(const float *src)
{
    float amax = 0.0f;
    float vmax = 0.0f;
    for (int j = 0; j < 32; ++j) {
        const float v = src[j];
        if (amax < fabsf(v)) {
            amax = fabsf(v);
            vmax = v;
        }
    }
    return vmax;
}

/* q4_0: llama-kvmem-stagein.cu:200-233 (d = vmax/-8, q = min(15,
 * (int)(x*id + 8.5f)), element j in the low nibble, j+16 in the high). */
void ora_quantize_q4_0(const float *x, int64_t n, uint8_t *y)
{
    const int64_t nb = n / 32;
    for (int64_t i = 0; i < nb; ++i) {
        const float *src = x + i * 32;
        uint8_t *blk = y + i * 18;
        const float vmax = first_absmax(src);
        const float d = vmax / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        put_f16(blk, d);
        for (int j = 0; j < 16; ++j) {
            const float x0 = src[j] * id;
            const float x1 = src[j + 16] * id;
            int q0 = (int)(x0 + 8.5f);
            int q1 = (int)(x1 + 8.5f);
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            blk[2 + j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
        }
    }
}

/* q5_0: ggml block_q5_0 (d = vmax/-16, q = min(31, (int)(x*id + 16.5f)),
 * low nibbles packed like q4_0, bit 4 of element i at bit i of qh). */
void ora_quantize_q5_0(const float *x, int64_t n, uint8_t *y)
{
    const int64_t nb = n / 32;
    for (int64_t i = 0; i < nb; ++i) {
        const float *src = x + i * 32;
        uint8_t *blk = y + i * 22;
        const float vmax = first_absmax(src);
        const float d = vmax / -16.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        put_f16(blk, d);
        uint32_t qh = 0;
        for (int j = 0; j < 16; ++j) {
            const float x0 = src[j] * id;
            const float x1 = src[j + 16] * id;
            int q0 = (int)(x0 + 16.5f);
            int q1 = (int)(x1 + 16.5f);
            if (q0 > 31) q0 = 31;
            if (q1 > 31) q1 = 31;
            blk[6 + j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
            qh |= (uint32_t)((q0 >> 4) & 1) << j;
            qh |= (uint32_t)((q1 >> 4) & 1) << (j + 16);
        }
        blk[2] = (uint8_t)(qh & 0xffu);
        blk[3] = (uint8_t)((qh >> 8) & 0xffu);
        blk[4] = (uint8_t)((qh >> 16) & 0xffu);
        blk[5] = (uint8_t)(qh >> 24);
    }
}

typedef struct {
    int type;
    const uint16_t *src;
    uint32_t n_embd;
    uint64_t rb;
    uint8_t *dst;
} quant_rows_ctx;

static void quant_rows_range(void *vctx, int64_t lo, int64_t hi)
{
    const quant_rows_ctx *c = (const quant_rows_ctx *)vctx;
    float *row = (float *)malloc(sizeof(float) * 4096u);
    for (int64_t r = lo; r < hi; ++r) {
        const uint16_t *s = c->src + r * (int64_t)c->n_embd;
        uint8_t *o = c->dst + (uint64_t)r * c->rb;
        for (uint32_t c0 = 0; c0 < c->n_embd; c0 += 4096u) {
            const uint32_t nc = c->n_embd - c0 < 4096u ? c->n_embd - c0 : 4096u;
            uint8_t *oc = o + ora_row_bytes(c->type, c0);
            if (c->type == ORA_TYPE_F16) {
                memcpy(oc, s + c0, (size_t)nc * 2u);
                continue;
            }
            for (uint32_t j = 0; j < nc; ++j) {
                row[j] = ora_f16_to_f32(s[c0 + j]);
            }
            if (c->type == ORA_TYPE_Q8_0) {
                ora_quantize_q8_0(row, nc, oc);
            } else if (c->type == ORA_TYPE_Q4_0) {
                ora_quantize_q4_0(row, nc, oc);
            } else {
                ora_quantize_q5_0(row, nc, oc);
            }
        }
    }
    free(row);
}

int ora_quantize_rows_f16(int type, const uint16_t *src, int64_t n_rows,
                          uint32_t n_embd, uint8_t *dst, int n_threads)
{
    const uint64_t rb = ora_row_bytes(type, n_embd);
    if (rb == 0 || n_embd % 32u != 0) {
        return -1;
    }
    quant_rows_ctx c = { type, src, n_embd, rb, dst };
    ora_parallel_for(n_rows, n_threads, quant_rows_range, &c);
    return 0;
}

/* ------------------------------------------------------------ transforms --
 * RoPE: kvmem/src/host/rope.cpp:8-45 (theta table, then per token and head
 * x0*c - x1*s, x0*s + x1*c with c = cos(pos*theta_i), s = sin(pos*theta_i)).
 * Hadamard: fwht_kernel, src/adapter/llama-kvmem-stagein.cu:104-130.
 * attn_rot sizes: src/adapter/llama-kvmem-quant.h:22-40.
 */
void ora_rope_theta(uint32_t n_rot, float freq_base, float freq_scale, float *theta)
{
    for (uint32_t i = 0; i < n_rot / 2u; ++i) {
        theta[i] = powf(freq_base, -2.0f * (float)i / (float)n_rot);
        theta[i] *= freq_scale;
    }
}

void ora_rope_neox_rows(float *x, int64_t n_tokens, uint32_t n_head, uint32_t head_dim,
                        uint32_t n_rot, int32_t pos0, const float *theta)
{
    const uint32_t half = n_rot / 2u;
    for (int64_t t = 0; t < n_tokens; ++t) {
        const float pos = (float)(pos0 + (int32_t)t);
        for (uint32_t h = 0; h < n_head; ++h) {
            float *row = x + ((uint64_t)t * n_head + h) * head_dim;
            for (uint32_t i = 0; i < half; ++i) {
                const float c = cosf(pos * theta[i]);
                const float s = sinf(pos * theta[i]);
                const float x0 = row[i];
                const float x1 = row[i + half];
                row[i] = x0 * c - x1 * s;
                row[i + half] = x0 * s + x1 * c;
            }
        }
    }
}

void ora_fwht_rows(float *x, int64_t n_rows, uint32_t n_embd, uint32_t nrot)
{
    if (nrot == 0 || n_embd % nrot != 0) {
        return;
    }
    const float scale = 1.0f / sqrtf((float)nrot);
    const int64_t chunks = n_rows * (int64_t)(n_embd / nrot);
    for (int64_t c = 0; c < chunks; ++c) {
        float *v = x + c * (int64_t)nrot;
        for (uint32_t i = 0; i < nrot; ++i) {
            v[i] = v[i] * scale;
        }
        for (uint32_t h = 1; h < nrot; h *= 2) {
            for (uint32_t i = 0; i < nrot; i += 2 * h) {
                for (uint32_t j = 0; j < h; ++j) {
                    const float a = v[i + j];
                    const float b = v[i + j + h];
                    v[i + j] = a + b;
                    v[i + j + h] = a - b;
                }
            }
        }
    }
}

uint32_t ora_attn_rot_nrot(int type, uint32_t head_dim, int is_k)
{
    if (type != ORA_TYPE_Q8_0 && type != ORA_TYPE_Q4_0 && type != ORA_TYPE_Q5_0) {
        return 0;
    }
    if (head_dim < 64 || head_dim % 64 != 0) {
        return 0;
    }
    if (!is_k) {
        return 64;
    }
    uint32_t nrot = 64;
    do {
        nrot *= 2;
    } while (head_dim % nrot == 0);
    return nrot / 2;
}

/* ---------------------------------------------------------------- mean-K --
 * kvmem/src/host/raw_kv_store.cpp:204-223 (add_mean_f32: zero-filled F32
 * accumulator, tokens added in order) and :976-1000 (mean_k: sum * (1.0f/n),
 * never normalized in place; zeros when no statistics exist).
 */
void ora_block_sum_f16(const uint16_t *k, uint32_t n_tokens, uint32_t n_embd,
                       uint64_t row_stride, float *sum)
{
    for (uint32_t d = 0; d < n_embd; ++d) {
        sum[d] = 0.0f;
    }
    for (uint32_t t = 0; t < n_tokens; ++t) {
        const uint16_t *row = k + (uint64_t)t * row_stride;
        for (uint32_t d = 0; d < n_embd; ++d) {
            sum[d] += ora_f16_to_f32(row[d]);
        }
    }
}

void ora_mean_k(const float *sum, uint32_t mean_tokens, uint32_t n_embd,
                float *out)
{
    if (mean_tokens == 0) {
        for (uint32_t d = 0; d < n_embd; ++d) {
            out[d] = 0.0f;
        }
        return;
    }
    const float inv = 1.0f / (float)mean_tokens;
    for (uint32_t d = 0; d < n_embd; ++d) {
        out[d] = sum[d] * inv;
    }
}

/* ---------------------------------------------------------------- scorer --
 * src/adapter/llama-memory-kvmem.cpp:2869-2916.  Same loop nest, same types:
 * per-head dot/nq/nk accumulate in float over d in order, the head result
 * dot/(sqrt(nq)*sqrt(nk)+1e-6f) is added to a double per layer, the layer
 * contributes layer/H_kv to a double per block, and the block score is the
 * mean over layers that have a query (q_count > 0).  Blocks without stored
 * data score 0.
 */
typedef struct {
    const float *sums;
    const uint32_t *mean_tok;
    const uint8_t *has_block;
    uint32_t n_blocks, n_layer;
    const float *q_sum;
    const uint32_t *q_count;
    uint32_t n_head_kv, n_head_q, head_dim;
    double *scores, *terms;
} score_ctx;

static void score_range(void *vctx, int64_t lo, int64_t hi)
{
    const score_ctx *c = (const score_ctx *)vctx;
    const uint32_t n_head_kv = c->n_head_kv;
    const uint32_t n_head_q = c->n_head_q;
    const uint32_t head_dim = c->head_dim;
    const uint32_t n_blocks = c->n_blocks;
    const uint32_t n_embd = n_head_kv * head_dim;
    const uint32_t g = n_head_kv == 0 ? 1u : n_head_q / n_head_kv;
    const uint32_t gg = g > 1u ? g : 1u;
    const uint32_t hk = n_head_kv > 1u ? n_head_kv : 1u;
    float *mk = (float *)malloc(sizeof(float) * (n_embd ? n_embd : 1u));
    float *qh = (float *)malloc(sizeof(float) * (head_dim ? head_dim : 1u));
    for (int64_t bi = lo; bi < hi; ++bi) {
        const uint32_t b = (uint32_t)bi;
        if (!c->has_block[b]) {
            c->scores[b] = 0.0;
            continue;
        }
        double acc = 0;
        uint32_t nlay = 0;
        for (uint32_t il = 0; il < c->n_layer; ++il) {
            if (c->q_count[il] == 0) {
                continue;
            }
            ora_mean_k(c->sums + ((uint64_t)il * n_blocks + b) * n_embd,
                       c->mean_tok[(uint64_t)il * n_blocks + b], n_embd, mk);
            double layer = 0;
            const float invq = 1.0f / (float)(c->q_count[il] * gg);
            for (uint32_t h = 0; h < n_head_kv; ++h) {
                for (uint32_t d = 0; d < head_dim; ++d) {
                    qh[d] = 0.0f;
                }
                for (uint32_t gi = 0; gi < g; ++gi) {
                    const uint32_t qh_i = h * g + gi;
                    if (qh_i >= n_head_q) {
                        break;
                    }
                    const float *q = c->q_sum + (uint64_t)il * n_head_q * head_dim
                                   + (uint64_t)qh_i * head_dim;
                    for (uint32_t d = 0; d < head_dim; ++d) {
                        qh[d] += q[d];
                    }
                }
                const float *kh = mk + h * head_dim;
                float dot = 0, nq = 0, nk = 0;
                for (uint32_t d = 0; d < head_dim; ++d) {
                    const float qv = qh[d] * invq;
                    dot += qv * kh[d];
                    nq += qv * qv;
                    nk += kh[d] * kh[d];
                }
                layer += dot / (sqrtf(nq) * sqrtf(nk) + 1e-6f);
            }
            const double term = layer / (double)hk;
            if (c->terms) {
                c->terms[(uint64_t)il * n_blocks + b] = term;
            }
            acc += term;
            nlay++;
        }
        c->scores[b] = nlay ? acc / nlay : 0;
    }
    free(mk);
    free(qh);
}

void ora_score(const float *sums, const uint32_t *mean_tok,
               const uint8_t *has_block, uint32_t n_blocks, uint32_t n_layer,
               const float *q_sum, const uint32_t *q_count, uint32_t n_head_kv,
               uint32_t n_head_q, uint32_t head_dim, double *scores,
               double *terms, int n_threads)
{
    if (terms) {
        memset(terms, 0, sizeof(double) * (size_t)n_layer * n_blocks);
    }
    score_ctx c = { sums, mean_tok, has_block, n_blocks, n_layer, q_sum,
                    q_count, n_head_kv, n_head_q, head_dim, scores, terms };
    ora_parallel_for(n_blocks, n_threads, score_range, &c);
}

/* ------------------------------------------------------------- selection --
 * kvmem/src/host/kvmem_store.cpp:482-623 (pick_topk_ungrouped, TopK policy):
 * select everything when n <= budget; else keep sinks 0..sink-1, then the
 * mandatory list walked from its end (newest first), then `recent` suffix
 * blocks, each only while kept < budget; fill the rest with the best
 * candidates ordered by score descending then block id descending.  The
 * reference uses nth_element; under this strict total order a full sort
 * selects the same set.  Output is ascending.
 */
static const double *g_sort_scores;

static int better_cmp(const void *pa, const void *pb)
{
    const uint32_t a = *(const uint32_t *)pa;
    const uint32_t b = *(const uint32_t *)pb;
    const double sa = g_sort_scores[a];
    const double sb = g_sort_scores[b];
    if (sa != sb) {
        return sa > sb ? -1 : 1;
    }
    return a > b ? -1 : (a < b ? 1 : 0);
}

/* Candidate order of pick_semantic_groups (kvmem_store.cpp:712-716): score
 * descending, then group index descending. */
typedef struct ora_group_cand {
    uint32_t group, first, last;
    double score;
} ora_group_cand;

static int group_cmp(const void *pa, const void *pb)
{
    const ora_group_cand *a = (const ora_group_cand *)pa;
    const ora_group_cand *b = (const ora_group_cand *)pb;
    if (a->score != b->score) {
        return a->score > b->score ? -1 : 1;
    }
    return a->group > b->group ? -1 : (a->group < b->group ? 1 : 0);
}

uint32_t ora_pick_semantic_groups(const ora_cfg *cfg, uint32_t n, uint64_t covered_tokens,
                                  const uint32_t *spans, const double *scores,
                                  uint32_t n_groups, const uint32_t *mandatory,
                                  uint32_t n_mandatory, uint32_t *out)
{
    if (n == 0) {
        return 0;
    }
    const uint32_t budget = cfg->budget_blocks;
    if (budget == 0 || n <= budget) {
        for (uint32_t i = 0; i < n; ++i) {
            out[i] = i;
        }
        return n;
    }
    uint8_t *kept = (uint8_t *)calloc(n, 1);
    uint32_t kept_count = 0;
#define ORA_KEEP(id_)                                                    \
    do {                                                                 \
        const uint32_t id__ = (id_);                                     \
        if (id__ < n && !kept[id__]) {                                   \
            kept[id__] = 1;                                              \
            ++kept_count;                                                \
        }                                                                \
    } while (0)
    const uint32_t sink = cfg->sink_blocks < n ? cfg->sink_blocks : n;
    const uint32_t recent = cfg->recent_blocks < n ? cfg->recent_blocks : n;
    for (uint32_t i = 0; i < sink && kept_count < budget; ++i) {
        ORA_KEEP(i);
    }
    for (uint32_t i = n_mandatory; i > 0 && kept_count < budget; --i) {
        ORA_KEEP(mandatory[i - 1]);
    }
    for (uint32_t i = 0; i < recent && kept_count < budget; ++i) {
        ORA_KEEP(n - 1 - i);
    }
    const uint32_t bt = cfg->block_tokens ? cfg->block_tokens : 1;
    ora_group_cand *cand = (ora_group_cand *)malloc(sizeof(ora_group_cand) * (n_groups ? n_groups : 1));
    uint32_t nc = 0;
    for (uint32_t g = 0; g < n_groups; ++g) {
        const uint32_t begin = spans[2 * g];
        const uint32_t end = spans[2 * g + 1];
        if (end <= begin || begin >= covered_tokens) {
            continue;
        }
        const uint32_t capped = end < covered_tokens ? end : (uint32_t)covered_tokens;
        const uint32_t first = begin / bt;
        uint32_t last = (capped - 1) / bt;
        if (first >= n) {
            continue;
        }
        if (last > n - 1) {
            last = n - 1;
        }
        cand[nc].group = g;
        cand[nc].first = first;
        cand[nc].last = last;
        cand[nc].score = scores[g];
        ++nc;
    }
    qsort(cand, nc, sizeof(ora_group_cand), group_cmp);
    for (uint32_t c = 0; c < nc; ++c) {
        uint32_t fresh = 0;
        for (uint32_t id = cand[c].first; id <= cand[c].last; ++id) {
            fresh += kept[id] ? 0u : 1u;
        }
        if (fresh > budget - kept_count) {
            continue;
        }
        for (uint32_t id = cand[c].first; id <= cand[c].last; ++id) {
            ORA_KEEP(id);
        }
        if (kept_count == budget) {
            break;
        }
    }
#undef ORA_KEEP
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (kept[i]) {
            out[m++] = i;
        }
    }
    free(cand);
    free(kept);
    return m;
}

uint32_t ora_pick_topk(const ora_cfg *cfg, const double *scores, uint32_t n,
                       const uint32_t *mandatory, uint32_t n_mandatory,
                       uint32_t *out)
{
    if (n == 0) {
        return 0;
    }
    const uint32_t budget = cfg->budget_blocks;
    if (budget == 0 || n <= budget) {
        for (uint32_t i = 0; i < n; ++i) {
            out[i] = i;
        }
        return n;
    }
    const uint32_t sink = cfg->sink_blocks < n ? cfg->sink_blocks : n;
    const uint32_t recent = cfg->recent_blocks < n ? cfg->recent_blocks : n;
    uint8_t *kept = (uint8_t *)calloc(n, 1);
    uint32_t kept_count = 0;
#define ORA_KEEP(id_)                                                    \
    do {                                                                 \
        const uint32_t id__ = (id_);                                     \
        if (id__ < n && !kept[id__]) {                                   \
            kept[id__] = 1;                                              \
            ++kept_count;                                                \
        }                                                                \
    } while (0)
    for (uint32_t i = 0; i < sink && kept_count < budget; ++i) {
        ORA_KEEP(i);
    }
    for (uint32_t i = n_mandatory; i > 0 && kept_count < budget; --i) {
        ORA_KEEP(mandatory[i - 1]);
    }
    for (uint32_t i = 0; i < recent && kept_count < budget; ++i) {
        ORA_KEEP(n - 1 - i);
    }
    if (kept_count < budget) {
        uint32_t *cand = (uint32_t *)malloc(sizeof(uint32_t) * n);
        uint32_t nc = 0;
        for (uint32_t i = 0; i < n; ++i) {
            if (!kept[i]) {
                cand[nc++] = i;
            }
        }
        const uint32_t need = budget - kept_count;
        uint32_t take = nc;
        if (need < nc) {
            g_sort_scores = scores;
            qsort(cand, nc, sizeof(uint32_t), better_cmp);
            take = need;
        }
        for (uint32_t i = 0; i < take; ++i) {
            ORA_KEEP(cand[i]);
        }
        free(cand);
    }
#undef ORA_KEEP
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (kept[i]) {
            out[m++] = i;
        }
    }
    free(kept);
    return m;
}

/* ------------------------------------------------------------------ diff --
 * kvmem/src/host/kvmem_store.cpp:758-882 (set_selection).
 */
static int cmp_u32(const void *pa, const void *pb)
{
    const uint32_t a = *(const uint32_t *)pa;
    const uint32_t b = *(const uint32_t *)pb;
    return a < b ? -1 : (a > b ? 1 : 0);
}

int ora_set_selection(const ora_cfg *cfg, ora_blocks *b, uint32_t n,
                      const uint32_t *ids_in, uint32_t n_ids,
                      int force_raw_refresh, ora_plan *p)
{
    uint32_t *ids = (uint32_t *)malloc(sizeof(uint32_t) * (n_ids ? n_ids : 1u));
    memcpy(ids, ids_in, sizeof(uint32_t) * n_ids);
    qsort(ids, n_ids, sizeof(uint32_t), cmp_u32);
    uint32_t m = 0;
    for (uint32_t i = 0; i < n_ids; ++i) {
        if (m > 0 && ids[m - 1] == ids[i]) {
            continue;
        }
        ids[m++] = ids[i];
    }
    uint32_t k = 0;
    for (uint32_t i = 0; i < m; ++i) {
        if (ids[i] < n) {
            ids[k++] = ids[i];
        }
    }

    p->n_stage_in = p->n_stage_out = p->n_remaps = 0;
    p->total_window_tokens = 0;
    p->selection_overlap_blocks = p->gpu_reused_blocks = 0;
    p->retained_position_stable = p->retained_position_moved = 0;

    uint8_t *now = (uint8_t *)calloc(n ? n : 1u, 1);
    uint8_t *was = (uint8_t *)calloc(n ? n : 1u, 1);
    for (uint32_t i = 0; i < k; ++i) {
        now[ids[i]] = 1;
    }
    for (uint32_t i = 0; i < n; ++i) {
        was[i] = b->in_working_set[i];
        if (b->in_working_set[i] && now[i]) {
            ++p->selection_overlap_blocks;
        }
    }
    const int force_full_reload = !cfg->optimize_stage_in;
    for (uint32_t i = 0; i < n; ++i) {
        if (b->tier[i] == ORA_TIER_GPU && (!now[i] || force_full_reload)) {
            p->stage_out[p->n_stage_out++] = i;
            b->in_working_set[i] = 0;
        }
    }
    const int imm = cfg->immutable_source_k != 0;
    uint32_t window_pos = 0;
    int rc = 0;
    for (uint32_t s = 0; s < k; ++s) {
        const uint32_t id = ids[s];
        const int reusable = was[id] && b->tier[id] == ORA_TIER_GPU;
        if (reusable) {
            if (b->baked_pos[id] == (int64_t)window_pos) {
                ++p->retained_position_stable;
            } else {
                ++p->retained_position_moved;
            }
            if (!force_full_reload) {
                ++p->gpu_reused_blocks;
            }
        }
        const int cold = b->tier[id] != ORA_TIER_GPU || force_full_reload;
        if (!b->in_working_set[id]) {
            p->stage_in[p->n_stage_in++] = id;
        }
        const int64_t baked = b->baked_pos[id];
        const int wkr = !cold;
        const int same = baked == (int64_t)window_pos;
        const int skip = same && (!imm || wkr) && !force_raw_refresh;
        int raw = 0;
        const uint64_t delta = (uint64_t)(baked > (int64_t)window_pos
                                              ? baked - (int64_t)window_pos
                                              : (int64_t)window_pos - baked);
        if (imm && (cold || !same)) {
            const uint64_t lim = cfg->immutable_refresh_abs_delta_tokens;
            const int remap_limit = cfg->immutable_refresh_remaps > 0 &&
                b->remap_count[id] >= cfg->immutable_refresh_remaps;
            const uint64_t have = b->remap_abs_delta[id];
            const int delta_limit = lim > 0 &&
                (have >= lim || delta >= lim - (have < lim ? have : lim));
            const uint64_t maxp = cfg->immutable_max_baked_position;
            const int out_of_range = maxp > 0 &&
                (baked < 0 || (uint64_t)baked + b->n_tokens[id] > maxp);
            raw = cold || remap_limit || delta_limit || out_of_range;
        }
        if (imm && force_raw_refresh) {
            raw = 1;
        }
        if (skip && raw) {
            rc = -1;        /* std::logic_error in the reference */
            break;
        }
        const uint32_t r = p->n_remaps++;
        p->rm_block_id[r] = id;
        p->rm_n_tokens[r] = b->n_tokens[id];
        p->rm_from_base[r] = (int32_t)baked;
        p->rm_to_base[r] = (int32_t)window_pos;
        p->rm_working_k_resident[r] = (uint8_t)wkr;
        p->rm_skip[r] = (uint8_t)skip;
        p->rm_raw_refresh[r] = (uint8_t)raw;

        b->in_working_set[id] = 1;
        if (!skip) {
            if (raw) {
                b->remap_count[id] = 0;
                b->remap_abs_delta[id] = 0;
            } else {
                ++b->remap_count[id];
                b->remap_abs_delta[id] += delta;
            }
        }
        b->baked_pos[id] = (int64_t)window_pos;
        window_pos += b->n_tokens[id];
    }
    p->total_window_tokens = window_pos;
    free(now);
    free(was);
    free(ids);
    return rc;
}

/* ---------------------------------------------------------------- layout --
 * src/adapter/llama-memory-kvmem.cpp:931-1254 (layout_gpu_slots_by_orig_pos)
 * with reset_slots :621-627 and alloc_slot :693-700: resident blocks sorted
 * by original position get slots 0,1,2,... in that order; a resident block
 * keeps its bytes through a device move, a non-resident one is written from
 * the host store.  Blocks are dense in append order (orig_pos_start =
 * id * block_tokens, kvmem_store.cpp:179-205), so ascending id is
 * chronological order.
 */
int ora_layout(const uint32_t *sel, uint32_t n_sel, const int32_t *slot_before,
               uint32_t n_blocks, int32_t *slot_after, uint32_t *mv_block,
               int32_t *mv_from, int32_t *mv_to, uint32_t *n_moves,
               uint32_t *cold_block, int32_t *cold_to, uint32_t *n_cold)
{
    *n_moves = 0;
    *n_cold = 0;
    for (uint32_t i = 0; i < n_blocks; ++i) {
        slot_after[i] = -1;
    }
    for (uint32_t i = 0; i < n_sel; ++i) {
        const uint32_t id = sel[i];
        slot_after[id] = (int32_t)i;
        if (slot_before[id] >= 0) {
            if (slot_before[id] != (int32_t)i) {
                mv_block[*n_moves] = id;
                mv_from[*n_moves] = slot_before[id];
                mv_to[*n_moves] = (int32_t)i;
                ++*n_moves;
            }
        } else {
            cold_block[*n_cold] = id;
            cold_to[*n_cold] = (int32_t)i;
            ++*n_cold;
        }
    }
    return 0;
}
