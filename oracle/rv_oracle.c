/* rv_oracle.c - CPU restatement of Rosevine's Q8_0 CPU-experts MoE path.
 * TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU baseline);
 * see rv_oracle.h for the rules and the reference citations.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off; the AVX2 routine is
 * compiled for avx2+fma by a target attribute and selected at run time).
 */
#include "rv_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define QK 32
#define Q4_BLOCK 18
#define Q8_BLOCK 34

/* ---------------------------------------------------------------- scalars */

/* IEEE half to f32 by fields, subnormals normalised (ops.rs:7-24). */
float rvo_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0 && man == 0) {
        bits = sign;
    } else if (exp == 0) {
        /* leading_zeros of the 32-bit mantissa minus 21 = shift to normalise */
        uint32_t shift = (uint32_t)__builtin_clz(man) - 21;
        uint32_t m = (man << shift) & 0x3ff;
        bits = sign | ((113 - shift) << 23) | (m << 13);
    } else if (exp == 0x1f && man == 0) {
        bits = sign | 0x7f800000u;
    } else if (exp == 0x1f) {
        bits = sign | 0x7fc00000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* f32 to IEEE half, round to nearest even, NaN -> quiet 0x7e00|sign (ops.rs:27-59). */
uint16_t rvo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    int32_t exp = (int32_t)((x >> 23) & 0xff);
    uint32_t man = x & 0x7fffff;
    if (exp == 0xff) return sign | 0x7c00 | (man != 0 ? 0x200 : 0);
    int32_t e = exp - 127 + 15;
    if (e >= 0x1f) return sign | 0x7c00;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half = 1u << (shift - 1);
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t r = m >> shift;
        if (rem > half || (rem == half && (r & 1))) r += 1;
        return sign | (uint16_t)r;
    }
    uint32_t r = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) r += 1; /* carry into the exponent is correct */
    return sign | (uint16_t)r;
}

float rvo_bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float ld_f16(const uint8_t *p) { return rvo_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

static inline float ld_act(const void *x, int dtype, size_t i) {
    return dtype == RVO_BF16 ? rvo_bf16_to_f32(((const uint16_t *)x)[i]) : ((const float *)x)[i];
}

/* Q8_0 quantisation of one row as quantize_row_q8_0_ref (ops.rs:95-105):
 * d = amax / 127 in f32, stored as f16 (RNE); id = 1/d from the f32 d;
 * q = roundf(v * id) (half away from zero), saturated to i8. */
void rvo_quantize_q8_0(const float *x, int k, uint8_t *out) {
    for (int b = 0; b < k / QK; ++b) {
        const float *xs = x + (size_t)b * QK;
        uint8_t *blk = out + (size_t)b * Q8_BLOCK;
        float amax = 0.0f;
        for (int j = 0; j < QK; ++j) amax = fmaxf(amax, fabsf(xs[j]));
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = rvo_f32_to_f16(d);
        blk[0] = (uint8_t)(dh & 0xff);
        blk[1] = (uint8_t)(dh >> 8);
        for (int j = 0; j < QK; ++j) {
            float v = roundf(xs[j] * id);
            /* Rust `as i8` saturates (and maps NaN to 0) */
            int q = v != v ? 0 : (v > 127.0f ? 127 : (v < -128.0f ? -128 : (int)v));
            blk[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

/* f32 exp and tanh as Rust's f32::exp / f32::tanh reach them: the platform libm. The checker
 * takes the correctly rounded f32 result (the double-precision function rounded once), which
 * is what glibc >= 2.41 returns for tanhf (CORE-MATH) and what glibc's expf returns except
 * within its documented 0.502-ulp error, so parity does not depend on the host's glibc. */
float rvo_expf(float x) { return (float)exp((double)x); }
float rvo_tanhf(float x) { return (float)tanh((double)x); }

/* tanh-approximation GELU, evaluated left to right as ops.rs:145-149. */
float rvo_gelu(float x) {
    const float A = 0.044715f;
    const float S = 0.7978846f; /* 0.797_884_6 */
    float inner = (S * x) * (1.0f + (A * x) * x);
    return (0.5f * x) * (1.0f + rvo_tanhf(inner));
}

/* ops.rs:131-139 row by row, with rvhip.hip:84-88's post factor between scale and weight. */
void rvo_rms_norm(const float *x, float *out, const float *weight, int rows, int width, float eps, float post) {
    for (int r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * width;
        float *o = out + (size_t)r * width;
        double sum = 0.0;
        for (int i = 0; i < width; ++i) sum += (double)xr[i] * (double)xr[i];
        const float mean = (float)(sum / (double)width);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int i = 0; i < width; ++i) {
            float v = xr[i] * scale;
            if (post != 1.0f) v = v * post;
            if (weight) v = v * weight[i];
            o[i] = v;
        }
    }
}

/* ops.rs:83-92 (dequant_q4_0) then ops.rs:249-266 (matmul_q4_0): each row dequantised to f32,
 * (q - 8) * d, and each (token, row) dot the sequential sum of the rounded products, starting
 * from -0 as Rust's f32 sum does. */
void rvo_matmul_q4_0(const uint8_t *w, int k, const float *x, int n_in, float *y, int n_out) {
    const int nb = k / 32;
    float *row = (float *)malloc(sizeof(float) * (size_t)k);
    if (!row) return;
    for (int r = 0; r < n_out; ++r) {
        const uint8_t *wr = w + (size_t)r * nb * 18;
        for (int b = 0; b < nb; ++b) {
            const float d = ld_f16(wr + 18 * b);
            for (int j = 0; j < 16; ++j) {
                const uint8_t q = wr[18 * b + 2 + j];
                row[32 * b + j] = (float)((int)(q & 15) - 8) * d;
                row[32 * b + j + 16] = (float)((int)(q >> 4) - 8) * d;
            }
        }
        for (int t = 0; t < n_in; ++t) {
            const float *xt = x + (size_t)t * k;
            float s = -0.0f;
            for (int i = 0; i < k; ++i) {
                const float p = row[i] * xt[i];
                s = s + p;
            }
            y[(size_t)t * n_out + r] = s;
        }
    }
    free(row);
}

/* The shared dense MLP of exec.rs:438-453: cur = rms_norm(x) * ffn_norm; gate, up =
 * matmul_q4_0(cur); mlp = gelu(gate) * up; out = rms_norm(matmul_q4_0(down, mlp)) * post_norm. */
void rvo_shared_mlp(const uint8_t *gate, const uint8_t *up, const uint8_t *down, const float *ffn_norm,
                    const float *post_norm, const float *x, int n_tok, int n_embd, int ff, float eps, float *out) {
    float *cur = (float *)malloc(sizeof(float) * (size_t)n_tok * n_embd);
    float *g = (float *)malloc(sizeof(float) * (size_t)n_tok * ff);
    float *u = (float *)malloc(sizeof(float) * (size_t)n_tok * ff);
    if (cur && g && u) {
        rvo_rms_norm(x, cur, ffn_norm, n_tok, n_embd, eps, 1.0f);
        rvo_matmul_q4_0(gate, n_embd, cur, n_tok, g, ff);
        rvo_matmul_q4_0(up, n_embd, cur, n_tok, u, ff);
        for (size_t i = 0; i < (size_t)n_tok * ff; ++i) g[i] = rvo_gelu(g[i]) * u[i];
        rvo_matmul_q4_0(down, ff, g, n_tok, out, n_embd);
        rvo_rms_norm(out, out, post_norm, n_tok, n_embd, eps, 1.0f);
    }
    free(cur);
    free(g);
    free(u);
}

/* Softmax with f32 exp and an f64 sum, scaled by (1/sum) rounded to f32 (ops.rs:170-179). */
void rvo_softmax(float *x, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) mx = fmaxf(mx, x[i]); /* f32::max ignores NaN like fmaxf */
    double sum = 0.0;
    for (int i = 0; i < n; ++i) {
        x[i] = rvo_expf(x[i] - mx);
        sum += (double)x[i];
    }
    float inv = (float)(1.0 / sum);
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* IEEE totalOrder key (Rust f32::total_cmp): flip the magnitude bits of negatives. */
static inline int32_t total_key(float f) {
    int32_t b;
    memcpy(&b, &f, 4);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return b;
}

/* Top k by value descending, ties to the lower index (ops.rs:182-187). O(n k) selection,
 * identical to the stable sort for the first k. */
void rvo_top_k(const float *x, int n, int k, int32_t *idx) {
    for (int s = 0; s < k; ++s) {
        int best = -1;
        int32_t bk = 0;
        for (int i = 0; i < n; ++i) {
            int taken = 0;
            for (int q = 0; q < s; ++q) taken |= idx[q] == i;
            if (taken) continue;
            int32_t key = total_key(x[i]);
            if (best < 0 || key > bk) { /* strict: equal keys keep the lower index */
                best = i;
                bk = key;
            }
        }
        idx[s] = best;
    }
}

/* Router logits: sequential f32 dot per expert row, as matvec_f32 (ops.rs:321-326), which
 * Rust's f32 Sum folds from -0.0; then an optional additive bias. */
void rvo_router_logits(const void *x, int x_dtype, const void *w, int w_dtype, const float *bias, int bias_stride,
                       int n_tok, int n_embd, int n_experts, float *logits) {
    for (int t = 0; t < n_tok; ++t) {
        for (int e = 0; e < n_experts; ++e) {
            float s = -0.0f;
            for (int k = 0; k < n_embd; ++k) {
                float wv = ld_act(w, w_dtype, (size_t)e * n_embd + k);
                float xv = ld_act(x, x_dtype, (size_t)t * n_embd + k);
                float p = wv * xv;
                s = s + p;
            }
            if (bias) s = s + bias[(size_t)t * bias_stride + e];
            logits[(size_t)t * n_experts + e] = s;
        }
    }
}

#define ROUTER_SUM_MIN (1.0f / 16384.0f) /* exec.rs:124-125 */

/* Selection and renormalisation (exec.rs:507-517). */
void rvo_select_experts(float *logits, int n_tok, int n_experts, int used, int32_t *ids, float *weights) {
    for (int t = 0; t < n_tok; ++t) {
        float *lg = logits + (size_t)t * n_experts;
        rvo_softmax(lg, n_experts);
        int32_t *top = ids + (size_t)t * used;
        rvo_top_k(lg, n_experts, used, top);
        float sum = -0.0f;
        for (int j = 0; j < used; ++j) sum = sum + lg[top[j]];
        sum = fmaxf(sum, ROUTER_SUM_MIN);
        for (int j = 0; j < used; ++j) weights[(size_t)t * used + j] = lg[top[j]] / sum;
    }
}

/* ----------------------------------------------------------- Q4 x Q8 dots */

int32_t rvo_block_sumi(const uint8_t *w, const uint8_t *x) {
    int32_t sumi = 0;
    for (int j = 0; j < 16; ++j) {
        uint8_t b = w[2 + j];
        sumi += ((int32_t)(b & 15) - 8) * (int32_t)(int8_t)x[2 + j];
        sumi += ((int32_t)(b >> 4) - 8) * (int32_t)(int8_t)x[18 + j];
    }
    return sumi;
}

/* Generic order of ggml_vec_dot_q4_0_q8_0: exact block integer sum, then one f32
 * multiply-add per block, acc += sumi * (dw * dx) (expert_kernel.rs:147-161). */
float rvo_dot_q8_scalar(const uint8_t *row, const uint8_t *xq, int k) {
    float acc = 0.0f;
    for (int b = 0; b < k / QK; ++b) {
        const uint8_t *w = row + (size_t)b * Q4_BLOCK;
        const uint8_t *x = xq + (size_t)b * Q8_BLOCK;
        float dw = ld_f16(w), dx = ld_f16(x);
        int32_t sumi = rvo_block_sumi(w, x);
        acc = acc + (float)sumi * (dw * dx);
    }
    return acc;
}

int rvo_have_avx2(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

#if defined(__x86_64__)
/* AVX2 int8 routine (expert_kernel.rs:163-191): nibbles widened to bytes, |qw| x sign-adjusted
 * qx with maddubs, pairs summed with madd, and one fmadd of the block scale into 8 f32 lanes;
 * the 8 lanes are summed in order at the end (Rust f32 Sum, folded from -0.0). */
__attribute__((target("avx2,fma"))) float rvo_dot_q8_avx2(const uint8_t *row, const uint8_t *xq, int k) {
    __m256 acc = _mm256_setzero_ps();
    const __m256i low = _mm256_set1_epi8(15);
    const __m256i bias = _mm256_set1_epi8(8);
    const __m256i ones = _mm256_set1_epi16(1);
    for (int b = 0; b < k / QK; ++b) {
        const uint8_t *w = row + (size_t)b * Q4_BLOCK;
        const uint8_t *x = xq + (size_t)b * Q8_BLOCK;
        float d = ld_f16(w) * ld_f16(x);
        __m128i packed = _mm_loadu_si128((const __m128i *)(w + 2));
        __m256i both = _mm256_set_m128i(_mm_srli_epi16(packed, 4), packed);
        __m256i qw = _mm256_sub_epi8(_mm256_and_si256(both, low), bias);
        __m256i qx = _mm256_loadu_si256((const __m256i *)(x + 2));
        __m256i prod = _mm256_maddubs_epi16(_mm256_sign_epi8(qw, qw), _mm256_sign_epi8(qx, qw));
        __m256i sumi = _mm256_madd_epi16(prod, ones);
        acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
    }
    float lanes[8];
    _mm256_storeu_ps(lanes, acc);
    float s = -0.0f;
    for (int i = 0; i < 8; ++i) s = s + lanes[i];
    return s;
}
#else
float rvo_dot_q8_avx2(const uint8_t *row, const uint8_t *xq, int k) { return rvo_dot_q8_scalar(row, xq, k); }
#endif

/* ------------------------------------------------------------------ plan */

/* Stable sort of pair indices by (expert, pair): a counting sort keeps pair order within an
 * expert, which is the same permutation as sort_by_key((expert, i)) (exec.rs:541-557). */
void rvo_moe_plan(const int32_t *ids, int n_pairs, int n_experts, int32_t *order, int32_t *pos_of, int32_t *counts) {
    for (int e = 0; e < n_experts; ++e) counts[e] = 0;
    for (int p = 0; p < n_pairs; ++p) counts[ids[p]]++;
    int32_t *start = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_experts);
    int32_t acc = 0;
    for (int e = 0; e < n_experts; ++e) {
        start[e] = acc;
        acc += counts[e];
    }
    for (int p = 0; p < n_pairs; ++p) {
        int32_t k = start[ids[p]]++;
        order[k] = p;
        pos_of[p] = k;
    }
    free(start);
}

/* ------------------------------------------------------------------ pool */

typedef struct {
    const uint8_t *w; /* n_out Q4_0 rows of k */
    const uint8_t *xq; /* n_in Q8_0 rows of k */
    int n_out, n_in;
    size_t y_off;
} seg_t;

typedef struct {
    const seg_t *segs;
    const int64_t *starts; /* n_segs + 1 */
    int n_segs;
    int k;
    int64_t total;
    float *y;
    atomic_llong next;
} job_t;

struct rvo_pool {
    pthread_t *threads;
    int n_threads;
    int kernel;
    pthread_mutex_t mu;
    pthread_cond_t wake, done;
    uint64_t generation;
    int remaining;
    int stop;
    job_t *job;
};

static float pool_dot(int kernel, const uint8_t *w, const uint8_t *xq, int k) {
    return kernel == RVO_KERNEL_AVX2 ? rvo_dot_q8_avx2(w, xq, k) : rvo_dot_q8_scalar(w, xq, k);
}

/* Job::execute (expert_pool.rs:86-135): grab 16 global rows at a time, every input of the row. */
static void job_execute(job_t *j, int kernel) {
    const size_t row_bytes = (size_t)j->k / QK * Q4_BLOCK;
    const size_t q_bytes = (size_t)j->k / QK * Q8_BLOCK;
    for (;;) {
        int64_t a = atomic_fetch_add_explicit(&j->next, 16, memory_order_relaxed);
        if (a >= j->total) break;
        int64_t b = a + 16 < j->total ? a + 16 : j->total;
        int si = 0;
        while (j->starts[si + 1] <= a) ++si;
        for (int64_t g = a; g < b; ++g) {
            while (g >= j->starts[si + 1]) ++si;
            const seg_t *s = &j->segs[si];
            int64_t r = g - j->starts[si];
            const uint8_t *w = s->w + (size_t)r * row_bytes;
            for (int t = 0; t < s->n_in; ++t)
                j->y[s->y_off + (size_t)t * s->n_out + (size_t)r] = pool_dot(kernel, w, s->xq + (size_t)t * q_bytes, j->k);
        }
    }
}

static void *worker_main(void *arg) {
    rvo_pool *p = (rvo_pool *)arg;
    uint64_t seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        while (!p->stop && p->generation == seen) pthread_cond_wait(&p->wake, &p->mu);
        if (p->stop) {
            pthread_mutex_unlock(&p->mu);
            return NULL;
        }
        seen = p->generation;
        job_t *j = p->job;
        pthread_mutex_unlock(&p->mu);
        job_execute(j, p->kernel);
        pthread_mutex_lock(&p->mu);
        if (--p->remaining == 0) pthread_cond_broadcast(&p->done);
        pthread_mutex_unlock(&p->mu);
    }
}

rvo_pool *rvo_pool_new(int threads, int kernel) {
    if (threads < 1 || threads > 1024) return NULL;
    rvo_pool *p = (rvo_pool *)calloc(1, sizeof(rvo_pool));
    if (!p) return NULL;
    if (kernel == RVO_KERNEL_BEST) kernel = rvo_have_avx2() ? RVO_KERNEL_AVX2 : RVO_KERNEL_SCALAR;
    if (kernel == RVO_KERNEL_AVX2 && !rvo_have_avx2()) kernel = RVO_KERNEL_SCALAR;
    p->kernel = kernel;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->wake, NULL);
    pthread_cond_init(&p->done, NULL);
    p->threads = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    for (int i = 0; i < threads; ++i) {
        if (pthread_create(&p->threads[i], NULL, worker_main, p) != 0) {
            p->n_threads = i;
            rvo_pool_free(p);
            return NULL;
        }
        p->n_threads = i + 1;
    }
    return p;
}

void rvo_pool_free(rvo_pool *p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->stop = 1;
    pthread_cond_broadcast(&p->wake);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->n_threads; ++i) pthread_join(p->threads[i], NULL);
    free(p->threads);
    pthread_mutex_destroy(&p->mu);
    pthread_cond_destroy(&p->wake);
    pthread_cond_destroy(&p->done);
    free(p);
}

int rvo_pool_threads(const rvo_pool *p) { return p ? p->n_threads : 0; }

/* WorkerPool::matmul + submit (expert_pool.rs:282-392), with the activation rows already
 * quantised by the caller thread. */
static void pool_matmul(rvo_pool *p, const seg_t *segs, int n_segs, int k, float *y) {
    int64_t *starts = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_segs + 1));
    int64_t total = 0;
    for (int i = 0; i < n_segs; ++i) {
        starts[i] = total;
        total += segs[i].n_out;
    }
    starts[n_segs] = total;
    if (total > 0) {
        job_t j = {segs, starts, n_segs, k, total, y, 0};
        atomic_init(&j.next, 0);
        pthread_mutex_lock(&p->mu);
        p->job = &j;
        p->remaining = p->n_threads;
        p->generation++;
        pthread_cond_broadcast(&p->wake);
        while (p->remaining > 0) pthread_cond_wait(&p->done, &p->mu);
        p->job = NULL;
        pthread_mutex_unlock(&p->mu);
    }
    free(starts);
}

/* ---------------------------------------------------------------- experts */

int rvo_experts_q8(rvo_pool *pool, const void *x_expert, int x_dtype, const uint8_t *gate_up, const uint8_t *down,
                   const float *down_scale, const int32_t *ids, const float *weights, int n_tok, int n_embd, int ff,
                   int n_experts, int used, float *out, float *h_dbg, float *y_dbg) {
    if (!pool || n_tok < 0 || n_embd <= 0 || n_embd % QK || ff <= 0 || ff % QK || used <= 0 || n_experts <= 0)
        return -1;
    if (n_tok == 0) return 0;
    const int pairs = n_tok * used;
    for (int p = 0; p < pairs; ++p)
        if (ids[p] < 0 || ids[p] >= n_experts) return -1;
    const int gu_rows = 2 * ff;
    const size_t gu_bytes = (size_t)gu_rows * (n_embd / QK) * Q4_BLOCK;
    const size_t dn_bytes = (size_t)n_embd * (ff / QK) * Q4_BLOCK;
    const size_t qx_row = (size_t)n_embd / QK * Q8_BLOCK;
    const size_t qh_row = (size_t)ff / QK * Q8_BLOCK;

    int32_t *order = (int32_t *)malloc(sizeof(int32_t) * pairs);
    int32_t *pos_of = (int32_t *)malloc(sizeof(int32_t) * pairs);
    int32_t *counts = (int32_t *)malloc(sizeof(int32_t) * n_experts);
    float *xrow = (float *)malloc(sizeof(float) * n_embd);
    uint8_t *qx = (uint8_t *)malloc(qx_row * pairs);
    float *gu = (float *)malloc(sizeof(float) * (size_t)pairs * gu_rows);
    float *h = (float *)malloc(sizeof(float) * (size_t)pairs * ff);
    uint8_t *qh = (uint8_t *)malloc(qh_row * pairs);
    float *y = (float *)malloc(sizeof(float) * (size_t)pairs * n_embd);
    seg_t *segs = (seg_t *)malloc(sizeof(seg_t) * n_experts);
    if (!order || !pos_of || !counts || !xrow || !qx || !gu || !h || !qh || !y || !segs) {
        free(order), free(pos_of), free(counts), free(xrow), free(qx), free(gu), free(h), free(qh), free(y), free(segs);
        return -1;
    }
    rvo_moe_plan(ids, pairs, n_experts, order, pos_of, counts);

    /* Copy each pair's input into plan order (exec.rs:585-588) and quantise it on the caller
     * thread, once per row (expert_pool.rs:311-320). */
    for (int k = 0; k < pairs; ++k) {
        int t = order[k] / used;
        for (int i = 0; i < n_embd; ++i) xrow[i] = ld_act(x_expert, x_dtype, (size_t)t * n_embd + i);
        rvo_quantize_q8_0(xrow, n_embd, qx + (size_t)k * qx_row);
    }
    int ns = 0, st = 0;
    for (int e = 0; e < n_experts; ++e) {
        if (!counts[e]) continue;
        segs[ns].w = gate_up + (size_t)e * gu_bytes;
        segs[ns].xq = qx + (size_t)st * qx_row;
        segs[ns].n_out = gu_rows;
        segs[ns].n_in = counts[e];
        segs[ns].y_off = (size_t)st * gu_rows;
        ++ns;
        st += counts[e];
    }
    pool_matmul(pool, segs, ns, n_embd, gu);

    /* GELU-tanh(gate) * up on the caller (exec.rs:606-611). */
    for (int k = 0; k < pairs; ++k)
        for (int j = 0; j < ff; ++j)
            h[(size_t)k * ff + j] = rvo_gelu(gu[(size_t)k * gu_rows + j]) * gu[(size_t)k * gu_rows + ff + j];
    for (int k = 0; k < pairs; ++k) rvo_quantize_q8_0(h + (size_t)k * ff, ff, qh + (size_t)k * qh_row);

    ns = 0, st = 0;
    for (int e = 0; e < n_experts; ++e) {
        if (!counts[e]) continue;
        segs[ns].w = down + (size_t)e * dn_bytes;
        segs[ns].xq = qh + (size_t)st * qh_row;
        segs[ns].n_out = n_embd;
        segs[ns].n_in = counts[e];
        segs[ns].y_off = (size_t)st * n_embd;
        ++ns;
        st += counts[e];
    }
    pool_matmul(pool, segs, ns, ff, y);

    /* Slot-order combine: first term assigned, then +=, each (y * ds) * w (exec.rs:626-638). */
    for (int t = 0; t < n_tok; ++t) {
        float *o = out + (size_t)t * n_embd;
        for (int j = 0; j < used; ++j) {
            int p = t * used + j;
            int ex = ids[p];
            float wt = weights[p];
            float ds = down_scale ? down_scale[ex] : 1.0f;
            const float *yr = y + (size_t)pos_of[p] * n_embd;
            if (j == 0)
                for (int i = 0; i < n_embd; ++i) o[i] = yr[i] * ds * wt;
            else
                for (int i = 0; i < n_embd; ++i) o[i] = o[i] + yr[i] * ds * wt;
        }
    }
    if (h_dbg) memcpy(h_dbg, h, sizeof(float) * (size_t)pairs * ff);
    if (y_dbg) memcpy(y_dbg, y, sizeof(float) * (size_t)pairs * n_embd);
    free(order), free(pos_of), free(counts), free(xrow), free(qx), free(gu), free(h), free(qh), free(y), free(segs);
    return 0;
}

int rvo_moe_layer(rvo_pool *pool, const void *x_router, const void *x_expert, int x_dtype, const void *w_router,
                  int w_dtype, const float *bias, int bias_stride, const uint8_t *gate_up, const uint8_t *down,
                  const float *down_scale, int n_tok, int n_embd, int ff, int n_experts, int used, float *logits_out,
                  int32_t *ids_out, float *w_out, float *out) {
    if (n_tok < 0 || used > n_experts) return -1;
    if (n_tok == 0) return 0;
    float *lg = (float *)malloc(sizeof(float) * (size_t)n_tok * n_experts);
    int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_tok * used);
    float *wt = (float *)malloc(sizeof(float) * (size_t)n_tok * used);
    if (!lg || !ids || !wt) {
        free(lg), free(ids), free(wt);
        return -1;
    }
    rvo_router_logits(x_router, x_dtype, w_router, w_dtype, bias, bias_stride, n_tok, n_embd, n_experts, lg);
    if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)n_tok * n_experts);
    rvo_select_experts(lg, n_tok, n_experts, used, ids, wt);
    int rc = rvo_experts_q8(pool, x_expert, x_dtype, gate_up, down, down_scale, ids, wt, n_tok, n_embd, ff, n_experts,
                            used, out, NULL, NULL);
    if (ids_out) memcpy(ids_out, ids, sizeof(int32_t) * (size_t)n_tok * used);
    if (w_out) memcpy(w_out, wt, sizeof(float) * (size_t)n_tok * used);
    free(lg), free(ids), free(wt);
    return rc;
}
