// router.cuh - fused MoE router for sm_100a.
//
// Replaces the reference's router chain: rvh_f32_mm (runtime/hip/rvhip.hip:170-180, called at
// runtime/src/hip_exec.rs:787), the blocking logits download (:789), and the host-side
// select_experts / MoePlan (runtime/src/exec.rs:507-558).
//
// Parity: the logits are computed in the reference's exact order (matvec_f32,
// runtime/src/ops.rs:321-326: a sequential f32 sum of separately rounded products, folded
// from -0.0), so they are bit-identical. Softmax follows ops.rs:170-179 (f32 exp of
// (l - max), f64 sum, f32 scale by (1/sum)); top-8 follows ops.rs:182-187 (descending,
// ties to the lower index, IEEE total order); renormalisation follows exec.rs:507-517.
#pragma once
#include "common.cuh"

namespace rvc {

enum { DT_F32 = 0, DT_BF16 = 1 };

template <typename T>
__device__ __forceinline__ float ld_val(const T *p, size_t i);
template <>
__device__ __forceinline__ float ld_val<float>(const float *p, size_t i) { return __ldg(p + i); }
template <>
__device__ __forceinline__ float ld_val<uint16_t>(const uint16_t *p, size_t i) {
    return bf16_bits_to_f32(__ldg(p + i));
}

// Load 8 consecutive values starting at element i (i multiple of 8, row 16-byte aligned).
template <typename T>
__device__ __forceinline__ void ld8(const T *p, size_t i, float v[8]);
template <>
__device__ __forceinline__ void ld8<float>(const float *p, size_t i, float v[8]) {
    float4 a = __ldg(reinterpret_cast<const float4 *>(p + i));
    float4 b = __ldg(reinterpret_cast<const float4 *>(p + i + 4));
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <>
__device__ __forceinline__ void ld8<uint16_t>(const uint16_t *p, size_t i, float v[8]) {
    uint4 a = __ldg(reinterpret_cast<const uint4 *>(p + i));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
}

// ---------------------------------------------------------------- exact logits
// One thread per expert row, TOK tokens per CTA. Each (token, expert) logit is one
// sequential chain s = (s + w*x) with separately rounded multiply and add; the TOK
// independent chains per thread give instruction-level parallelism.
template <int TOK, typename XT, typename WT>
__global__ void __launch_bounds__(128) k_router_logits_exact(const XT *__restrict__ x, const WT *__restrict__ w,
                                                             const float *__restrict__ bias, int bias_stride,
                                                             int n_tok, int n_experts, int n_embd,
                                                             float *__restrict__ logits) {
    const int e = blockIdx.y * blockDim.x + threadIdx.x;
    const int t0 = blockIdx.x * TOK;
    if (e >= n_experts) return;
    float s[TOK];
#pragma unroll
    for (int i = 0; i < TOK; ++i) s[i] = -0.0f;
    const int nt = min(TOK, n_tok - t0);
    const WT *wr = w + (size_t)e * n_embd;
    for (int k = 0; k < n_embd; k += 8) {
        float wv[8];
        ld8<WT>(wr, k, wv);
        float xv[TOK][8];
#pragma unroll
        for (int i = 0; i < TOK; ++i) {
            if (i < nt) ld8<XT>(x + (size_t)(t0 + i) * n_embd, k, xv[i]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int i = 0; i < TOK; ++i) s[i] = __fadd_rn(s[i], __fmul_rn(wv[j], xv[i][j]));
        }
    }
#pragma unroll
    for (int i = 0; i < TOK; ++i) {
        if (i < nt) {
            float v = s[i];
            if (bias) v = __fadd_rn(v, __ldg(bias + (size_t)(t0 + i) * bias_stride + e));
            logits[(size_t)(t0 + i) * n_experts + e] = v;
        }
    }
}

// IEEE totalOrder key (as f32::total_cmp): larger key = larger value.
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

constexpr float ROUTER_SUM_MIN = 1.0f / 16384.0f;  // exec.rs:124-125
constexpr int MAX_EXPERTS = 256;
constexpr int MAX_USED = 16;

// ----------------------------------------------------------- select + quantise
// One warp per token: softmax over n_experts (<= 256) logits, top `used`, renormalised
// weights; then Q8_0 quantisation of the token's expert input (n_embd/32 blocks).
// Q8 planes: xq[t][nb][32] int8, xd[t][nb] f32 (the f16 scale widened), xs[t][nb] sum of q.
template <typename XT>
__global__ void __launch_bounds__(256) k_select_quant(const float *__restrict__ logits, const XT *__restrict__ x_expert,
                                                      int n_tok, int n_experts, int used, int n_embd,
                                                      int32_t *__restrict__ ids, float *__restrict__ wts,
                                                      float *__restrict__ probs_out, int8_t *__restrict__ xq,
                                                      float *__restrict__ xd, int32_t *__restrict__ xs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= n_tok) return;
    constexpr int PER = MAX_EXPERTS / 32;
    const float *lg = logits + (size_t)t * n_experts;
    float v[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < n_experts ? lg[e] : -INFINITY;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (e < n_experts) {
            v[i] = (float)exp((double)__fsub_rn(v[i], mx));
            sum += (double)v[i];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = __double2float_rn(1.0 / sum);
    int32_t key[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        v[i] = __fmul_rn(v[i], inv);
        key[i] = e < n_experts ? total_key(v[i]) : INT32_MIN;
        if (probs_out && e < n_experts) probs_out[(size_t)t * n_experts + e] = v[i];
    }
    // top-`used`: repeated warp argmax over (key desc, index asc)
    float sel_p = 0.0f;
    int sel_e = 0;
    float psum = -0.0f;
    float ptop[MAX_USED];
    int etop[MAX_USED];
    for (int j = 0; j < used; ++j) {
        int32_t bk = INT32_MIN;
        int be = 0x7fffffff;
        float bp = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = lane + 32 * i;
            if (e < n_experts && (key[i] > bk || (key[i] == bk && e < be))) bk = key[i], be = e, bp = v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            int32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
            int oe = __shfl_xor_sync(0xffffffffu, be, o);
            float op = __shfl_xor_sync(0xffffffffu, bp, o);
            if (ok > bk || (ok == bk && oe < be)) bk = ok, be = oe, bp = op;
        }
        // remove the winner
#pragma unroll
        for (int i = 0; i < PER; ++i)
            if (lane + 32 * i == be) key[i] = INT32_MIN, v[i] = -INFINITY;
        if (j < MAX_USED) ptop[j] = bp, etop[j] = be;
        psum = __fadd_rn(psum, bp);  // f32 sum in top order (exec.rs:512)
        (void)sel_p, (void)sel_e;
    }
    psum = fmaxf(psum, ROUTER_SUM_MIN);
    if (lane < used) {
        float p = 0.0f;
        int e = 0;
#pragma unroll
        for (int j = 0; j < MAX_USED; ++j)
            if (j == lane) p = ptop[j], e = etop[j];
        ids[(size_t)t * used + lane] = e;
        wts[(size_t)t * used + lane] = __fdiv_rn(p, psum);
    }
    // Q8_0 of the expert input (ops.rs:95-105), one block of 32 per warp iteration.
    if (xq) {
        const int nb = n_embd / QK;
        const XT *xr = x_expert + (size_t)t * n_embd;
        for (int b = 0; b < nb; ++b) {
            float val = ld_val<XT>(xr, (size_t)b * QK + lane);
            uint16_t dbits;
            int qsum;
            int8_t q = quant_q8_lane(val, &dbits, &qsum);
            xq[((size_t)t * nb + b) * QK + lane] = q;
            if (lane == 0) {
                xd[(size_t)t * nb + b] = f16_bits_to_f32(dbits);
                xs[(size_t)t * nb + b] = qsum;
            }
        }
    }
}

// ------------------------------------------------------------------- plan
// Stable grouping of the (token, slot) pairs by expert (exec.rs:541-557): order[] is the
// permutation sort_by_key((expert, pair)), pos_of[order[k]] = k, counts/offsets per
// expert, and the ascending list of experts with at least one pair. Single CTA of 1024
// threads; pairs are ranked chunk by chunk with warp match masks.
constexpr int PLAN_THREADS = 1024;

__global__ void __launch_bounds__(PLAN_THREADS) k_plan(const int32_t *__restrict__ ids, int n_pairs, int n_experts,
                                                       int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
                                                       int32_t *__restrict__ order, int32_t *__restrict__ pos_of,
                                                       int32_t *__restrict__ active, int32_t *__restrict__ n_active,
                                                       int *status) {
    __shared__ int s_count[MAX_EXPERTS];
    __shared__ int s_base[MAX_EXPERTS];
    __shared__ int s_warp[32][MAX_EXPERTS];  // per-warp counts within a chunk
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < MAX_EXPERTS; e += PLAN_THREADS) s_count[e] = 0;
    __syncthreads();
    for (int p = tid; p < n_pairs; p += PLAN_THREADS) {
        int e = ids[p];
        if (e < 0 || e >= n_experts) {
            set_status(status, STATUS_BAD_INDEX);
            continue;
        }
        atomicAdd(&s_count[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scan over experts (n_experts <= 256: 8 per lane)
        int local[MAX_EXPERTS / 32];
        int run = 0;
#pragma unroll
        for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
            int e = lane * (MAX_EXPERTS / 32) + i;
            local[i] = run;
            run += e < n_experts ? s_count[e] : 0;
        }
        int incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int excl = incl - run;
#pragma unroll
        for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
            int e = lane * (MAX_EXPERTS / 32) + i;
            if (e < n_experts) {
                s_base[e] = excl + local[i];
                offsets[e] = excl + local[i];
                counts[e] = s_count[e];
            }
        }
        if (lane == 31) offsets[n_experts] = incl;
        // active expert list, ascending
        int flags = 0;
#pragma unroll
        for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
            int e = lane * (MAX_EXPERTS / 32) + i;
            flags += (e < n_experts && s_count[e] > 0);
        }
        int fin = flags;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, fin, o);
            if (lane >= o) fin += y;
        }
        int slot = fin - flags;
#pragma unroll
        for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
            int e = lane * (MAX_EXPERTS / 32) + i;
            if (e < n_experts && s_count[e] > 0) active[slot++] = e;
        }
        if (lane == 31) *n_active = fin;
    }
    __syncthreads();
    // stable scatter, one chunk of PLAN_THREADS pairs at a time
    for (int c0 = 0; c0 < n_pairs; c0 += PLAN_THREADS) {
        const int p = c0 + tid;
        const int nw = (min(PLAN_THREADS, n_pairs - c0) + 31) >> 5;
        int e = -1, rank = 0;
        if (p < n_pairs) {
            e = ids[p];
            if (e < 0 || e >= n_experts) e = -1;
        }
        if (warp < nw) {
            for (int i = lane; i < n_experts; i += 32) s_warp[warp][i] = 0;
        }
        __syncthreads();
        if (warp < nw) {
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            rank = __popc(peers & ((1u << lane) - 1));
            if (e >= 0 && rank == 0) s_warp[warp][e] = __popc(peers);
        }
        __syncthreads();
        // per expert, exclusive scan over the chunk's warps
        for (int x = tid; x < n_experts; x += PLAN_THREADS) {
            int run = s_base[x];
            for (int w = 0; w < nw; ++w) {
                int c = s_warp[w][x];
                s_warp[w][x] = run;
                run += c;
            }
            s_base[x] = run;
        }
        __syncthreads();
        if (e >= 0) {
            const int k = s_warp[warp][e] + rank;
            order[k] = p;
            pos_of[p] = k;
        }
        __syncthreads();
    }
}

}  // namespace rvc
