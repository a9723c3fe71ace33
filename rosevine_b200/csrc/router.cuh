// router.cuh - fused MoE router for sm_100a.
//
// Replaces the reference's router chain: rvh_f32_mm (runtime/hip/rvhip.hip:170-180, called at
// runtime/src/hip_exec.rs:787), the blocking logits download (:789), and the host-side
// select_experts / MoePlan (runtime/src/exec.rs:507-558).
//
// Parity: logits are computed in the reference's exact order by router_fast.cuh (matvec_f32,
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

// IEEE totalOrder key (as f32::total_cmp): larger key = larger value.
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

constexpr float ROUTER_SUM_MIN = 1.0f / 16384.0f;  // exec.rs:124-125
constexpr int MAX_EXPERTS = 256;
constexpr int MAX_USED = 16;

// ------------------------------------------------------------- selection
// One warp: softmax over n_experts (<= 256) logits, top `used`, renormalised weights, for
// one token (ops.rs:170-187, exec.rs:507-517). Logits are read with ld.global.cg so a CTA may
// select on logits other CTAs wrote before a release/acquire handoff. ids/wts get `used`
// entries in slot order; probs (may be NULL) all n_experts probabilities.
__device__ __forceinline__ void warp_select(const float *lg, int n_experts, int used, int32_t *ids, float *wts,
                                            float *probs) {
    const int lane = threadIdx.x & 31;
    constexpr int PER = MAX_EXPERTS / 32;
    float v[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < n_experts ? __ldcg(lg + e) : -INFINITY;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (e < n_experts) {
            v[i] = fd_exp_f32(__fsub_rn(v[i], mx));
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
        if (probs && e < n_experts) probs[e] = v[i];
    }
    // top-`used`: repeated warp argmax over (key desc, index asc); lane j keeps winner j
    float psum = -0.0f, my_p = 0.0f;
    int my_e = 0;
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
#pragma unroll
        for (int i = 0; i < PER; ++i)
            if (lane + 32 * i == be) key[i] = INT32_MIN;
        if (lane == j) my_p = bp, my_e = be;
        psum = __fadd_rn(psum, bp);  // f32 sum in top order (exec.rs:512)
    }
    psum = fmaxf(psum, ROUTER_SUM_MIN);
    if (lane < used) {
        ids[lane] = my_e;
        wts[lane] = __fdiv_rn(my_p, psum);
    }
}

// ----------------------------------------------------------------- select
// One warp per token: warp_select over the token's logits.
__global__ void __launch_bounds__(256) k_select(const float *__restrict__ logits, int n_tok, int n_experts, int used,
                                                int32_t *__restrict__ ids, float *__restrict__ wts,
                                                float *__restrict__ probs_out) {
    const int warp = threadIdx.x >> 5;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= n_tok) return;
    warp_select(logits + (size_t)t * n_experts, n_experts, used, ids + (size_t)t * used, wts + (size_t)t * used,
                probs_out ? probs_out + (size_t)t * n_experts : nullptr);
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
                                                       int *status, int align = 1, int2 *__restrict__ tiles = nullptr,
                                                       int32_t *__restrict__ n_tiles = nullptr, int tile_rows = 128,
                                                       bool stable = true, bool skip_neg = false) {
    __shared__ int s_count[MAX_EXPERTS];
    __shared__ int s_base[MAX_EXPERTS];
    __shared__ int s_warp[32][MAX_EXPERTS];  // per-warp counts within a chunk
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < MAX_EXPERTS; e += PLAN_THREADS) s_count[e] = 0;
    __syncthreads();
    for (int p = tid; p < n_pairs; p += PLAN_THREADS) {
        int e = ids[p];
        if (e < 0 || e >= n_experts) {
            if (!(skip_neg && e == -1)) set_status(status, STATUS_BAD_INDEX);  // -1: an empty slot
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
            run += e < n_experts ? (s_count[e] + align - 1) / align * align : 0;
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
        if (tiles) {
            // (expert | positions << 8, first position) per tile of up to tile_rows positions
            int nt_l = 0;
#pragma unroll
            for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
                int e = lane * (MAX_EXPERTS / 32) + i;
                nt_l += e < n_experts ? (s_count[e] + tile_rows - 1) / tile_rows : 0;
            }
            int tinc = nt_l;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int y = __shfl_up_sync(0xffffffffu, tinc, o);
                if (lane >= o) tinc += y;
            }
            int k = tinc - nt_l;
            for (int i = 0; i < MAX_EXPERTS / 32; ++i) {
                int e = lane * (MAX_EXPERTS / 32) + i;
                if (e >= n_experts) break;
                for (int c = 0; c < s_count[e]; c += tile_rows)
                    tiles[k++] = make_int2(e | (min(tile_rows, s_count[e] - c) << 8), s_base[e] + c);
            }
            if (lane == 31) *n_tiles = tinc;
        }
    }
    __syncthreads();
    if (!stable) {
        // positions within a group in arrival order (callers whose results do not depend on
        // the order inside a group): one shared-memory atomic per pair
        for (int p = tid; p < n_pairs; p += PLAN_THREADS) {
            const int e = ids[p];
            if (e < 0 || e >= n_experts) continue;
            const int k = atomicAdd(&s_base[e], 1);
            order[k] = p;
            pos_of[p] = k;
        }
        return;
    }
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
