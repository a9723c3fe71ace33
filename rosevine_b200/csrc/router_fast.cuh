// router_fast.cuh - decode-latency routing: exact-order chains (K0) and a verified fast router (K1).
//
// The reference router is a sequential f32 dot per (token, expert) (matvec_f32,
// runtime/src/ops.rs:321-326), so its logits carry that order's rounding. Two kernels
// reproduce its selection (exec.rs:507-517) without putting a 2816-step dependent chain in
// front of the expert GEMVs:
//
// K0 k_router_chains: the exact chains themselves, one per thread, with whole rows of the
//    router and of x staged into shared memory by a few large 1-D TMA bulk copies. Logits are
//    bit-identical to the reference; the last CTA selects (softmax, top-k, renormalised
//    weights) - these are the weights the combine uses. It runs on a side branch, concurrently
//    with K1 and the gate/up GEMV.
// K1 k_route_fast: every (token, expert) dot in parallel in f64 (the products of bf16/f32
//    operands are exact in f64), plus a rigorous bound on how far the sequential f32 result
//    can be from it: |s_seq - S| <= u * (sum_i |S_i| + sum_i |p_i|) * (1 + 1e-2), S_i the
//    exact prefix sums (Higham, Accuracy and Stability of Numerical Algorithms, 2nd ed.,
//    eq. 4.4 with products rounded once), plus the rounding of the bias add and of the f32
//    store. A token whose top-(used+1) are separated by more than their bounds has the same
//    ids in the reference; any other token gets its logits from exact chains inside K1 (about
//    3% of tokens at the benchmark's distributions). K1 also quantises x to Q8_0 and builds
//    the dispatch plan, so the expert kernels can start as soon as it ends.
#pragma once
#include "common.cuh"
#include "router.cuh"

namespace rvc {

struct PlanOut {
    int32_t *counts, *offsets, *order, *pos_of, *active, *n_active;
};

struct RouteArgs {
    const void *x;
    const void *w;
    const float *bias;
    int bias_stride;
    int n_tok, n_experts, n_embd, used;
    float *lfast, *lbound;  // [n_tok][n_experts] (K1)
    float *lexact;          // [n_tok][n_experts] exact logits (K0; K1 fallback)
    uint8_t *xrec;          // Q8_0 records of x (K1), may be NULL
    unsigned *done_cnt;     // last-CTA counter (zero between launches)
    unsigned *fallback_cnt; // (K1) cumulative count of tokens routed through the exact fallback
    int32_t *ids;           // [n_tok][used]
    float *wts;             // [n_tok][used] (K0)
    PlanOut plan;           // (K1)
    int *status;
};

constexpr int RF_MAX_TOK = 64;  // decode tokens per call

template <typename T>
__device__ __forceinline__ void lds8(const T *p, float v[8]);
template <>
__device__ __forceinline__ void lds8<float>(const float *p, float v[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <>
__device__ __forceinline__ void lds8<uint16_t>(const uint16_t *p, float v[8]) {
    const uint4 a = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
}

// One step of the reference chain s = s + w*x (separately rounded). When both operands are
// bf16 their product has at most 16 significant bits and is exact in f32 (outside the subnormal
// range, far below any router value), so the fused multiply-add rounds once at the same place
// and gives the same bits with one instruction.
template <typename XT, typename WT>
__device__ __forceinline__ float chain_step(float s, float w, float x) {
    if constexpr (sizeof(XT) == 2 && sizeof(WT) == 2)
        return __fmaf_rn(w, x, s);
    else
        return __fadd_rn(s, __fmul_rn(w, x));
}

// ------------------------------------------------------------- block selection
// softmax / top-`used` / renormalisation of one token (ops.rs:170-187, exec.rs:507-517) by a
// whole CTA: each thread owns experts tid, tid + blockDim.x, ...; the order of selection is
// each expert's rank under (probability descending, index ascending), counted in parallel.
struct SelScratch {
    float p[MAX_EXPERTS];
    int32_t key[MAX_EXPERTS];
    int top[MAX_USED];
    float redf[32];
    double redd[32];
};

__device__ __forceinline__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = -INFINITY;
    for (int i = 0; i < nw; ++i) r = fmaxf(r, red[i]);
    return r;
}

__device__ __forceinline__ double block_sum_d(double v, double *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double r = 0.0;
    for (int i = 0; i < nw; ++i) r += red[i];
    return r;
}

// lg may point to global memory written by other CTAs before a release/acquire handoff (read
// with ld.global.cg).
__device__ void block_select(const float *lg, int ne, int used, int32_t *ids, float *wts, SelScratch &sc) {
    const int tid = threadIdx.x, nth = blockDim.x;
    float m = -INFINITY;
    for (int e = tid; e < ne; e += nth) {
        const float v = __ldcg(lg + e);
        sc.p[e] = v;
        m = fmaxf(m, v);
    }
    m = block_max(m, sc.redf);
    double sum = 0.0;
    for (int e = tid; e < ne; e += nth) {
        const float ex = (float)exp((double)__fsub_rn(sc.p[e], m));
        sc.p[e] = ex;
        sum += (double)ex;
    }
    sum = block_sum_d(sum, sc.redd);
    const float inv = __double2float_rn(1.0 / sum);
    for (int e = tid; e < ne; e += nth) {
        const float p = __fmul_rn(sc.p[e], inv);
        sc.p[e] = p;
        sc.key[e] = total_key(p);
    }
    __syncthreads();
    for (int e = tid; e < ne; e += nth) {
        const int32_t k = sc.key[e];
        int rank = 0;
        for (int f = 0; f < ne; ++f) {
            const int32_t kf = sc.key[f];
            rank += (kf > k) | ((kf == k) & (f < e));
        }
        if (rank < used) sc.top[rank] = e;
    }
    __syncthreads();
    if (tid == 0) {
        float psum = -0.0f;  // f32 sum in top order (exec.rs:512)
        for (int j = 0; j < used; ++j) psum = __fadd_rn(psum, sc.p[sc.top[j]]);
        psum = fmaxf(psum, ROUTER_SUM_MIN);
        for (int j = 0; j < used; ++j) {
            ids[j] = sc.top[j];
            if (wts) wts[j] = __fdiv_rn(sc.p[sc.top[j]], psum);
        }
    }
    __syncthreads();
}

// ------------------------------------------------------------------ K0
// A tile of C0_EPC experts x tpc tokens per CTA (one chain per thread). The tile's router rows
// and x rows are staged whole into shared memory by a few large 1-D TMA bulk copies, split in
// C0_CHUNKS column chunks with one mbarrier each so the chains start on the first chunk. Rows
// are padded by 16 B so threads reading 16 B at the same column of consecutive rows hit
// distinct banks. grid (ceil(n_experts / C0_EPC), ceil(n_tok / tpc)), block max(32, 8 * tpc).
constexpr int C0_EPC = 8;
constexpr int C0_CHUNKS = 4;

template <typename T>
__host__ __device__ inline int c0_row_bytes(int n_embd) {
    return n_embd * (int)sizeof(T) + 16;
}

template <typename XT, typename WT>
__global__ void __launch_bounds__(128) k_router_chains(RouteArgs a, int tpc) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[C0_CHUNKS];
    __shared__ int s_last;
    __shared__ SelScratch sc;
    RVC_MARK(0, 0);
    const int e0 = blockIdx.x * C0_EPC, t0 = blockIdx.y * tpc;
    const int nw = min(C0_EPC, a.n_experts - e0), nx = min(tpc, a.n_tok - t0);
    const int tid = threadIdx.x;
    const int n = a.n_embd, ck = n / C0_CHUNKS;
    const int wrow = c0_row_bytes<WT>(n), xrow = c0_row_bytes<XT>(n);
    const WT *w = static_cast<const WT *>(a.w);
    const XT *x = static_cast<const XT *>(a.x);
    if (tid == 0) {
        for (int c = 0; c < C0_CHUNKS; ++c) mbar_init(&bars[c], nw + nx);  // one arrival per row
        fence_barrier_init();
    }
    __syncthreads();
    if (tid < nw + nx) {  // thread r stages row r (router rows first, then x rows), chunk by chunk
        const bool isw = tid < nw;
        const int r = isw ? tid : tid - nw;
        const uint32_t cbytes = (uint32_t)ck * (isw ? sizeof(WT) : sizeof(XT));
        uint8_t *dst = smem + (isw ? r * wrow : C0_EPC * wrow + r * xrow);
        const uint8_t *src = isw ? reinterpret_cast<const uint8_t *>(w + (size_t)(e0 + r) * n)
                                 : reinterpret_cast<const uint8_t *>(x + (size_t)(t0 + r) * n);
        for (int c = 0; c < C0_CHUNKS; ++c) {
            mbar_arrive_expect_tx(&bars[c], cbytes);
            bulk_g2s(dst + c * cbytes, src + (size_t)c * cbytes, cbytes, &bars[c]);
        }
    }
    const int el = tid / tpc, tl = tid % tpc;
    const bool active = tid < C0_EPC * tpc && el < nw && tl < nx;
    float s = -0.0f;
    bool ok = true;
    for (int c = 0; c < C0_CHUNKS; ++c) {
        if (!mbar_wait(&bars[c], 0, a.status)) ok = false;
        if (c == 0) RVC_MARK(0, 1);
        if (active && ok) {
            const WT *wr = reinterpret_cast<const WT *>(smem + el * wrow) + c * ck;
            const XT *xr = reinterpret_cast<const XT *>(smem + C0_EPC * wrow + tl * xrow) + c * ck;
#pragma unroll 4
            for (int k = 0; k < ck; k += 8) {
                float wv[8], xv[8];
                lds8<WT>(wr + k, wv);
                lds8<XT>(xr + k, xv);
#pragma unroll
                for (int j = 0; j < 8; ++j) s = chain_step<XT, WT>(s, wv[j], xv[j]);
            }
        }
    }
    if (__syncthreads_or(!ok)) return;
    RVC_MARK(0, 2);
    if (active) {
        float v = s;
        if (a.bias) v = __fadd_rn(v, __ldg(a.bias + (size_t)(t0 + tl) * a.bias_stride + e0 + el));
        a.lexact[(size_t)(t0 + tl) * a.n_experts + e0 + el] = v;
    }
    if (!a.done_cnt) return;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(a.done_cnt, 1u) == gridDim.x * gridDim.y - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int t = 0; t < a.n_tok; ++t)
        block_select(a.lexact + (size_t)t * a.n_experts, a.n_experts, a.used, a.ids + (size_t)t * a.used,
                     a.wts + (size_t)t * a.used, sc);
    if (tid == 0) *a.done_cnt = 0;
    RVC_MARK(0, 3);
}

// Exact chain of one (token, expert) logit with the router row streamed from global memory
// (L2) through a double-buffered register window of 64 elements, and x from shared memory.
template <typename WT>
struct RowWin {
    static constexpr int NV = 64 * (int)sizeof(WT) / 16;  // uint4 per 64 elements
    uint4 v[NV];
    __device__ __forceinline__ void load(const WT *p) {
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = __ldg(reinterpret_cast<const uint4 *>(p) + i);
    }
    __device__ __forceinline__ float at(int j) const;
};
template <>
__device__ __forceinline__ float RowWin<uint16_t>::at(int j) const {
    const uint32_t wd = (&v[j >> 3].x)[(j >> 1) & 3];
    return __uint_as_float((j & 1) ? (wd & 0xffff0000u) : (wd << 16));
}
template <>
__device__ __forceinline__ float RowWin<float>::at(int j) const {
    return __uint_as_float((&v[j >> 2].x)[j & 3]);
}

template <typename XT, typename WT>
__device__ float chain_streamed(const WT *wrow, const float *xs, int n) {
    RowWin<WT> A, B;
    A.load(wrow);
    float s = -0.0f;
    for (int k = 0; k < n; k += 64) {
        if (k + 64 < n) B.load(wrow + k + 64);
#pragma unroll
        for (int j = 0; j < 64; ++j) s = chain_step<XT, WT>(s, A.at(j), xs[k + j]);
        A = B;
    }
    return s;
}

// Dispatch plan (MoePlan, exec.rs:541-557) of n_pairs <= RF_MAX_TOK * MAX_USED pairs inside one
// CTA, by ranks: a pair's plan position is the number of pairs with a smaller expert plus the
// number of earlier pairs with the same expert. ids in shared memory.
__device__ void rank_plan(const int32_t *s_ids, int n_pairs, int n_experts, PlanOut p, int *s_count, int *s_base) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nth = blockDim.x;
    for (int e = tid; e < MAX_EXPERTS; e += nth) {
        int c = 0;
        if (e < n_experts)
            for (int q = 0; q < n_pairs; ++q) c += s_ids[q] == e;
        s_count[e] = c;
    }
    __syncthreads();
    if (warp == 0) {
        constexpr int PL = MAX_EXPERTS / 32;
        int run = 0, flags = 0;
#pragma unroll
        for (int i = 0; i < PL; ++i) {
            const int e = lane * PL + i;
            run += e < n_experts ? s_count[e] : 0;
            flags += (e < n_experts && s_count[e] > 0);
        }
        int incl = run, fin = flags;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o), z = __shfl_up_sync(0xffffffffu, fin, o);
            if (lane >= o) incl += y, fin += z;
        }
        int base = incl - run, slot = fin - flags;
#pragma unroll
        for (int i = 0; i < PL; ++i) {
            const int e = lane * PL + i;
            if (e < n_experts) {
                s_base[e] = base;
                p.offsets[e] = base;
                p.counts[e] = s_count[e];
                if (s_count[e] > 0) p.active[slot++] = e;
                base += s_count[e];
            }
        }
        if (lane == 31) {
            p.offsets[n_experts] = incl;
            *p.n_active = fin;
        }
    }
    __syncthreads();
    for (int q = tid; q < n_pairs; q += nth) {
        const int e = s_ids[q];
        int k = s_base[e];
        for (int r = 0; r < q; ++r) k += s_ids[r] == e;
        p.order[k] = q;
        p.pos_of[q] = k;
    }
}

// ------------------------------------------------------------------ K1
constexpr int RF_THREADS = 256;
constexpr double RF_U = 5.9604644775390625e-08;  // 2^-24, unit roundoff of f32

struct VerifyScratch {
    int32_t key[MAX_EXPERTS];
    float l[MAX_EXPERTS], bd[MAX_EXPERTS];
    int top[MAX_USED + 1];
    float redf[32];
};

// grid: min(n_experts, #SMs) CTAs, 256 threads; dynamic smem: one x row as f32 (fallback).
// The lane K chunk is NB8 groups of 8 elements (n_embd = 256 * NB8); each group's f64 sums are
// formed separately so every dependent chain is short (8 products, then NB8 group sums).
template <typename XT, typename WT, int NB8>
__global__ void __launch_bounds__(RF_THREADS) k_route_fast(RouteArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];  // fallback: one x row as f32
    __shared__ int s_last, s_nflag;
    __shared__ int s_flag[RF_MAX_TOK];
    __shared__ int32_t s_ids[RF_MAX_TOK * MAX_USED];
    __shared__ int s_count[MAX_EXPERTS], s_base[MAX_EXPERTS];
    __shared__ union {
        VerifyScratch v;
        SelScratch s;
    } sc;
    RVC_MARK(1, 0);
    const XT *x = static_cast<const XT *>(a.x);
    const WT *w = static_cast<const WT *>(a.w);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ne = a.n_experts;
    constexpr int chunk = NB8 * 8;

    // 1. every (token, expert) dot in f64 with its bound; warp per dot, lane per K chunk
    for (int e = blockIdx.x; e < ne; e += gridDim.x) {
        for (int t = warp; t < a.n_tok; t += RF_THREADS / 32) {
            const WT *wr = w + (size_t)e * a.n_embd + (size_t)lane * chunk;
            const XT *xr = x + (size_t)t * a.n_embd + (size_t)lane * chunk;
            // pass 1: per-group f64 sums (exact-ish) and sum |p| (f32 is enough for a bound)
            double gsum[NB8];
            float P = 0.0f;
#pragma unroll
            for (int g = 0; g < NB8; ++g) {
                float wv[8], xv[8];
                ld8<WT>(wr, g * 8, wv);
                ld8<XT>(xr, g * 8, xv);
                double s8 = 0.0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const double p = (double)wv[j] * (double)xv[j];
                    s8 += p;
                    P += fabsf(wv[j] * xv[j]);
                }
                gsum[g] = s8;
            }
            double c = 0.0;
            float gpre[NB8];
#pragma unroll
            for (int g = 0; g < NB8; ++g) gpre[g] = (float)c, c += gsum[g];
            double incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const float off = (float)(incl - c);
            // pass 2: sum over the prefix sums |S_i| (f32; relative error far inside the 1% margin)
            float A = 0.0f;
#pragma unroll 1
            for (int g = 0; g < NB8; ++g) {
                float wv[8], xv[8];
                ld8<WT>(wr, g * 8, wv);
                ld8<XT>(xr, g * 8, xv);
                float r = off + gpre[g], ag = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    r += wv[j] * xv[j];
                    ag += fabsf(r);
                }
                A += ag;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                A += __shfl_xor_sync(0xffffffffu, A, o);
                P += __shfl_xor_sync(0xffffffffu, P, o);
            }
            const double S = __shfl_sync(0xffffffffu, incl, 31);
            if (lane == 0) {
                const double b = a.bias ? (double)__ldg(a.bias + (size_t)t * a.bias_stride + e) : 0.0;
                const double l = S + b;
                const double bd = 1.02 * RF_U * ((double)A + (double)P) + 2.02 * RF_U * (fabs(S) + fabs(b)) + 1e-30;
                a.lfast[(size_t)t * ne + e] = (float)l;
                a.lbound[(size_t)t * ne + e] = (float)(bd * 1.001);
            }
        }
    }
    RVC_MARK(1, 1);
    // 2. Q8_0 of x, spread over every warp of the grid
    if (a.xrec) {
        const int nb = a.n_embd / QK;
        const long long total = (long long)a.n_tok * nb;
        for (long long i = (long long)blockIdx.x * (RF_THREADS / 32) + warp; i < total;
             i += (long long)gridDim.x * (RF_THREADS / 32)) {
            const long long t = i / nb, b = i % nb;
            const float v = ld_val<XT>(x, (size_t)t * a.n_embd + (size_t)b * QK + lane);
            uint16_t dbits;
            int qsum;
            const int8_t q = quant_q8_lane(v, &dbits, &qsum);
            q8rec_store(a.xrec + (size_t)t * q8rec_bytes(nb), nb, (int)b, lane, q, dbits, qsum);
        }
    }
    // 3. the last CTA verifies, falls back, selects and plans
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(a.done_cnt, 1u) == gridDim.x - 1;
        s_nflag = 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    RVC_MARK(1, 2);
    const int used = a.used;
    for (int t = 0; t < a.n_tok; ++t) {
        VerifyScratch &v = sc.v;
        float mo = -INFINITY;
        for (int e = tid; e < ne; e += RF_THREADS) {
            v.l[e] = __ldcg(a.lfast + (size_t)t * ne + e);
            v.bd[e] = __ldcg(a.lbound + (size_t)t * ne + e);
            v.key[e] = total_key(v.l[e]);
        }
        __syncthreads();
        for (int e = tid; e < ne; e += RF_THREADS) {
            const int32_t k = v.key[e];
            int rank = 0;
            for (int f = 0; f < ne; ++f) rank += (v.key[f] > k) | ((v.key[f] == k) & (f < e));
            if (rank < used)
                v.top[rank] = e;
            else
                mo = fmaxf(mo, v.l[e] + v.bd[e]);  // every expert left out, with its bound
        }
        mo = block_max(mo, v.redf);
        if (tid == 0) {
            bool ok = true;
            const float l0 = v.l[v.top[0]];
            for (int j = 0; j < used; ++j) {
                const int ej = v.top[j];
                const float lo = v.l[ej] - v.bd[ej];
                // strictly above the next pick (or, for the last pick, every expert left out)
                const bool last = j + 1 == used;
                const float hi = last ? mo : v.l[v.top[j + 1]] + v.bd[v.top[j + 1]];
                const float nxt = last ? mo : v.l[v.top[j + 1]];
                if (!(lo > hi + 1e-6f * (1.0f + fabsf(nxt - l0)))) ok = false;
                if (!(v.l[ej] - l0 > -80.0f)) ok = false;  // far from underflow in softmax
                s_ids[t * used + j] = ej;
            }
            s_flag[t] = !ok;
            if (!ok) ++s_nflag;
        }
        __syncthreads();
    }
    RVC_MARK(1, 3);
    if (tid == 0 && a.fallback_cnt && s_nflag > 0) atomicAdd(a.fallback_cnt, (unsigned)s_nflag);
    if (s_nflag > 0) {
        // exact chains for the ambiguous tokens, one token at a time: x staged in shared memory
        // as f32, one thread per expert streaming its router row from L2
        float *xs = reinterpret_cast<float *>(smem);
        for (int t = 0; t < a.n_tok; ++t) {
            if (!s_flag[t]) continue;
            for (int k = tid; k < a.n_embd; k += RF_THREADS) xs[k] = ld_val<XT>(x, (size_t)t * a.n_embd + k);
            __syncthreads();
            for (int e = tid; e < ne; e += RF_THREADS) {
                float v = chain_streamed<XT, WT>(w + (size_t)e * a.n_embd, xs, a.n_embd);
                if (a.bias) v = __fadd_rn(v, __ldg(a.bias + (size_t)t * a.bias_stride + e));
                a.lexact[(size_t)t * ne + e] = v;
            }
            __syncthreads();
            block_select(a.lexact + (size_t)t * ne, ne, used, s_ids + t * used, nullptr, sc.s);
        }
    }
    __syncthreads();
    const int n_pairs = a.n_tok * used;
    for (int q = tid; q < n_pairs; q += RF_THREADS) a.ids[q] = s_ids[q];
    RVC_MARK(1, 4);
    rank_plan(s_ids, n_pairs, ne, a.plan, s_count, s_base);
    if (tid == 0) *a.done_cnt = 0;
    RVC_MARK(1, 5);
}

}  // namespace rvc
