// router_fast.cuh - the reference's exact router order, and the bound that lets a fast router skip it.
//
// The reference router is a sequential f32 dot per (token, expert) (matvec_f32,
// runtime/src/ops.rs:321-326), so its logits carry that order's rounding.
//
// k_router_chains: the exact chains themselves, one per thread, with whole rows of the router
//    and of x staged into shared memory by a few large 1-D TMA bulk copies. Logits are
//    bit-identical to the reference (rvc_moe_router returns them); with a done counter the
//    last CTA also selects (softmax, top-k, renormalised weights: block_select).
// The decode kernel (decode_fused.cuh) instead forms every (token, expert) dot in f64 (the
//    products of bf16/f32 operands are exact in f64) together with a rigorous bound on how far
//    the sequential f32 result can be from it: |s_seq - S| <= u * (sum_i |S_i| + sum_i |p_i|)
//    * (1 + 1e-2), S_i the exact prefix sums (Higham, Accuracy and Stability of Numerical
//    Algorithms, 2nd ed., eq. 4.4 with products rounded once), plus the rounding of the bias
//    add and of the f32 store (RF_U below). A token whose top-(used+1) are separated by more
//    than their bounds has the same ids in the reference; any other token gets its logits from
//    exact chains (chain_streamed) - about 3% of tokens at the benchmark's distributions.
#pragma once
#include "common.cuh"
#include "router.cuh"

namespace rvc {

struct RouteArgs {
    const void *x;
    const void *w;
    const float *bias;
    int bias_stride;
    int n_tok, n_experts, n_embd, used;
    float *lexact;          // [n_tok][n_experts] exact logits
    unsigned *done_cnt;     // last-CTA counter (zero between launches), or NULL: no selection
    int32_t *ids;           // [n_tok][used]
    float *wts;             // [n_tok][used]
    int *status;
};

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
        const float ex = fd_exp_f32(__fsub_rn(sc.p[e], m));
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
        if (!fd_mbar_wait(&bars[c], 0, a.status)) ok = false;
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

// ------------------------------------------------------------------ K0, batches
// The same exact chains for batches of 32 tokens and more: a tile of C4_E experts x C4_T tokens
// per CTA of 128 threads, each thread running 4 independent chains (2 experts x 2 tokens) so
// that the FMA latency of one chain hides behind the other three; the tile's rows stream in
// chunks of C4_CH columns through two shared-memory buffers (1-D TMA bulk copies, one per row
// and chunk). Every chain is still the reference's sequential order over all columns.
constexpr int C4_E = 16, C4_T = 32, C4_CH = 352, C4_THREADS = 128;

template <typename T>
__host__ __device__ constexpr int c4_row_bytes() {
    return C4_CH * (int)sizeof(T) + 16;  // padded: rows of one column start in different banks
}
template <typename XT, typename WT>
__host__ __device__ constexpr int c4_buf_bytes() {
    return C4_E * c4_row_bytes<WT>() + C4_T * c4_row_bytes<XT>();
}

template <typename XT, typename WT>
__global__ void __launch_bounds__(C4_THREADS) k_router_chains4(RouteArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[2];
    const int e0 = blockIdx.x * C4_E, t0 = blockIdx.y * C4_T;
    const int nw = min(C4_E, a.n_experts - e0), nx = min(C4_T, a.n_tok - t0);
    const int tid = threadIdx.x, n = a.n_embd, nch = n / C4_CH;
    constexpr int wrb = c4_row_bytes<WT>(), xrb = c4_row_bytes<XT>(), bb = c4_buf_bytes<XT, WT>();
    const WT *w = static_cast<const WT *>(a.w);
    const XT *x = static_cast<const XT *>(a.x);
    if (tid == 0) {
        mbar_init(&full[0], nw + nx);  // one arrival per staged row
        mbar_init(&full[1], nw + nx);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int c) {  // thread r < nw + nx: row r's chunk c (router rows, then x rows)
        if (tid >= nw + nx) return;
        uint8_t *base = smem + (c & 1) * bb;
        const bool isw = tid < nw;
        const int r = isw ? tid : tid - nw;
        const uint32_t bytes = (uint32_t)C4_CH * (isw ? sizeof(WT) : sizeof(XT));
        uint8_t *dst = isw ? base + r * wrb : base + C4_E * wrb + r * xrb;
        const uint8_t *src = isw ? reinterpret_cast<const uint8_t *>(w + (size_t)(e0 + r) * n + (size_t)c * C4_CH)
                                 : reinterpret_cast<const uint8_t *>(x + (size_t)(t0 + r) * n + (size_t)c * C4_CH);
        mbar_arrive_expect_tx(&full[c & 1], bytes);
        bulk_g2s(dst, src, bytes, &full[c & 1]);
    };
    issue(0);
    if (nch > 1) issue(1);
    const int ep = tid >> 4, tp = tid & 15;  // experts e0 + 2 ep (+1), tokens t0 + 2 tp (+1)
    float s00 = -0.0f, s01 = -0.0f, s10 = -0.0f, s11 = -0.0f;
    for (int c = 0; c < nch; ++c) {
        const int b = c & 1;
        const bool ok = fd_mbar_wait(&full[b], (uint32_t)(c >> 1) & 1u, a.status);
        if (__syncthreads_or(!ok)) return;
        const uint8_t *base = smem + b * bb;
        const WT *w0 = reinterpret_cast<const WT *>(base + (2 * ep) * wrb), *w1 = reinterpret_cast<const WT *>(base + (2 * ep + 1) * wrb);
        const XT *x0 = reinterpret_cast<const XT *>(base + C4_E * wrb + (2 * tp) * xrb);
        const XT *x1 = reinterpret_cast<const XT *>(base + C4_E * wrb + (2 * tp + 1) * xrb);
#pragma unroll 2
        for (int k = 0; k < C4_CH; k += 8) {
            float wa[8], wb[8], xa[8], xb[8];
            lds8<WT>(w0 + k, wa);
            lds8<WT>(w1 + k, wb);
            lds8<XT>(x0 + k, xa);
            lds8<XT>(x1 + k, xb);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                s00 = chain_step<XT, WT>(s00, wa[j], xa[j]);
                s01 = chain_step<XT, WT>(s01, wa[j], xb[j]);
                s10 = chain_step<XT, WT>(s10, wb[j], xa[j]);
                s11 = chain_step<XT, WT>(s11, wb[j], xb[j]);
            }
        }
        __syncthreads();  // every thread is done with buffer b
        if (c + 2 < nch) issue(c + 2);
    }
    const float sv[2][2] = {{s00, s01}, {s10, s11}};
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int el = 2 * ep + i, tl = 2 * tp + j;
            if (el < nw && tl < nx) {
                float v = sv[i][j];
                if (a.bias) v = __fadd_rn(v, __ldg(a.bias + (size_t)(t0 + tl) * a.bias_stride + e0 + el));
                a.lexact[(size_t)(t0 + tl) * a.n_experts + e0 + el] = v;
            }
        }
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

constexpr double RF_U = 5.9604644775390625e-08;  // 2^-24, unit roundoff of f32

}  // namespace rvc
