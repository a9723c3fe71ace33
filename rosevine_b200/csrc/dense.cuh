// dense.cuh - the layer's shared dense MLP (gate / up / down Q4_0 matrices, F32 activations).
//
// The reference runs it beside the MoE branch (runtime/src/exec.rs:438-453 on the CPU,
// runtime/src/hip_exec.rs:770-778 on the device): cur = rms_norm(o) * ffn_norm; gate = Wg . cur,
// up = Wu . cur (ops::matmul_q4_0, ops.rs:249-266); mlp = gelu(gate) * up; cur = Wd . mlp; then
// rms_norm(cur) * post_ffw_norm_1. Its matmul dequantises each Q4_0 row to f32 ((q - 8) * d, exact)
// and sums the rounded products of a row and a token in sequence from -0 (Rust's f32 sum). The
// kernels here keep that order: every (row, token) dot is one sequential f32 chain, so the
// outputs are the CPU reference's bit for bit, and a token's result does not depend on the
// batch it is in (the batch invariance the reference asks of its device matmul,
// runtime/tests/hip_ops.rs:73-79).
//
// k_q4_chains: a CTA holds a tile of rows x 32 tokens; per chunk of 256 columns its threads
// dequantise the tile's rows into shared memory (one 32-element Q4_0 block per thread) and copy
// the tokens' columns beside them, then each thread advances four chains over the chunk:
//   PLAIN  rows r, r + 16 of one matrix x tokens t, t + 16            (32 rows per CTA)
//   GU     row r of the gate and of the up matrix x tokens t, t + 16 (16 rows per CTA), and at
//          the end mlp = gelu(gate) * up (ops.rs:145-149), fused.
// The chains' dependent additions bound a small batch (2816 of them per dot); with many tokens
// the kernel is bound by the f32 pipe (2 operations per product). A warp holds 16 rows and two
// token slots: its weight loads (16 rows, 260-float stride) fall in distinct banks, its token
// loads are broadcasts.
#pragma once
#include "common.cuh"

namespace rvc {

constexpr int DN_T = 32;                 // tokens per CTA
constexpr int DN_KC = 256;               // columns per chunk (8 Q4_0 blocks)
constexpr int DN_LD = DN_KC + 4;         // shared row stride in floats (bank spread)
constexpr int DN_THREADS = 256;
constexpr int DN_ROWS = 32;              // matrix rows per CTA (both layouts hold 32 dequantised rows)
constexpr int DN_SMEM = 2 * (DN_ROWS + DN_T) * DN_LD * 4;  // two buffers: 133,120 B
constexpr int DN_XQ = DN_T * DN_KC / 4 / DN_THREADS;      // float4 of token columns per thread and chunk

struct DenseArgs {
    const uint8_t *w0;  // PLAIN: the matrix; GU: the gate matrix (Q4_0 rows of k columns)
    const uint8_t *w1;  // GU: the up matrix
    const float *x;     // [n_tok][k]
    float *y;           // PLAIN: [n_tok][n_out]; GU: mlp [n_tok][n_out]
    int n_out, k, n_tok;
};

// Dequantise one Q4_0 block, given as its nine little-endian 16-bit words (ops.rs:83-92: element
// j < 16 the low nibble of byte j, element j + 16 its high nibble, value (q - 8) * d), into 32
// floats at dst (16-byte aligned).
__device__ __forceinline__ void dq_block(const uint16_t (&h)[9], float *dst) {
    const float d = f16_bits_to_f32(h[0]);
    uint32_t b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = (uint32_t)h[1 + 2 * i] | ((uint32_t)h[2 + 2 * i] << 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float4 lo, hi;
        lo.x = __fmul_rn((float)((int)(b[i] & 15u) - 8), d);
        lo.y = __fmul_rn((float)((int)((b[i] >> 8) & 15u) - 8), d);
        lo.z = __fmul_rn((float)((int)((b[i] >> 16) & 15u) - 8), d);
        lo.w = __fmul_rn((float)((int)((b[i] >> 24) & 15u) - 8), d);
        hi.x = __fmul_rn((float)((int)((b[i] >> 4) & 15u) - 8), d);
        hi.y = __fmul_rn((float)((int)((b[i] >> 12) & 15u) - 8), d);
        hi.z = __fmul_rn((float)((int)((b[i] >> 20) & 15u) - 8), d);
        hi.w = __fmul_rn((float)((int)(b[i] >> 28) - 8), d);
        reinterpret_cast<float4 *>(dst)[i] = lo;
        reinterpret_cast<float4 *>(dst + 16)[i] = hi;
    }
}

template <bool GU>
__global__ void __launch_bounds__(DN_THREADS) k_q4_chains(DenseArgs a) {
    extern __shared__ __align__(16) float dsm[];
    constexpr int RPC = GU ? DN_ROWS / 2 : DN_ROWS;  // output rows per CTA
    const int tid = threadIdx.x;
    const int r0 = blockIdx.x * RPC, t0 = blockIdx.y * DN_T;
    const int nb = a.k / QK, rowb = nb * 18;  // Q4_0 blocks and bytes per row
    const int nch = (a.k + DN_KC - 1) / DN_KC;
    // chains: rows rr, rr + 16 (PLAIN) or row rr of both matrices (GU), tokens tt, tt + 16. The
    // tokens vary across warps (warp w holds tt = 2w, 2w + 1), so with a small batch whole warps
    // have no token and skip the arithmetic.
    const int rr = tid & 15, tt = tid >> 4;
    const bool active = t0 + (tt & ~1) < a.n_tok || t0 + (tt & ~1) + 16 < a.n_tok;  // warp-uniform
    // staging: block (srow, sblk) of the chunk's weights, and DN_XQ float4 of the tokens'
    // columns; the next chunk's bytes are loaded into registers before this chunk's arithmetic
    // and written to shared memory after it, so that the loads' latency overlaps the chains
    const int srow = tid >> 3, sblk = tid & 7;
    const uint8_t *wm = GU ? (srow < 16 ? a.w0 : a.w1) : a.w0;
    const int grow = r0 + (GU ? (srow & 15) : srow);
    uint16_t wq[9];
    float4 xq[DN_XQ];
    auto load = [&](int c) {
        const int b = c * (DN_KC / QK) + sblk;
        if (b < nb && grow < a.n_out) {
            const uint16_t *h = reinterpret_cast<const uint16_t *>(wm + (size_t)grow * rowb + (size_t)b * 18);
#pragma unroll
            for (int i = 0; i < 9; ++i) wq[i] = __ldg(h + i);
        } else {
#pragma unroll
            for (int i = 0; i < 9; ++i) wq[i] = 0;  // d = 0: zero weights
        }
        const int kc4 = min(DN_KC, a.k - c * DN_KC) / 4;
#pragma unroll
        for (int j = 0; j < DN_XQ; ++j) {
            const int i = tid + j * DN_THREADS, t = i / (DN_KC / 4), q = i - t * (DN_KC / 4);
            xq[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q < kc4 && t0 + t < a.n_tok)
                xq[j] = __ldg(reinterpret_cast<const float4 *>(a.x + (size_t)(t0 + t) * a.k + c * DN_KC) + q);
        }
    };
    auto store = [&](int c, int buf) {
        float *W = dsm + buf * (DN_ROWS + DN_T) * DN_LD;
        float *X = W + DN_ROWS * DN_LD;
        if (c * (DN_KC / QK) + sblk < nb) dq_block(wq, W + srow * DN_LD + sblk * QK);
#pragma unroll
        for (int j = 0; j < DN_XQ; ++j) {
            const int i = tid + j * DN_THREADS, t = i / (DN_KC / 4), q = i - t * (DN_KC / 4);
            reinterpret_cast<float4 *>(X + t * DN_LD)[q] = xq[j];
        }
    };
    float s00 = -0.0f, s01 = -0.0f, s10 = -0.0f, s11 = -0.0f;  // [row or matrix][token]
    load(0);
    store(0, 0);
    __syncthreads();
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) load(c + 1);
        if (active) {
            const float *W = dsm + (c & 1) * (DN_ROWS + DN_T) * DN_LD;
            const float *X = W + DN_ROWS * DN_LD;
            const float *wa = W + rr * DN_LD, *wb = W + (rr + 16) * DN_LD;
            const float *xa = X + tt * DN_LD, *xb = X + (tt + 16) * DN_LD;
            const int kc = min(DN_KC, a.k - c * DN_KC);
#pragma unroll 2
            for (int k = 0; k < kc; k += 4) {
                const float4 w0 = *reinterpret_cast<const float4 *>(wa + k), w1 = *reinterpret_cast<const float4 *>(wb + k);
                const float4 x0 = *reinterpret_cast<const float4 *>(xa + k), x1 = *reinterpret_cast<const float4 *>(xb + k);
                const float w0v[4] = {w0.x, w0.y, w0.z, w0.w}, w1v[4] = {w1.x, w1.y, w1.z, w1.w};
                const float x0v[4] = {x0.x, x0.y, x0.z, x0.w}, x1v[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // s = s + w * x, product and sum rounded separately
                    s00 = __fadd_rn(s00, __fmul_rn(w0v[j], x0v[j]));
                    s01 = __fadd_rn(s01, __fmul_rn(w0v[j], x1v[j]));
                    s10 = __fadd_rn(s10, __fmul_rn(w1v[j], x0v[j]));
                    s11 = __fadd_rn(s11, __fmul_rn(w1v[j], x1v[j]));
                }
            }
        }
        if (c + 1 < nch) store(c + 1, (c + 1) & 1);  // the buffer chunk c - 1 used: free since the last barrier
        __syncthreads();
    }
    const int ta = t0 + tt, tb = t0 + tt + 16;
    if (GU) {
        const int r = r0 + rr;
        if (r < a.n_out) {
            if (ta < a.n_tok) a.y[(size_t)ta * a.n_out + r] = __fmul_rn(gelu_tanh(s00), s10);
            if (tb < a.n_tok) a.y[(size_t)tb * a.n_out + r] = __fmul_rn(gelu_tanh(s01), s11);
        }
    } else {
        const int ra = r0 + rr, rb = r0 + rr + 16;
        if (ra < a.n_out && ta < a.n_tok) a.y[(size_t)ta * a.n_out + ra] = s00;
        if (ra < a.n_out && tb < a.n_tok) a.y[(size_t)tb * a.n_out + ra] = s01;
        if (rb < a.n_out && ta < a.n_tok) a.y[(size_t)ta * a.n_out + rb] = s10;
        if (rb < a.n_out && tb < a.n_tok) a.y[(size_t)tb * a.n_out + rb] = s11;
    }
}

// out[i] = gelu(g[i]) * u[i] (the contract of rvh_geglu, runtime/hip/rvhip.h:65).
__global__ void k_geglu(const float *__restrict__ g, const float *__restrict__ u, float *out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fmul_rn(gelu_tanh(g[i]), u[i]);
}

}  // namespace rvc
