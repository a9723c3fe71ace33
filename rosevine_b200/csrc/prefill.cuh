// prefill.cuh - the MoE layer for prefill batches (and the expert-parallel layer's expert step):
// everything around the grouped expert GEMM (prefill_tc.cuh), sm_100a.
//
// Replaces the reference's per-expert device loop (runtime/src/hip_exec.rs:820-843) for batches
// of more than 16 tokens and computes what its CPU-experts Q8_0 path computes
// (runtime/src/exec.rs:572-640, expert_pool.rs:282-355, expert_kernel.rs:147-161):
//
//   k_plan        (router.cuh) expert groups in plan order, each group starting at a multiple
//                 of 4 positions, and the list of (expert, 128-position) tiles.
//   k_pf_quant    Q8_0 of x once per token, scattered to the token's plan positions, with each
//                 block's scale in a block-major f32 plane (the layout the GEMM copies).
//   k_pf_gemm_tc  (prefill_tc.cuh) gate/up: per (expert, 128 packed gate/up rows, 128 positions)
//                 tile the exact int32 block dots on the tensor cores, the scalar reference's
//                 per-block scaling, h = gelu(gate) * up and its Q8_0 records; down: the same
//                 over the down rows and the h records, y per (position, row).
//   k_pf_combine  out[t] = slot-order sum of (y * down_scale) * w (exec.rs:626-638).
#pragma once
#include "common.cuh"
#include "pack.cuh"

#include <cuda.h>

namespace rvc {

// Bytes of one position's activation operand for the grouped GEMM (the prefill path's x and h
// records): nblk blocks of 32 quants held as f16 integers.
__host__ __device__ constexpr int pf_rec_bytes(int nblk) { return nblk * 64; }

// Activation block scales: a block-major f32 plane, ppad floats per block (ppad a multiple of
// 4, so that a tile's 128 positions start 16-byte aligned for the GEMM's tensor copies).
__device__ __forceinline__ void pf_store_scale(float *plane, int ppad, int b, int k, float d) {
    plane[(size_t)b * ppad + k] = d;
}

// ------------------------------------------------------------------ quantise + scatter
// Q8_0 of x, once per token, written to the token's `used` plan positions pos_of[t used + j]: the
// quants as f16 integers in the GEMM's activation operand (pf_rec_bytes per position, 32 f16
// per block), each block's scale in the block-major plane xsc the GEMM's scale tiles come from.
// Four lanes per block: lane l of warp w takes values 8 (l & 3) .. + 7 of block 8 w' + (l >> 2)
// of its token (one 16-byte load for bf16, two for f32; rows are 16-byte aligned, as the entry
// points require), so a warp quantises 8 blocks at once, each amax taking two shuffles within
// the group of four lanes, and writes a plan position's 8 quants per lane with one 16-byte
// store. Per value the arithmetic is quant_q8_lane's (ops.rs:95-105); a block's amax does not
// depend on the reduction order.
template <typename XT>
__global__ void __launch_bounds__(256) k_pf_quant(const XT *__restrict__ x, int n_embd, int n_tok, int used,
                                                  const int32_t *__restrict__ pos_of, uint8_t *__restrict__ xperm,
                                                  float *__restrict__ xsc, int ppad) {
    const int nb = n_embd / QK;
    const int lane = threadIdx.x & 31, part = lane & 3;
    const int nc = (nb + 7) / 8, wi = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (wi >= n_tok * nc) return;  // whole warps leave together
    const int t = wi / nc, b = (wi - t * nc) * 8 + (lane >> 2);
    const bool in = b < nb;  // lanes past the row's last block take part in the shuffles only
    float v[8];
    if (in) {
        ld8<XT>(x + (size_t)t * n_embd, (size_t)b * QK + part * 8, v);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.0f;
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t qh[4];  // the 8 quants as f16 (exact integers), two per word
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float r = roundf(__fmul_rn(v[k], id));
        const int q = r != r ? 0 : (r > 127.0f ? 127 : (r < -128.0f ? -128 : (int)r));
        const uint32_t h = __half_as_ushort(__int2half_rn(q));
        qh[k >> 1] = (k & 1) ? (qh[k >> 1] | (h << 16)) : h;
    }
    const float df = f16_bits_to_f32(f32_to_f16_bits(d));
    const int my_pos = lane < used ? __ldg(pos_of + (size_t)t * used + lane) : 0;
    const int xrb = pf_rec_bytes(nb);
    for (int j = 0; j < used; ++j) {
        const int k = __shfl_sync(0xffffffffu, my_pos, j);
        if (in) {
            uint8_t *rec = xperm + (size_t)k * xrb;
            *reinterpret_cast<uint4 *>(rec + b * 64 + part * 16) = make_uint4(qh[0], qh[1], qh[2], qh[3]);
            if (part == 0) pf_store_scale(xsc, ppad, b, k, df);
        }
    }
}

// ------------------------------------------------------------------ combine
// out[t][r] = slot-order sum over j of (y[pos_of[p_j]][r] * down_scale[e_j]) * w_j (exec.rs:626-638)
// over the occupied slots p_j = t used + j of token (or received row) t; one CTA per token, four
// rows per thread and step.
__global__ void __launch_bounds__(256) k_pf_combine(const float *__restrict__ y, const int32_t *__restrict__ pos_of,
                                                    const int32_t *__restrict__ ids, const float *__restrict__ wts,
                                                    const float *__restrict__ down_scale, int used, int n_embd,
                                                    int n_tok, float *__restrict__ out, int *status) {
    __shared__ const float4 *s_row[MAX_USED];
    __shared__ float s_ds[MAX_USED], s_w[MAX_USED];
    __shared__ int s_n;
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {  // the token's occupied slots, in slot order (-1: a slot whose expert is elsewhere)
        int n = 0;
        for (int j = 0; j < used; ++j) {
            const int p = t * used + j, e = __ldg(ids + p);
            if (e < 0) continue;
            s_row[n] = reinterpret_cast<const float4 *>(y + (size_t)__ldg(pos_of + p) * n_embd);
            s_ds[n] = down_scale ? __ldg(down_scale + e) : 1.0f;
            s_w[n] = __ldg(wts + p);
            ++n;
        }
        s_n = n;
    }
    __syncthreads();
    const int n = s_n;
    float4 *o4 = reinterpret_cast<float4 *>(out + (size_t)t * n_embd);
    const bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    for (int r = threadIdx.x; r < n_embd / 4; r += blockDim.x) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);  // a token with no slot here reads 0
        for (int j = 0; j < n; ++j) {
            const float4 v = __ldg(s_row[j] + r);
            const float ds = s_ds[j], w = s_w[j];
            const float4 c = make_float4(__fmul_rn(__fmul_rn(v.x, ds), w), __fmul_rn(__fmul_rn(v.y, ds), w),
                                         __fmul_rn(__fmul_rn(v.z, ds), w), __fmul_rn(__fmul_rn(v.w, ds), w));
            if (j == 0)
                o = c;
            else
                o = make_float4(__fadd_rn(o.x, c.x), __fadd_rn(o.y, c.y), __fadd_rn(o.z, c.z), __fadd_rn(o.w, c.w));
        }
        if (aligned) {
            o4[r] = o;
        } else {  // a caller's output that is only 4-byte aligned
            float *op = out + (size_t)t * n_embd + 4 * r;
            op[0] = o.x, op[1] = o.y, op[2] = o.z, op[3] = o.w;
        }
    }
}

// ------------------------------------------------------------------ expert parallelism
// Q8_0 records of n_rows rows of x (the rows a rank sends to the ranks holding their experts).
template <typename XT>
__global__ void __launch_bounds__(256) k_quant_rows(const XT *__restrict__ x, int n_embd, int n_rows,
                                                    uint8_t *__restrict__ rec) {
    const int nb = n_embd / QK, xrb = q8rec_bytes(nb);
    const int lane = threadIdx.x & 31;
    const long long total = (long long)n_rows * nb;
    for (long long i = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); i < total; i += (long long)gridDim.x * 8) {
        const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
        uint16_t dbits;
        int qsum;
        const int8_t q = quant_q8_lane(ld_val<XT>(x, (size_t)r * n_embd + (size_t)b * QK + lane), &dbits, &qsum);
        q8rec_store(rec + (size_t)r * xrb, nb, b, lane, q, dbits, qsum);
    }
}

constexpr int EP_MAX_RANKS = 32;  // ranks of an expert-parallel group (a token's ranks form a 32-bit mask)

// Sent rows: a token's Q8_0 record followed by its slots at the destination rank, `used` int32
// local expert ids (-1: the slot's expert is elsewhere) and `used` f32 routing weights.
__host__ __device__ constexpr int ep_row_bytes(int nb, int used) { return q8rec_bytes(nb) + used * 8; }

// Rows per destination rank: rank r holds experts [r n_local, (r + 1) n_local); a token goes once
// to every rank holding one of its experts.
__global__ void __launch_bounds__(256) k_ep_count(const int32_t *__restrict__ ids, int n_tok, int used, int n_local,
                                                  int world, int32_t *__restrict__ counts, int *status) {
    __shared__ int s_cnt[EP_MAX_RANKS];
    for (int r = threadIdx.x; r < world; r += blockDim.x) s_cnt[r] = 0;
    __syncthreads();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_tok) {
        unsigned hit = 0;
        for (int j = 0; j < used; ++j) {
            const int e = __ldg(ids + (size_t)t * used + j), r = e / n_local;
            if (e < 0 || r >= world) {
                set_status(status, STATUS_BAD_INDEX);
                continue;
            }
            hit |= 1u << r;
        }
        for (unsigned h = hit; h; h &= h - 1) atomicAdd(&s_cnt[__ffs(h) - 1], 1);
    }
    __syncthreads();
    for (int r = threadIdx.x; r < world; r += blockDim.x)
        if (s_cnt[r]) atomicAdd(counts + r, s_cnt[r]);
}

// Packing: warp w takes token w; for each rank it goes to (ascending), lane 0 takes a row in the
// rank's group (groups in rank order, rows within a group in arrival order), the warp copies the
// record and writes the slot metadata, and owner_map[t][r] gets the row (-1 for the ranks it
// does not go to).
__global__ void __launch_bounds__(256) k_ep_pack(const int32_t *__restrict__ ids, const float *__restrict__ wts,
                                                 const uint8_t *__restrict__ rec, int nb, int n_tok, int used,
                                                 int n_local, int world, const int32_t *__restrict__ counts,
                                                 int32_t *__restrict__ cursor, uint8_t *__restrict__ send,
                                                 int32_t *__restrict__ owner_map) {
    const int lane = threadIdx.x & 31, t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= n_tok) return;
    const int xrb = q8rec_bytes(nb), rb = ep_row_bytes(nb, used);
    const int e = lane < used ? __ldg(ids + (size_t)t * used + lane) : -1;
    const float wv = lane < used ? __ldg(wts + (size_t)t * used + lane) : 0.0f;
    const int my_r = e >= 0 ? e / n_local : -1;
    int base = 0;
    for (int r = 0; r < world; ++r) {
        const unsigned m = __ballot_sync(0xffffffffu, my_r == r);
        int row = -1;
        if (m) {
            if (lane == 0) row = base + atomicAdd(cursor + r, 1);
            row = __shfl_sync(0xffffffffu, row, 0);
            uint8_t *dst = send + (size_t)row * rb;
            const uint4 *src = reinterpret_cast<const uint4 *>(rec + (size_t)t * xrb);
            for (int i = lane; i < xrb / 16; i += 32) reinterpret_cast<uint4 *>(dst)[i] = __ldg(src + i);
            if (lane < used) {
                reinterpret_cast<int32_t *>(dst + xrb)[lane] = my_r == r ? e - r * n_local : -1;
                reinterpret_cast<float *>(dst + xrb + used * 4)[lane] = my_r == r ? wv : 0.0f;
            }
        }
        if (lane == 0) owner_map[(size_t)t * world + r] = row;
        base += __ldg(counts + r);
    }
}

// The slot metadata of received rows into contiguous per-(row, slot) arrays for the plan.
__global__ void __launch_bounds__(256) k_ep_meta(const uint8_t *__restrict__ rows, int nb, int n_rows, int used,
                                                 int32_t *__restrict__ slot_e, float *__restrict__ slot_w) {
    const int xrb = q8rec_bytes(nb), rb = ep_row_bytes(nb, used);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * used; i += gridDim.x * blockDim.x) {
        const int r = i / used, j = i - r * used;
        const uint8_t *m = rows + (size_t)r * rb + xrb;
        slot_e[i] = reinterpret_cast<const int32_t *>(m)[j];
        slot_w[i] = reinterpret_cast<const float *>(m + used * 4)[j];
    }
}

// Received rows to plan positions: warp task (row r, block b) writes the block's quants as f16
// integers into the activation operand of each occupied slot's plan position, and its scale into
// the block-major plane.
__global__ void __launch_bounds__(256) k_ep_scatter(const uint8_t *__restrict__ rows, int nb, int n_rows, int used,
                                                    const int32_t *__restrict__ slot_e,
                                                    const int32_t *__restrict__ pos_of, uint8_t *__restrict__ xperm,
                                                    float *__restrict__ xsc, int ppad) {
    const int rb = ep_row_bytes(nb, used), xrb = pf_rec_bytes(nb);
    const int lane = threadIdx.x & 31;
    const long long total = (long long)n_rows * nb;
    for (long long i = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); i < total; i += (long long)gridDim.x * 8) {
        const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
        const uint8_t *src = rows + (size_t)r * rb;
        const uint16_t qh = __half_as_ushort(__int2half_rn((int)(int8_t)src[q8rec_q_off(nb, b, lane)]));
        const float d = reinterpret_cast<const float *>(src + nb * 32)[b];
        for (int j = 0; j < used; ++j) {
            const int p = r * used + j;
            if (__ldg(slot_e + p) < 0) continue;
            const int k = __ldg(pos_of + p);
            reinterpret_cast<uint16_t *>(xperm + (size_t)k * xrb)[b * 32 + lane] = qh;
            if (lane == 0) pf_store_scale(xsc, ppad, b, k, d);
        }
    }
}

// Owner-side sum of the partials returned for its tokens: out[t] = the partials
// back[owner_map[t][r]] over the ranks r it was sent to, added in rank order.
__global__ void __launch_bounds__(256) k_ep_reduce(const float *__restrict__ back, const int32_t *__restrict__ owner_map,
                                                   int world, int n_embd, float *__restrict__ out) {
    __shared__ int s_row[EP_MAX_RANKS];
    const int t = blockIdx.x;
    if (threadIdx.x < world) s_row[threadIdx.x] = __ldg(owner_map + (size_t)t * world + threadIdx.x);
    __syncthreads();
    for (int r4 = threadIdx.x; r4 < n_embd / 4; r4 += blockDim.x) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        bool first = true;
        for (int r = 0; r < world; ++r) {
            if (s_row[r] < 0) continue;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(back + (size_t)s_row[r] * n_embd) + r4);
            o = first ? v : make_float4(__fadd_rn(o.x, v.x), __fadd_rn(o.y, v.y), __fadd_rn(o.z, v.z), __fadd_rn(o.w, v.w));
            first = false;
        }
        reinterpret_cast<float4 *>(out + (size_t)t * n_embd)[r4] = o;
    }
}

}  // namespace rvc
