// experts_decode.cuh - Q4_0 x Q8_0 expert GEMVs for decode batches (sm_100a).
//
// Replaces the reference's per-expert device loop (runtime/src/hip_exec.rs:820-843:
// gather_rows, q4_mm per group, geglu_split, q4_mm per group, moe_combine) and computes
// what the CPU-experts Q8_0 path computes (runtime/src/exec.rs:572-640 with
// Activation::Q8_0, runtime/src/expert_pool.rs:311-320 and
// runtime/src/expert_kernel.rs:147-161):
//   gate/up:  y = sum_b sumi_b * (dw_b * dx_b), sumi_b the exact int32 block dot, summed in
//             block order with separately rounded f32 operations (the scalar reference order);
//   h = gelu_tanh(gate) * up, re-quantised to Q8_0 per 32 columns;
//   down:     the same block dot over h;
//   combine:  out[t] = sum_j (y_j * down_scale[e_j]) * w_j in slot order (bit-exact order).
//
// Weights are the packed planes written by k_pack_experts (pack.cuh): nibbles and f16 scales
// in separate 16-byte-aligned planes, gate and up rows interleaved per 32 columns so that one
// unit of 64 packed rows carries gate and up for the same 32 h columns. Whole units are
// staged into shared memory with 1-D TMA bulk copies (cp.async.bulk) on an mbarrier.
#pragma once
#include "common.cuh"

namespace rvc {

struct PlanView {
    const int32_t *counts;   // [n_experts]
    const int32_t *offsets;  // [n_experts + 1]
    const int32_t *order;    // [pairs] pair index at plan position k
    const int32_t *pos_of;   // [pairs]
    const int32_t *active;   // [n_experts] ascending experts with pairs
    const int32_t *n_active; // [1]
};

// Packed expert planes (byte offsets inside the packed buffer are computed on the host).
struct PackedView {
    const uint8_t *gu_nib;   // [E][2*ff packed rows][nb][16]
    const uint16_t *gu_scl;  // [E][2*ff][nb]
    const uint8_t *dn_nib;   // [E][n_embd][nbh][16]
    const uint16_t *dn_scl;  // [E][n_embd][nbh]
};

struct Q8View {
    const int8_t *q;   // [rows][nblk][32]
    const float *d;    // [rows][nblk]
    const int32_t *s;  // [rows][nblk]
};

constexpr int GU_UNIT_ROWS = 64;  // 32 gate + 32 up rows = one Q8 block of h
constexpr int GU_TOK = 4;         // tokens processed together per pass

// grid: (ff/32 column groups, max active experts); block 256 (8 warps).
// Warp w, pass p handles packed rows p*32 + w*4 + lane/8; lane%8 strides the nb blocks.
__global__ void __launch_bounds__(256) k_gate_up_decode(PackedView pk, int n_embd, int ff, Q8View x, PlanView plan,
                                                        int used, int8_t *__restrict__ hq, float *__restrict__ hd,
                                                        int32_t *__restrict__ hs, int *status) {
    const int nb = n_embd / QK;
    const int q = blockIdx.x;
    const int a = blockIdx.y;
    if (a >= __ldg(plan.n_active)) return;
    const int e = __ldg(plan.active + a);
    const int p0 = __ldg(plan.offsets + e);
    const int n_e = __ldg(plan.counts + e);
    const int nbh = ff / QK;

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *snib = smem;
    uint16_t *sscl = reinterpret_cast<uint16_t *>(smem + (size_t)GU_UNIT_ROWS * nb * 16);
    __shared__ uint64_t bar;
    __shared__ float sg[GU_TOK][32], su[GU_TOK][32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        const size_t row0 = (size_t)e * 2 * ff + (size_t)q * GU_UNIT_ROWS;
        const uint32_t nib_bytes = GU_UNIT_ROWS * nb * 16, scl_bytes = GU_UNIT_ROWS * nb * 2;
        mbar_arrive_expect_tx(&bar, nib_bytes + scl_bytes);
        bulk_g2s(snib, pk.gu_nib + row0 * nb * 16, nib_bytes, &bar);
        bulk_g2s(sscl, pk.gu_scl + row0 * nb, scl_bytes, &bar);
    }
    if (!mbar_wait(&bar, 0, status)) return;

    // Each row's dot follows the reference's scalar order exactly (expert_kernel.rs:147-161):
    // acc = 0; for b in 0..nb: acc = acc + (float)sumi_b * (dw_b * dx_b), each operation
    // rounded separately. The 8 lanes of a row group each form one block term per chunk of 8
    // blocks; the terms are then added in block order through shuffles.
    const int grp = lane >> 3, l8 = lane & 7;
    for (int c0 = 0; c0 < n_e; c0 += GU_TOK) {
        const int nt = min(GU_TOK, n_e - c0);
        int tok[GU_TOK];
#pragma unroll
        for (int i = 0; i < GU_TOK; ++i) tok[i] = i < nt ? __ldg(plan.order + p0 + c0 + i) / used : 0;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
            const int r = pass * 32 + warp * 4 + grp;  // packed row within the unit
            float acc[GU_TOK];
#pragma unroll
            for (int i = 0; i < GU_TOK; ++i) acc[i] = 0.0f;
            for (int cb = 0; cb < nb; cb += 8) {
                const int b = cb + l8;
                const uint4 nib = *reinterpret_cast<const uint4 *>(snib + ((size_t)r * nb + b) * 16);
                const float dw = f16_bits_to_f32(sscl[r * nb + b]);
                float term[GU_TOK];
#pragma unroll
                for (int i = 0; i < GU_TOK; ++i) {
                    term[i] = 0.0f;
                    if (i < nt) {
                        const size_t xb = (size_t)tok[i] * nb + b;
                        const int4 qa = __ldg(reinterpret_cast<const int4 *>(x.q + xb * QK));
                        const int4 qb = __ldg(reinterpret_cast<const int4 *>(x.q + xb * QK + 16));
                        const int sumi = q4q8_sumi(nib, qa, qb, __ldg(x.s + xb));
                        term[i] = __fmul_rn((float)sumi, __fmul_rn(dw, __ldg(x.d + xb)));
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
#pragma unroll
                    for (int i = 0; i < GU_TOK; ++i)
                        acc[i] = __fadd_rn(acc[i], __shfl_sync(0xffffffffu, term[i], (lane & ~7) | j));
                }
            }
#pragma unroll
            for (int i = 0; i < GU_TOK; ++i) {
                if (l8 == 0 && i < nt) {
                    const int col = warp * 4 + grp;
                    if (pass == 0)
                        sg[i][col] = acc[i];
                    else
                        su[i][col] = acc[i];
                }
            }
        }
        __syncthreads();
        // h = gelu(gate) * up for the 32 columns, then Q8_0 of the block (warp i: token i).
        if (warp < nt) {
            const float h = __fmul_rn(gelu_tanh(sg[warp][lane]), su[warp][lane]);
            uint16_t dbits;
            int qsum;
            const int8_t qv = quant_q8_lane(h, &dbits, &qsum);
            const size_t k = (size_t)(p0 + c0 + warp);  // plan position of this pair
            hq[(k * nbh + q) * QK + lane] = qv;
            if (lane == 0) {
                hd[k * nbh + q] = f16_bits_to_f32(dbits);
                hs[k * nbh + q] = qsum;
            }
        }
        __syncthreads();
    }
}

// Down projection + slot-order combine. grid: n_embd / DN_ROWS CTAs; block 256.
// Each CTA owns DN_ROWS output rows across every active expert, so the weighted combine of
// a token's `used` experts happens in shared memory in the reference's slot order.
constexpr int DN_ROWS = 16;
constexpr int DN_STAGES = 6;

__global__ void __launch_bounds__(256) k_down_combine_decode(PackedView pk, int n_embd, int ff, Q8View h,
                                                             PlanView plan, const int32_t *__restrict__ ids,
                                                             const float *__restrict__ wts,
                                                             const float *__restrict__ down_scale, int n_tok, int used,
                                                             float *__restrict__ out, int *status) {
    const int nbh = ff / QK;
    const int r0 = blockIdx.x * DN_ROWS;
    const int n_act = __ldg(plan.n_active);
    const int pairs = n_tok * used;
    const uint32_t nib_bytes = DN_ROWS * nbh * 16, scl_bytes = DN_ROWS * nbh * 2;
    const uint32_t stage_bytes = (nib_bytes + scl_bytes + 127) & ~127u;

    extern __shared__ __align__(128) uint8_t smem[];
    float *ysm = reinterpret_cast<float *>(smem + (size_t)DN_STAGES * stage_bytes);  // [pairs][DN_ROWS]
    __shared__ uint64_t bars[DN_STAGES];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        for (int s = 0; s < DN_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int a) {
        const int s = a % DN_STAGES;
        const int e = __ldg(plan.active + a);
        uint8_t *dst = smem + (size_t)s * stage_bytes;
        const size_t row0 = (size_t)e * n_embd + r0;
        mbar_arrive_expect_tx(&bars[s], nib_bytes + scl_bytes);
        bulk_g2s(dst, pk.dn_nib + row0 * nbh * 16, nib_bytes, &bars[s]);
        bulk_g2s(dst + nib_bytes, pk.dn_scl + row0 * nbh, scl_bytes, &bars[s]);
    };
    if (tid == 0)
        for (int a = 0; a < min(DN_STAGES, n_act); ++a) issue(a);

    for (int a = 0; a < n_act; ++a) {
        const int s = a % DN_STAGES;
        if (!mbar_wait(&bars[s], (a / DN_STAGES) & 1, status)) return;
        const int e = __ldg(plan.active + a);
        const int p0 = __ldg(plan.offsets + e), n_e = __ldg(plan.counts + e);
        const uint8_t *snib = smem + (size_t)s * stage_bytes;
        const uint16_t *sscl = reinterpret_cast<const uint16_t *>(snib + nib_bytes);
        // warp w: rows w and w + 8; lane b < nbh: block b
        for (int rr = warp; rr < DN_ROWS; rr += 8) {
            uint4 nib = make_uint4(0, 0, 0, 0);
            float dw = 0.0f;
            if (lane < nbh) {
                nib = *reinterpret_cast<const uint4 *>(snib + ((size_t)rr * nbh + lane) * 16);
                dw = f16_bits_to_f32(sscl[rr * nbh + lane]);
            }
            for (int j = 0; j < n_e; ++j) {
                const size_t k = (size_t)(p0 + j);
                float term = 0.0f;
                if (lane < nbh) {
                    const size_t hb = k * nbh + lane;
                    const int4 qa = __ldg(reinterpret_cast<const int4 *>(h.q + hb * QK));
                    const int4 qb = __ldg(reinterpret_cast<const int4 *>(h.q + hb * QK + 16));
                    const int sumi = q4q8_sumi(nib, qa, qb, __ldg(h.s + hb));
                    term = __fmul_rn((float)sumi, __fmul_rn(dw, __ldg(h.d + hb)));
                }
                // block terms added in block order, as the scalar reference (expert_kernel.rs:147-161)
                float acc = 0.0f;
                for (int b = 0; b < nbh; ++b) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, term, b));
                if (lane == 0) ysm[k * DN_ROWS + rr] = acc;
            }
        }
        __syncthreads();
        if (tid == 0 && a + DN_STAGES < n_act) issue(a + DN_STAGES);
    }
    __syncthreads();
    // slot-order combine (exec.rs:626-638): o = (y*ds)*w for j = 0, then o = o + (y*ds)*w
    for (int i = tid; i < n_tok * DN_ROWS; i += blockDim.x) {
        const int t = i / DN_ROWS, rr = i % DN_ROWS;
        float o = 0.0f;
        for (int j = 0; j < used; ++j) {
            const int p = t * used + j;
            const int e = __ldg(ids + p);
            const float ds = down_scale ? __ldg(down_scale + e) : 1.0f;
            const int k = __ldg(plan.pos_of + p);
            const float v = __fmul_rn(__fmul_rn(ysm[(size_t)k * DN_ROWS + rr], ds), __ldg(wts + p));
            o = j == 0 ? v : __fadd_rn(o, v);
        }
        out[(size_t)t * n_embd + r0 + rr] = o;
    }
    (void)pairs;
}

}  // namespace rvc
