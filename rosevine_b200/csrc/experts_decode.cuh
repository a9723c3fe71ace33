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
// Weights are the packed planes written by k_pack_q4 (pack.cuh): nibbles and f16 scales in
// separate 16-byte-aligned planes, gate and up rows interleaved per 32 columns so that one
// unit of 64 packed rows carries gate and up for the same 32 h columns. Activations are Q8_0
// row records (common.cuh). Everything a CTA reads repeatedly - its weight rows and the
// activation rows it needs - is staged into shared memory with 1-D TMA bulk copies
// (cp.async.bulk) on mbarriers, so no inner loop waits on global memory.
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

// ------------------------------------------------------------------ gate / up
constexpr int GU_UNIT_ROWS = 64;  // 32 gate + 32 up rows = one Q8 block of h
constexpr int GU_TOK = 2;         // token records staged (and processed) together

__host__ __device__ inline size_t gu_smem_bytes(int nb) {
    return (size_t)GU_UNIT_ROWS * nb * 18 + (size_t)GU_TOK * q8rec_bytes(nb);
}

// grid: (ff/32 column groups, max active experts); block 256 (8 warps).
// Warp w, pass p handles packed row p*32 + w*4 + lane/8; the 8 lanes of a row group own
// contiguous ranges of NB8 blocks each (lane l: blocks l*NB8 .. l*NB8 + NB8 - 1).
//
// Each row's dot follows the reference's scalar order exactly (expert_kernel.rs:147-161):
// acc = 0; for b in 0..nb: acc = acc + (float)sumi_b * (dw_b * dx_b), every operation rounded
// separately. Lanes first form their block terms in parallel; the running sum then visits the
// lanes in order, each adding its own NB8 terms, and is passed on with one shuffle per lane.
template <int NB8>
__global__ void __launch_bounds__(256) k_gate_up_decode(PackedView pk, int ff, const uint8_t *__restrict__ xrec,
                                                        PlanView plan, int used, uint8_t *__restrict__ hrec,
                                                        int *status) {
    RVC_MARK(2, 0);
    constexpr int nb = NB8 * 8;
    const int nbh = ff / QK;
    const int xrb = q8rec_bytes(nb), hrb = q8rec_bytes(nbh);
    const int q = blockIdx.x;
    const int a = blockIdx.y;
    if (a >= __ldg(plan.n_active)) return;
    const int e = __ldg(plan.active + a);
    const int p0 = __ldg(plan.offsets + e);
    const int n_e = __ldg(plan.counts + e);

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *snib = smem;
    uint16_t *sscl = reinterpret_cast<uint16_t *>(smem + (size_t)GU_UNIT_ROWS * nb * 16);
    uint8_t *stok = smem + (size_t)GU_UNIT_ROWS * nb * 18;  // GU_TOK token records
    __shared__ uint64_t bar_w, bar_t;
    __shared__ float sg[GU_TOK][32], su[GU_TOK][32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        mbar_init(&bar_w, 1);
        mbar_init(&bar_t, 1);
        fence_barrier_init();
    }
    __syncthreads();
    // one thread stages the records of tokens c0 .. c0 + GU_TOK - 1 of this expert (and, on
    // the first call, the unit's weight rows) on `bar`
    auto stage = [&](int c0, uint64_t *bar, bool weights) {
        const int nt = min(GU_TOK, n_e - c0);
        uint32_t bytes = nt * xrb;
        if (weights) bytes += GU_UNIT_ROWS * nb * 18;
        mbar_arrive_expect_tx(bar, bytes);
        if (weights) {
            const size_t row0 = (size_t)e * 2 * ff + (size_t)q * GU_UNIT_ROWS;
            bulk_g2s(snib, pk.gu_nib + row0 * nb * 16, GU_UNIT_ROWS * nb * 16, bar);
            bulk_g2s(sscl, pk.gu_scl + row0 * nb, GU_UNIT_ROWS * nb * 2, bar);
        }
        for (int i = 0; i < nt; ++i) {
            const int t = __ldg(plan.order + p0 + c0 + i) / used;
            bulk_g2s(stok + i * xrb, xrec + (size_t)t * xrb, xrb, bar);
        }
    };
    RVC_MARK(2, 1);
    if (tid == 0) stage(0, &bar_w, true);
    if (!mbar_wait(&bar_w, 0, status)) return;
    RVC_MARK(2, 2);

    const int grp = lane >> 3, l8 = lane & 7, b0 = l8 * NB8;
    for (int c0 = 0, chunk = 0; c0 < n_e; c0 += GU_TOK, ++chunk) {
        const int nt = min(GU_TOK, n_e - c0);
        if (chunk > 0 && !mbar_wait(&bar_t, (chunk - 1) & 1, status)) return;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
            const int r = pass * 32 + warp * 4 + grp;  // packed row within the unit
            const uint8_t *nrow = snib + (size_t)r * nb * 16;
            const uint16_t *srow = sscl + r * nb;
            float term[GU_TOK][NB8];
#pragma unroll
            for (int k = 0; k < NB8; ++k) {
                const int b = b0 + k;
                const uint4 nib = *reinterpret_cast<const uint4 *>(nrow + b * 16);
                const float dw = f16_bits_to_f32(srow[b]);
#pragma unroll
                for (int i = 0; i < GU_TOK; ++i) {
                    term[i][k] = 0.0f;
                    if (i < nt) {
                        const Q8Rec xr{stok + i * xrb, nb};
                        const int sumi = q4q8_sumi(nib, xr.qa(b), xr.qb(b), xr.s(b));
                        term[i][k] = __fmul_rn((float)sumi, __fmul_rn(dw, xr.d(b)));
                    }
                }
            }
            float acc[GU_TOK];
#pragma unroll
            for (int i = 0; i < GU_TOK; ++i) acc[i] = 0.0f;
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                if (l8 == l) {
#pragma unroll
                    for (int i = 0; i < GU_TOK; ++i)
                        if (i < nt) {
#pragma unroll
                            for (int k = 0; k < NB8; ++k) acc[i] = __fadd_rn(acc[i], term[i][k]);
                        }
                }
#pragma unroll
                for (int i = 0; i < GU_TOK; ++i)
                    if (i < nt) acc[i] = __shfl_sync(0xffffffffu, acc[i], (lane & ~7) | l);
            }
            if (l8 == 0) {
                const int col = warp * 4 + grp;
#pragma unroll
                for (int i = 0; i < GU_TOK; ++i) {
                    if (i < nt) {
                        if (pass == 0)
                            sg[i][col] = acc[i];
                        else
                            su[i][col] = acc[i];
                    }
                }
            }
        }
        __syncthreads();  // every warp is done with this chunk's token records
        RVC_MARK(2, 3);
        if (tid == 0 && c0 + GU_TOK < n_e) stage(c0 + GU_TOK, &bar_t, false);
        // h = gelu(gate) * up for the 32 columns, then Q8_0 of the block (warp i: token i).
        if (warp < nt) {
            const float hv = __fmul_rn(gelu_tanh(sg[warp][lane]), su[warp][lane]);
            uint16_t dbits;
            int qsum;
            const int8_t qv = quant_q8_lane(hv, &dbits, &qsum);
            const size_t k = (size_t)(p0 + c0 + warp);  // plan position of this pair
            q8rec_store(hrec + k * hrb, nbh, q, lane, qv, dbits, qsum);
        }
        __syncthreads();
    }
    RVC_MARK(2, 4);
}

// ------------------------------------------------------------ down + combine
// Down projection + slot-order combine for up to DN_MAX_PAIRS pairs. grid: n_embd / DN_ROWS
// CTAs; block 256. Each CTA owns DN_ROWS output rows across every active expert, so the
// weighted combine of a token's `used` experts happens in shared memory in the reference's
// slot order. All h records (one per pair) are staged once; the row tiles of DN_BATCH experts
// at a time are staged into one of `nbuf` buffers (with 2, the next batch loads while this one
// computes); every thread runs whole (row, pair) dots, block terms added in block order as the
// scalar reference does (expert_kernel.rs:147-161).
constexpr int DN_ROWS = 16;
constexpr int DN_BATCH = 8;
constexpr int DN_MAX_PAIRS = 64;

__host__ __device__ inline int dn_stage_bytes(int nbh) { return (DN_ROWS * nbh * 18 + 127) & ~127; }

__host__ __device__ inline size_t dn_smem_bytes(int nbh, int nbuf, int pairs) {
    return (size_t)nbuf * DN_BATCH * dn_stage_bytes(nbh) + (size_t)pairs * q8rec_bytes(nbh) +
           (size_t)pairs * DN_ROWS * 4;
}

__global__ void __launch_bounds__(256) k_down_combine_decode(PackedView pk, int n_embd, int ff,
                                                             const uint8_t *__restrict__ hrec, PlanView plan,
                                                             const int32_t *__restrict__ ids,
                                                             const int32_t *__restrict__ ids_check,
                                                             const float *__restrict__ wts,
                                                             const float *__restrict__ down_scale, int n_tok, int used,
                                                             int nbuf, float *__restrict__ out, int *status) {
    RVC_MARK(3, 0);
    const int nbh = ff / QK;
    const int hrb = q8rec_bytes(nbh);
    const int r0 = blockIdx.x * DN_ROWS;
    const int n_act = __ldg(plan.n_active);
    const int pairs = n_tok * used;
    const uint32_t nib_bytes = DN_ROWS * nbh * 16, scl_bytes = DN_ROWS * nbh * 2;
    const int stage_bytes = dn_stage_bytes(nbh);

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *sh = smem + (size_t)nbuf * DN_BATCH * stage_bytes;       // [pairs] h records
    float *ysm = reinterpret_cast<float *>(sh + (size_t)pairs * hrb);  // [pairs][DN_ROWS]
    __shared__ uint64_t bars[2 * DN_BATCH], bar_h;
    __shared__ int s_pre[DN_BATCH + 1], s_off[DN_BATCH];
    const int tid = threadIdx.x;

    if (tid == 0) {
        for (int s = 0; s < 2 * DN_BATCH; ++s) mbar_init(&bars[s], 1);
        mbar_init(&bar_h, 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int n_batches = (n_act + DN_BATCH - 1) / DN_BATCH;
    auto issue = [&](int j) {  // thread s < DN_BATCH issues expert slot s of batch j
        const int a = j * DN_BATCH + tid;
        if (j < n_batches && tid < DN_BATCH && a < n_act) {
            const int slot = (j % nbuf) * DN_BATCH + tid;
            const int e = __ldg(plan.active + a);
            uint8_t *dst = smem + (size_t)slot * stage_bytes;
            const size_t row0 = (size_t)e * n_embd + r0;
            mbar_arrive_expect_tx(&bars[slot], nib_bytes + scl_bytes);
            bulk_g2s(dst, pk.dn_nib + row0 * nbh * 16, nib_bytes, &bars[slot]);
            bulk_g2s(dst + nib_bytes, pk.dn_scl + row0 * nbh, scl_bytes, &bars[slot]);
        }
    };
    issue(0);
    if (nbuf > 1) issue(1);
    if (tid == DN_BATCH) {
        mbar_arrive_expect_tx(&bar_h, pairs * hrb);
        bulk_g2s(sh, hrec, pairs * hrb, &bar_h);
    }
    bool ok = mbar_wait(&bar_h, 0, status);
    for (int j = 0; j < n_batches; ++j) {
        const int cnt = min(DN_BATCH, n_act - j * DN_BATCH);
        const int buf = j % nbuf;
        if (tid == 0) {
            int run = 0;
            for (int s = 0; s < cnt; ++s) {
                const int e = __ldg(plan.active + j * DN_BATCH + s);
                s_off[s] = __ldg(plan.offsets + e);
                s_pre[s] = run;
                run += __ldg(plan.counts + e);
            }
            s_pre[cnt] = run;
        }
        for (int s = 0; s < cnt; ++s) ok &= mbar_wait(&bars[buf * DN_BATCH + s], (j / nbuf) & 1, status);
        if (__syncthreads_or(!ok)) return;
        if (j == 0) RVC_MARK(3, 1);
        const int items = DN_ROWS * s_pre[cnt];
        for (int it = tid; it < items; it += blockDim.x) {
            const int pr = it / DN_ROWS, rr = it % DN_ROWS;  // pair within the batch, row
            int s = 0;
            while (pr >= s_pre[s + 1]) ++s;
            const int k = s_off[s] + pr - s_pre[s];  // plan position
            const uint8_t *stg = smem + (size_t)(buf * DN_BATCH + s) * stage_bytes;
            const uint8_t *snib = stg + (size_t)rr * nbh * 16;
            const uint16_t *sscl = reinterpret_cast<const uint16_t *>(stg + nib_bytes) + rr * nbh;
            const Q8Rec hr{sh + (size_t)k * hrb, nbh};
            float acc = 0.0f;
            for (int b = 0; b < nbh; ++b) {
                const uint4 nib = *reinterpret_cast<const uint4 *>(snib + b * 16);
                const int sumi = q4q8_sumi(nib, hr.qa(b), hr.qb(b), hr.s(b));
                acc = __fadd_rn(acc, __fmul_rn((float)sumi, __fmul_rn(f16_bits_to_f32(sscl[b]), hr.d(b))));
            }
            ysm[k * DN_ROWS + rr] = acc;
        }
        __syncthreads();
        issue(j + nbuf);
    }
    __syncthreads();
    RVC_MARK(3, 2);
    // slot-order combine (exec.rs:626-638): o = (y*ds)*w for j = 0, then o = o + (y*ds)*w
    for (int i = tid; i < n_tok * DN_ROWS; i += blockDim.x) {
        const int t = i / DN_ROWS, rr = i % DN_ROWS;
        float o = 0.0f;
        for (int j = 0; j < used; ++j) {
            const int p = t * used + j;
            const int e = __ldg(ids + p);
            // the exact-order router must agree with the ids the GEMVs were run with
            if (ids_check && rr == 0 && blockIdx.x == 0 && __ldg(ids_check + p) != e)
                set_status(status, STATUS_ROUTE_MISMATCH);
            const float ds = down_scale ? __ldg(down_scale + e) : 1.0f;
            const int k = __ldg(plan.pos_of + p);
            const float v = __fmul_rn(__fmul_rn(ysm[(size_t)k * DN_ROWS + rr], ds), __ldg(wts + p));
            o = j == 0 ? v : __fadd_rn(o, v);
        }
        out[(size_t)t * n_embd + r0 + rr] = o;
    }
    RVC_MARK(3, 3);
}

// -------------------------------------------------- down (expert-major) + combine
// For more pairs than the fused kernel holds: CTA (row tile of DE_ROWS rows, active expert a)
// computes y for every pair of that expert on its rows and writes y [pairs][n_embd] in plan
// order; k_combine then forms the slot-order weighted sums. grid (n_embd / DE_ROWS, max active).
constexpr int DE_ROWS = 128;
constexpr int DE_CHUNK = 64;  // h records staged per chunk

__host__ __device__ inline size_t de_smem_bytes(int nbh) {
    return (size_t)DE_ROWS * nbh * 18 + (size_t)DE_CHUNK * q8rec_bytes(nbh);
}

__global__ void __launch_bounds__(256) k_down_expert(PackedView pk, int n_embd, int ff,
                                                     const uint8_t *__restrict__ hrec, PlanView plan,
                                                     float *__restrict__ y, int *status) {
    const int nbh = ff / QK;
    const int hrb = q8rec_bytes(nbh);
    const int r0 = blockIdx.x * DE_ROWS;
    const int a = blockIdx.y;
    if (a >= __ldg(plan.n_active)) return;
    const int e = __ldg(plan.active + a);
    const int p0 = __ldg(plan.offsets + e), n_e = __ldg(plan.counts + e);
    const uint32_t nib_bytes = DE_ROWS * nbh * 16, scl_bytes = DE_ROWS * nbh * 2;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *sh = smem + nib_bytes + scl_bytes;
    __shared__ uint64_t bar;
    const int tid = threadIdx.x;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    for (int c0 = 0, chunk = 0; c0 < n_e; c0 += DE_CHUNK, ++chunk) {
        const int np = min(DE_CHUNK, n_e - c0);
        if (tid == 0) {
            uint32_t bytes = np * hrb;
            if (chunk == 0) bytes += nib_bytes + scl_bytes;
            mbar_arrive_expect_tx(&bar, bytes);
            if (chunk == 0) {
                const size_t row0 = (size_t)e * n_embd + r0;
                bulk_g2s(smem, pk.dn_nib + row0 * nbh * 16, nib_bytes, &bar);
                bulk_g2s(smem + nib_bytes, pk.dn_scl + row0 * nbh, scl_bytes, &bar);
            }
            bulk_g2s(sh, hrec + (size_t)(p0 + c0) * hrb, np * hrb, &bar);
        }
        if (!mbar_wait(&bar, chunk & 1, status)) return;
        for (int it = tid; it < np * DE_ROWS; it += blockDim.x) {
            const int j = it / DE_ROWS, rr = it % DE_ROWS;
            const uint8_t *snib = smem + (size_t)rr * nbh * 16;
            const uint16_t *sscl = reinterpret_cast<const uint16_t *>(smem + nib_bytes) + rr * nbh;
            const Q8Rec hr{sh + (size_t)j * hrb, nbh};
            float acc = 0.0f;
            for (int b = 0; b < nbh; ++b) {
                const uint4 nib = *reinterpret_cast<const uint4 *>(snib + b * 16);
                const int sumi = q4q8_sumi(nib, hr.qa(b), hr.qb(b), hr.s(b));
                acc = __fadd_rn(acc, __fmul_rn((float)sumi, __fmul_rn(f16_bits_to_f32(sscl[b]), hr.d(b))));
            }
            y[(size_t)(p0 + c0 + j) * n_embd + r0 + rr] = acc;
        }
        __syncthreads();
    }
}

// out[t][r] = slot-order sum of (y[pos_of[p]][r] * down_scale[e]) * w[p] (exec.rs:626-638).
// grid (ceil(n_embd / 256), n_tok); block 256.
__global__ void __launch_bounds__(256) k_combine(const float *__restrict__ y, const int32_t *__restrict__ pos_of,
                                                 const int32_t *__restrict__ ids,
                                                 const int32_t *__restrict__ ids_check,
                                                 const float *__restrict__ wts, const float *__restrict__ down_scale,
                                                 int used, int n_embd, float *__restrict__ out, int *status) {
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_embd) return;
    float o = 0.0f;
    for (int j = 0; j < used; ++j) {
        const int p = t * used + j;
        const int e = __ldg(ids + p);
        if (ids_check && r == 0 && __ldg(ids_check + p) != e) set_status(status, STATUS_ROUTE_MISMATCH);
        const float ds = down_scale ? __ldg(down_scale + e) : 1.0f;
        const float v =
            __fmul_rn(__fmul_rn(__ldg(y + (size_t)__ldg(pos_of + p) * n_embd + r), ds), __ldg(wts + p));
        o = j == 0 ? v : __fadd_rn(o, v);
    }
    out[(size_t)t * n_embd + r] = o;
}

}  // namespace rvc
