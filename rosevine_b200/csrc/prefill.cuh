// prefill.cuh - the MoE layer for prefill batches (and the expert-parallel layer's expert step):
// a grouped expert GEMM fed by TMA tensor copies, sm_100a.
//
// Replaces the reference's per-expert device loop (runtime/src/hip_exec.rs:820-843) for batches
// of more than 16 tokens and computes what its CPU-experts Q8_0 path computes
// (runtime/src/exec.rs:572-640, expert_pool.rs:282-355, expert_kernel.rs:147-161):
//
//   k_plan        (router.cuh) expert groups in plan order, each group starting at a multiple
//                 of 4 positions, and the list of (expert, 128-position) tiles.
//   k_pf_quant    Q8_0 of x once per token, scattered to the token's plan positions, with each
//                 block's (scale, offset) pair block-major (the layout the GEMM copies).
//   k_pf_gemm_ms<GU> per (expert, 128 packed gate/up rows, 128 positions) tile and 32-column
//                 block b: the exact int32 block dots D_b (mma.sync m16n8k32, u8 nibbles x s8
//                 quants), then acc = acc + D_b * (dw_b * dx_b) per (row, position) in block
//                 order, each operation rounded as the scalar reference does; then
//                 h = gelu(gate) * up and its Q8_0 records.
//   k_pf_gemm_ms<DN> the same over the down rows and the h records: y per (position, row).
//   k_pf_combine  out[t] = slot-order sum of (y * down_scale) * w (exec.rs:626-638).
//
// Exactness. The nibbles n (0..15) multiply as unsigned bytes; the activation block's offset
// -(1.5 * 2^23 + 8 sum(q)) turns C + sum n q (C the accumulator's starting bits) into
// sum (n - 8) q exactly, so D_b equals the reference's integer block dot and the float
// operations that follow are the reference's, in its order (f32x2 instructions, two positions
// at a time, never contracted into an fma: see f2_prod).
//
// Why register accumulators. Scaling is per 32-column block, so every block's dots must reach
// the CUDA cores: 4 f32 operations per (row, position, block) against 64 int8 multiply-adds.
// The CUDA cores bound this GEMM (about 13% of the int8 tensor peak at best). With tcgen05 the
// dots sit in tensor memory and each block needs a tcgen05.ld (and a store of C) by the
// epilogue; on B200 a tcgen05.ld or .st waits for every MMA in flight in the CTA (measured:
// 140-330 ns per load under a stream of MMAs), which serialises the MMAs with the epilogue.
// A tcgen05 version of this pipeline (TMA, tensor-memory accumulators, warp-specialised
// unpack / MMA / epilogue) ran the 2048-token layer in 3.1 ms; this one runs it in 1.5 ms.
//
// Operands. Weights stay Q4_0 in HBM (the packed nibble and scale planes of pack.cuh); per stage
// of 8 blocks one TMA tensor copy brings a tile's 128 rows of nibbles (16 KB), one its 128
// positions' quants in K-halves x positions x 16 B order, one their (scale, offset) pairs.
#pragma once
#include "common.cuh"
#include "pack.cuh"

#include <cuda.h>

namespace rvc {

constexpr int PF_M = 128;  // weight rows per tile
constexpr int PF_N = 128;  // plan positions per tile
constexpr int PF_KB = 8;   // K-blocks per stage


// Every block's MMA accumulates onto the bits of 1.5 * 2^23: the int32 sum C + D of a block dot
// D (|D| < 2^22) then reads as the float 1.5 * 2^23 + D exactly, and one exact addition gives
// (float)D.
constexpr uint32_t PF_MAGIC_BITS = 0x4B400000u;
constexpr float PF_MAGIC = 12582912.0f;
// An activation block with quants q, scale d and sum(q) = qs enters the GEMM as the pair
// (d, -(C + 8 qs)): the MMA of the unsigned nibbles n gives C + sum n q, and adding the offset
// leaves sum (n - 8) q exactly (all values integers below 2^24).
__device__ __forceinline__ float2 pf_scale_offset(float d, int qs) { return make_float2(d, -(PF_MAGIC + 8.0f * (float)qs)); }

// The (scale, offset) plane of activation blocks (x: xso, h: hso) is block-major, 2 * ppad f32
// per block, each position pair (2k, 2k + 1) stored as [scale 2k, scale 2k + 1, offset 2k,
// offset 2k + 1]: the GEMM then loads a pair's two scales and its two offsets as ready f32x2
// operands (one 16-byte load, no register shuffling). ppad is even.
__device__ __forceinline__ void pf_store_so(float2 *plane, int ppad, int b, int k, float2 so) {
    float *p = reinterpret_cast<float *>(plane) + (size_t)b * 2 * ppad + 4 * (k >> 1) + (k & 1);
    p[0] = so.x;
    p[2] = so.y;
}

// ------------------------------------------------------------------ tcgen05 primitives
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {  // one full warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // one full warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle ("interleave"): 8-row x 16-byte core
// matrices; lbo = bytes between the two 16-byte K halves of a 32-byte K step, sbo = bytes
// between consecutive 8-row groups (descriptor format: start >> 4 at bits 0-13, lbo >> 4 at
// 16-29, sbo >> 4 at 32-45, version 1 at 46-47, layout type 0 at 61-63).
__device__ __forceinline__ uint64_t umma_desc(const void *smem_ptr, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_u32(smem_ptr);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), A unsigned or signed int8
// (bits 7-9 = 0 or 1), B signed (bits 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool a_signed = true) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

// D[tmem] = A * B (+ D if accumulate), one thread.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from tensor memory; tcgen05.wait::ld before use.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The wait with the loaded registers as operands: the compiler cannot move their uses above it
// (tcgen05.ld writes them asynchronously; plain register uses are not ordered by a memory clobber).
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&v)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                   "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]),
                   "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                   "+r"(v[30]), "+r"(v[31])
                 :
                 : "memory");
}

// 2-D TMA tensor copy global -> shared, completion on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// 3-D TMA tensor copy global -> shared, completion on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Signed int8 (n - 8) of four nibble values n in 0..15 (one per byte): adding 0x78 to each byte
// through (n | 0x80) - 8 cannot borrow across bytes; the xor restores the sign bit.
__device__ __forceinline__ uint32_t nib_to_s8(uint32_t v) { return ((v | 0x80808080u) - 0x08080808u) ^ 0x80808080u; }

// ------------------------------------------------------------------ MMA check (debug ABI)
// One tile through the same layouts and tensor-memory reads as k_pf_gemm: A [128 rows][32]
// and B [n rows][32] int8 (row-major in global), D [128][n] int32 = A . B^T. Thread r < 128
// places row r; warp w < 4 reads tensor-memory lanes 32 w .. 32 w + 31. n = 16 .. 128, step 16.
__global__ void __launch_bounds__(128) k_debug_mma_i8(const int8_t *__restrict__ A, const int8_t *__restrict__ B,
                                                      int n, int32_t *__restrict__ D, int *status) {
    __shared__ __align__(1024) uint8_t sa[2 * PF_M * 16];
    __shared__ __align__(1024) uint8_t sb[2 * PF_N * 16];
    __shared__ uint64_t bar;
    __shared__ uint32_t taddr_s;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (warp == 0) {
        tmem_alloc(&taddr_s, 128);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    // K halves k = 0, 1 of row r at k * (rows * 16) + r * 16 (core matrices of 8 rows)
    for (int k = 0; k < 2; ++k) {
        *reinterpret_cast<int4 *>(sa + k * PF_M * 16 + tid * 16) = *reinterpret_cast<const int4 *>(A + tid * 32 + k * 16);
        if (tid < n)
            *reinterpret_cast<int4 *>(sb + k * PF_N * 16 + tid * 16) =
                *reinterpret_cast<const int4 *>(B + tid * 32 + k * 16);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = taddr_s;
    if (tid == 0) {
        mma_i8(taddr, umma_desc(sa, PF_M * 16, 128), umma_desc(sb, PF_N * 16, 128), idesc_i8(PF_M, n), false);
        mma_commit(&bar);
    }
    const bool ok = fd_mbar_wait(&bar, 0, status);
    tc_fence_after();
    if (ok) {
        for (int c0 = 0; c0 < n; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(taddr + ((uint32_t)(32 * warp) << 16) + c0, v);
            tmem_ld_wait(v);
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (c0 + i < n) D[(size_t)tid * n + c0 + i] = (int32_t)v[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, 128);
}

// ------------------------------------------------------------------ quantise + scatter
// Q8_0 of x, once per token, written into the records of the token's `used` plan positions
// pos_of[t used + j], with each block's (scale, offset) pair in the block-major plane xso the
// GEMM's scale tiles come from. Four lanes per block: lane l of warp w takes values
// 8 (l & 3) .. + 7 of block 8 w' + (l >> 2) of its token (one 16-byte load for bf16, two for
// f32; rows are 16-byte aligned, as the entry points require), so a warp quantises 8 blocks at
// once, each reduction taking two shuffles within the group of four lanes, and writes a plan
// position's 8 quants per lane with one 8-byte store. Per value the arithmetic is
// quant_q8_lane's (ops.rs:95-105); a block's amax and integer sum do not depend on the
// reduction order.
template <typename XT>
__global__ void __launch_bounds__(256) k_pf_quant(const XT *__restrict__ x, int n_embd, int n_tok, int used,
                                                  const int32_t *__restrict__ pos_of, uint8_t *__restrict__ xperm,
                                                  float2 *__restrict__ xso, int ppad) {
    const int nb = n_embd / QK, xrb = q8rec_bytes(nb);
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
    uint32_t qw[2] = {0u, 0u};
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float r = roundf(__fmul_rn(v[k], id));
        const int q = r != r ? 0 : (r > 127.0f ? 127 : (r < -128.0f ? -128 : (int)r));
        s += q;
        qw[k >> 2] |= (uint32_t)(uint8_t)(int8_t)q << (8 * (k & 3));
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    const float df = f16_bits_to_f32(f32_to_f16_bits(d));
    const float2 so = pf_scale_offset(df, s);
    const int my_pos = lane < used ? __ldg(pos_of + (size_t)t * used + lane) : 0;
    for (int j = 0; j < used; ++j) {
        const int k = __shfl_sync(0xffffffffu, my_pos, j);
        if (in) {
            uint8_t *rec = xperm + (size_t)k * xrb;
            *reinterpret_cast<uint2 *>(rec + b * 32 + part * 8) = make_uint2(qw[0], qw[1]);
            if (part == 0) {
                reinterpret_cast<float *>(rec + nb * 32)[b] = df;
                reinterpret_cast<int *>(rec + nb * 36)[b] = s;
                pf_store_so(xso, ppad, b, k, so);
            }
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

// Received rows to plan positions: warp task (row r, block b) copies the block into the records
// of the row's occupied slots' plan positions, with its (scale, offset) pair.
__global__ void __launch_bounds__(256) k_ep_scatter(const uint8_t *__restrict__ rows, int nb, int n_rows, int used,
                                                    const int32_t *__restrict__ slot_e,
                                                    const int32_t *__restrict__ pos_of, uint8_t *__restrict__ xperm,
                                                    float2 *__restrict__ xso, int ppad) {
    const int xrb = q8rec_bytes(nb), rb = ep_row_bytes(nb, used);
    const int lane = threadIdx.x & 31;
    const long long total = (long long)n_rows * nb;
    for (long long i = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); i < total; i += (long long)gridDim.x * 8) {
        const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
        const uint8_t *src = rows + (size_t)r * rb;
        const uint8_t q = src[b * 32 + lane];
        const float d = reinterpret_cast<const float *>(src + nb * 32)[b];
        const int qs = reinterpret_cast<const int *>(src + nb * 36)[b];
        for (int j = 0; j < used; ++j) {
            const int p = r * used + j;
            if (__ldg(slot_e + p) < 0) continue;
            const int k = __ldg(pos_of + p);
            uint8_t *dst = xperm + (size_t)k * xrb;
            dst[b * 32 + lane] = q;
            if (lane == 0) {
                reinterpret_cast<float *>(dst + nb * 32)[b] = d;
                reinterpret_cast<int *>(dst + nb * 36)[b] = qs;
                pf_store_so(xso, ppad, b, k, pf_scale_offset(d, qs));
            }
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

// ------------------------------------------------------------------ grouped GEMM
struct PfArgs {
    const int2 *tiles;    // per tile: (expert | tokens << 8, first plan position), from k_plan
    const int *n_tiles;
    int rows_per_expert;  // 2 ff (gate/up) or n_embd (down)
    int nblk;             // K blocks (n_embd / 32 or ff / 32)
    const uint8_t *nib;   // weight nibbles [E][rows][nblk][16] (for the L2 prefetch; copies go through the map)
    const uint16_t *scl;  // weight scales [E][rows][nblk] (f16 bits)
    int nh;               // (gate/up) h blocks per pair (ff / 32): the h record geometry
    uint8_t *hrec;        // (gate/up) out: h records by plan position
    float2 *hso;          // (gate/up) out: h block (scale, offset) pairs, block-major [nh][ppad]
    int ppad;
    float *y;             // (down) out: [positions][n_embd]
    int n_embd;
    int *status;
    uint64_t negzero2;    // two f32 -0 (0x80000000 each): see f2_prod
};

constexpr int PF_GU = 0, PF_DN = 1;

// A stage of a tile in shared memory: the weight nibbles (128 rows x 8 blocks x 16 B), the
// activation quants (8 blocks x 2 halves x 128 positions x 16 B) and the positions' (scale,
// offset) pairs (8 blocks x 128 positions x 2 f32).
constexpr int PF_B_BYTES = PF_KB * 2 * PF_N * 16;  // 32 KB
constexpr int PF_NIB_BYTES = PF_M * PF_KB * 16;    // 16 KB
constexpr int PF_DX_BYTES = PF_N * PF_KB * 8;      // 8 KB: (scale, offset) per position and block

// Bounded mbarrier wait, inline (a call would make the caller save its live accumulators).
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, int *status) {
    for (long long i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    set_status(status, STATUS_TIMEOUT);
    return false;
}

// f32x2 multiply and add, each lane rounded to nearest even. A product that feeds an add comes
// from f2_prod, an fma whose addend is -0 held in a register loaded from the kernel's
// arguments: that is the rounded product (sign of zero included). The compiler contracts an
// f32x2 mul followed by an add into one fma, rounding once, for the intrinsics and for inline
// mul.rn/add.rn.f32x2 alike, and turns an fma with a literal -0 addend back into a mul (both
// measured on B200); an fma whose addend it cannot see, followed by an add, stays two
// roundings.
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x)),
          "l"(((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x)));
    return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}
__device__ __forceinline__ float2 f2_prod(float2 a, float2 b, uint64_t negzero2) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x)),
          "l"(((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x)), "l"(negzero2));
    return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}
// The same on f32x2 values kept packed in 64-bit registers (low half: the first lane), which
// the GEMM's inner loop uses so that no operand needs repacking.
__device__ __forceinline__ uint64_t f2x_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2x_prod(uint64_t a, uint64_t b, uint64_t negzero2) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(negzero2));
    return r;
}
__device__ __forceinline__ uint64_t f2x_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_splat(float v) {
    const uint64_t u = __float_as_uint(v);
    return (u << 32) | u;
}
__device__ __forceinline__ float f2x_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2x_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x)),
          "l"(((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x)));
    return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}

__device__ __forceinline__ void named_sync_n(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// ------------------------------------------------------------------ grouped GEMM, register accumulators
// The same tiles, with the block dots from mma.sync.m16n8k32 (u8 nibbles x s8 quants, s32
// accumulators in registers): each of 16 warps multiplies, scales and accumulates its own
// 32 rows x 32 positions, so a block's integers never leave the registers that receive them.
// A fragments come straight from the nibble tile: the 32-bit word at byte 4 (lane % 4) of a row's
// block holds elements 4 (lane % 4) .. + 3 in its low nibbles and the same + 16 in its high
// nibbles, which are exactly the a0 / a2 (a1 / a3 for row + 8) registers of the fragment.
// Stages of 8 blocks arrive by TMA (nibbles, quants, (scale, offset) pairs); each warp keeps its
// own rows' weight scales a stage ahead in its slice of shared memory, and runs through the
// stages on its own: per stage it waits for the copies (full) and releases the buffers (empty);
// thread 0 refills a slot once every warp holding tokens is past it. Warps whose 32 positions
// hold no token leave at once.
constexpr int PM_WARPS = 16;  // 4 row groups of 32 x 4 position groups of 32
constexpr int PM_THREADS = PM_WARPS * 32;
constexpr int PM_STAGES = 3;
constexpr int PM_OFF_B = PF_NIB_BYTES;
constexpr int PM_OFF_SO = PM_OFF_B + PF_B_BYTES;
constexpr int PM_STAGE_BYTES = PM_OFF_SO + PF_DX_BYTES;  // 56 KB
constexpr int PM_DW_WARP = 2 * PF_KB * 32;  // f32 per warp: [2 stages][8 blocks][8 g][4: row 16 i + 8 h + g]
constexpr int PM_OFF_DW = PM_STAGES * PM_STAGE_BYTES;
constexpr int PM_SMEM_BYTES = PM_OFF_DW + PM_WARPS * PM_DW_WARP * 4 + 1024;
constexpr int PM_H_PITCH = 33;  // gate/up staging [unit][gate|up][position][33]
static_assert(PM_SMEM_BYTES <= 227 * 1024, "shared memory of k_pf_gemm_ms");
static_assert(2 * 2 * PF_N * PM_H_PITCH * 4 <= PM_STAGES * PM_STAGE_BYTES, "gate/up staging");

// d = a . b + (c, c, c, c): 16 x 8 s32 from 16 x 32 u8 (row-major) and 32 x 8 s8 (column-major).
__device__ __forceinline__ void mma_u8s8(uint32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, uint32_t c) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}

// Four 8 x 8 b16 matrices from shared memory: lane L supplies the address of row L & 7 of
// matrix L >> 3 (16 bytes); each lane receives, per matrix, the 4 bytes at columns 4 (L & 3) ..
// of row L >> 2, the layout of an mma.sync m16n8k32 int8 operand fragment.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

template <bool B>
struct BoolTag {
    static constexpr bool value = B;
};

// The same MMA with the accumulator fragment returned as two f32x2-ready 64-bit values: rows g and
// g + 8, each (position 2 tq, position 2 tq + 1) in (low, high) halves.
__device__ __forceinline__ void mma_u8s8_x2(uint64_t (&d)[2], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1, uint32_t c) {
    asm("{\n\t.reg .b32 r0, r1, r2, r3;\n\t"
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {r0, r1, r2, r3}, {%2, %3, %4, %5}, {%6, %7}, "
        "{%8, %8, %8, %8};\n\t"
        "mov.b64 %0, {r0, r1};\n\tmov.b64 %1, {r2, r3};\n\t}"
        : "=l"(d[0]), "=l"(d[1])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}

template <int MODE>
__global__ void __launch_bounds__(PM_THREADS, 1) k_pf_gemm_ms(const __grid_constant__ CUtensorMap map_nib,
                                                              const __grid_constant__ CUtensorMap map_act,
                                                              const __grid_constant__ CUtensorMap map_so, PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, by an offset from the shared array itself (pointer arithmetic keeps
    // the compiler's knowledge that these are shared addresses: 32-bit LDS, not generic loads)
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t full[PM_STAGES], empty[PM_STAGES];
    if ((int)blockIdx.y >= __ldg(a.n_tiles)) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.nblk, rows = a.rows_per_expert;
    const int row0 = blockIdx.x * PF_M;
    const int2 td = __ldg(a.tiles + blockIdx.y);
    const int e = td.x & 0xFF, nt = td.x >> 8, p0 = td.y;
    const int nst = (nblk + PF_KB - 1) / PF_KB;
    const int wrow0 = e * rows + row0;
    const int n_active = 4 * min(4, (nt + 31) >> 5);  // warps 0 .. n_active - 1 hold tokens
    auto issue = [&](int st) {  // thread 0
        const int s = st % PM_STAGES;
        uint8_t *base = smem + s * PM_STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], PM_STAGE_BYTES);
        tma_load_3d(base, &map_nib, 0, st * PF_KB, wrow0, &full[s]);              // [128 rows][8 blocks][16 B]
        tma_load_3d(base + PM_OFF_B, &map_act, 0, p0, 2 * st * PF_KB, &full[s]);  // [16 halves][128 positions][16 B]
        tma_load_2d(base + PM_OFF_SO, &map_so, 2 * p0, st * PF_KB, &full[s]);     // [8 blocks][128 positions][2] f32
    };
    if (tid == 0) {
        for (int s = 0; s < PM_STAGES; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], n_active);
        fence_barrier_init();
        bulk_prefetch_l2(a.nib + (size_t)wrow0 * nblk * 16, (uint32_t)(PF_M * nblk * 16));
        for (int st = 0; st < min(nst, PM_STAGES); ++st) issue(st);
    }
    __syncthreads();
    if (warp >= n_active) return;

    const int wr = warp & 3, wc = warp >> 2;  // rows 32 wr .., positions 32 wc ..
    const int g = lane >> 2, tq = lane & 3;
    const int nj = min(4, (nt - 32 * wc + 7) >> 3);  // 8-position fragments holding tokens
    // this lane's row address for the ldmatrix loads of A (nibble rows) and B (position rows)
    const uint32_t a_row = (uint32_t)(32 * wr + lane) * (PF_KB * 16);
    const uint32_t b_lane = (uint32_t)((lane >> 3) & 1) * (PF_N * 16) + (uint32_t)(32 * wc + 8 * (lane >> 4) + (lane & 7)) * 16;
    // the warp's weight scales: lane l loads row 32 wr + l's 8 scales of a stage one stage ahead
    // (four f16 pairs) and stores them as f32 in the warp's own slice [2][8 blocks][8][4], where
    // row l = 16 i + 8 h + g sits at [g][2 i + h]: one 16-byte load gives a lane its four rows
    const uint32_t *srow = reinterpret_cast<const uint32_t *>(a.scl + (size_t)(wrow0 + 32 * wr + lane) * nblk);
    float *const sdw = reinterpret_cast<float *>(smem + PM_OFF_DW) + warp * PM_DW_WARP;
    uint32_t wn[4];
    auto ld_dw = [&](int st) {
#pragma unroll
        for (int k = 0; k < 4; ++k) wn[k] = st * PF_KB + 2 * k < nblk ? __ldg(srow + (st * PF_KB) / 2 + k) : 0u;
    };
    auto st_dw = [&](int st) {
        float *d = sdw + (st & 1) * (PF_KB * 32) + (lane & 7) * 4 + (lane >> 4) * 2 + ((lane >> 3) & 1);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            d[(2 * k) * 32] = f16_bits_to_f32((uint16_t)(wn[k] & 0xFFFFu));
            d[(2 * k + 1) * 32] = f16_bits_to_f32((uint16_t)(wn[k] >> 16));
        }
    };
    ld_dw(0);
    st_dw(0);
    __syncwarp();
    // [row fragment][position fragment][rows g, g + 8], f32x2 of positions 2 tq, 2 tq + 1 (low, high)
    uint64_t acc[2][4][2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj][0] = acc[i][jj][1] = 0ull;
    const uint64_t nz2 = a.negzero2;
    bool ok = true;
    for (int st = 0; st < nst && ok; ++st) {
        const int s = st % PM_STAGES;
        if (st + 1 < nst) ld_dw(st + 1);  // lands during this stage
        if (lane == 0) ok = pf_wait(&full[s], (uint32_t)(st / PM_STAGES) & 1u, a.status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) {
            const uint8_t *sN = smem + s * PM_STAGE_BYTES;
            const ulonglong2 *sSO = reinterpret_cast<const ulonglong2 *>(sN + PM_OFF_SO);
            const uint32_t sN32 = smem_u32(sN), sB32 = sN32 + PM_OFF_B;
            const float4 *dwp = reinterpret_cast<const float4 *>(sdw + (st & 1) * (PF_KB * 32)) + g;
            const int kn = min(PF_KB, nblk - st * PF_KB);
            // FULL: all four position fragments hold tokens (every warp of a full tile), so the
            // block loop runs without per-fragment branches (nor the convergence points
            // mma.sync needs after them)
            auto blocks = [&](auto full_tag) {
            constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll 2
            for (int jb = 0; jb < kn; ++jb) {
                const float4 w4 = dwp[jb * 8];  // rows g, g + 8, 16 + g, 24 + g of the warp
                const uint64_t dw[2][2] = {{f2_splat(w4.x), f2_splat(w4.y)}, {f2_splat(w4.z), f2_splat(w4.w)}};
                // A: one ldmatrix gives each lane 4 nibble bytes of rows g, g + 8, 16 + g, 24 + g
                // of the warp (lane L addresses row 8 (L >> 3) + (L & 7), whose swizzle key is
                // L & 7), the byte columns 4 tq .. of their block-jb chunks. A stage of 8 blocks
                // is one complete group, swizzled in the packed plane (nib_pos); a shorter last
                // stage is the row's unswizzled tail.
                uint32_t wq[4];
                ldsm_x4(sN32 + a_row + ((kn == PF_KB ? (jb ^ (lane & 7)) : jb) << 4), wq);
                uint32_t af[2][4];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint32_t w0 = wq[2 * i], w1 = wq[2 * i + 1];
                    af[i][0] = w0 & 0x0F0F0F0Fu, af[i][1] = w1 & 0x0F0F0F0Fu;
                    af[i][2] = (w0 >> 4) & 0x0F0F0F0Fu, af[i][3] = (w1 >> 4) & 0x0F0F0F0Fu;
                }
                // B: one ldmatrix per two position fragments: both K-halves of block jb for the
                // 8 positions of fragment jj and of jj + 1 (lane L addresses K-half 2 jb +
                // ((L >> 3) & 1), position 8 (L >> 4) + (L & 7) of the pair)
                uint32_t bq[2][4];
                ldsm_x4(sB32 + b_lane + jb * (2 * PF_N * 16), bq[0]);
                if (FULL || nj > 2) ldsm_x4(sB32 + b_lane + jb * (2 * PF_N * 16) + 16 * 16, bq[1]);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    if (FULL || jj < nj) {
                        const uint32_t b0 = bq[jj >> 1][2 * (jj & 1)], b1 = bq[jj >> 1][2 * (jj & 1) + 1];
                        // scales (x) and offsets (y) of positions 32 wc + 8 jj + 2 tq and + 1
                        const ulonglong2 so = sSO[(jb * PF_N + 32 * wc + 8 * jj + 2 * tq) >> 1];
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            uint64_t d[2];  // rows g, g + 8; each the f32x2 of positions 2 tq, 2 tq + 1
                            mma_u8s8_x2(d, af[i][0], af[i][1], af[i][2], af[i][3], b0, b1, PF_MAGIC_BITS);
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint64_t sc = f2x_mul(dw[i][h], so.x);
                                const uint64_t t = f2x_add(d[h], so.y);
                                acc[i][jj][h] = f2x_add(acc[i][jj][h], f2x_prod(t, sc, nz2));
                            }
                        }
                    }
                }
            }
            };
            if (nj == 4)
                blocks(BoolTag<true>{});
            else
                blocks(BoolTag<false>{});
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage's buffers
        if (st + 1 < nst) st_dw(st + 1);
        __syncwarp();
        // thread 0 refills the slot of the previous stage once every warp holding tokens is past it
        if (tid == 0 && st >= 1 && st - 1 + PM_STAGES < nst) {
            const int sp = st - 1;
            ok = ok && pf_wait(&empty[sp % PM_STAGES], (uint32_t)(sp / PM_STAGES) & 1u, a.status);
            if (ok) issue(sp + PM_STAGES);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (!ok) set_status(a.status, STATUS_TIMEOUT);
    // ------------------------------------------------ outputs
    if (MODE == PF_DN) {
        if (ok) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int row = row0 + 32 * wr + 16 * i + 8 * h + g, tok = 32 * wc + 8 * jj + 2 * tq;
                        if (tok < nt) a.y[(size_t)(p0 + tok) * a.n_embd + row] = f2x_lo(acc[i][jj][h]);
                        if (tok + 1 < nt) a.y[(size_t)(p0 + tok + 1) * a.n_embd + row] = f2x_hi(acc[i][jj][h]);
                    }
        }
    } else {
        // rows 32 wr .. + 31 of the tile are unit u = wr / 2, gate (wr even) or up, column
        // 16 i + 8 h + g. Staged as H[u][gate | up][position][33] in the (consumed) stage buffers;
        // then one warp per (position, unit): h = gelu(gate) * up over the unit's 32 columns,
        // quantised as one Q8_0 block (lane = column).
        // (the stage buffers are free once every warp holding tokens is past its last stage)
        float *H = reinterpret_cast<float *>(smem);
        const int u = wr >> 1, x = wr & 1;
        named_sync_n(6, n_active * 32);
        {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int c = 16 * i + 8 * h + g, tok = 32 * wc + 8 * jj + 2 * tq;
                        float *hp = H + ((size_t)(u * 2 + x) * PF_N + tok) * PM_H_PITCH + c;
                        hp[0] = f2x_lo(acc[i][jj][h]);
                        hp[PM_H_PITCH] = f2x_hi(acc[i][jj][h]);
                    }
        }
        named_sync_n(6, n_active * 32);
        if (ok) {
            const int hrb = q8rec_bytes(a.nh);
#pragma unroll 1
            for (int item = warp; item < 2 * nt; item += n_active) {
                const int uu = item & 1, tok = item >> 1;
                const float gv = H[((size_t)(uu * 2) * PF_N + tok) * PM_H_PITCH + lane];
                const float uv = H[((size_t)(uu * 2 + 1) * PF_N + tok) * PM_H_PITCH + lane];
                const float hv = __fmul_rn(gelu_tanh(gv), uv);
                uint16_t dbits;
                int qsum;
                const int8_t qv = quant_q8_lane(hv, &dbits, &qsum);
                const int q = (row0 >> 6) + uu;  // h block within the expert's ff columns
                q8rec_store(a.hrec + (size_t)(p0 + tok) * hrb, a.nh, q, lane, qv, dbits, qsum);
                if (lane == 0) pf_store_so(a.hso, a.ppad, q, p0 + tok, pf_scale_offset(f16_bits_to_f32(dbits), qsum));
            }
        }
    }
}

}  // namespace rvc
