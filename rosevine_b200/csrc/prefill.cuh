// prefill.cuh - the MoE layer for prefill batches: a grouped expert GEMM on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in tensor memory), sm_100a.
//
// Replaces the reference's per-expert device loop (runtime/src/hip_exec.rs:820-843) for batches
// above the decode kernels' 64 tokens and computes what its CPU-experts Q8_0 path computes
// (runtime/src/exec.rs:572-640, expert_pool.rs:282-355, expert_kernel.rs:147-161):
//
//   k_plan        (router.cuh) expert groups in plan order, each group starting at a multiple
//                 of 4 positions, and the list of (expert, 128-position) tiles.
//   k_pf_quant    Q8_0 of x once per token, scattered to the token's plan positions; the block
//                 scales also block-major (the layout the GEMM's scale tiles are copied from).
//   k_pf_gemm<GU> for each (expert, 128 packed gate/up rows, 128 positions) tile: per 32-column
//                 block b, two tcgen05.mma (M=128, N<=128, K=32, kind::i8) give the exact int32
//                 block dots D_b; the epilogue warps read D_b from tensor memory and accumulate
//                 acc = acc + D_b * (dw_b * dx_b) per (row, token) in block order, each operation
//                 rounded as the scalar reference does; then h = gelu(gate)*up and its Q8_0
//                 records.
//   k_pf_gemm<DN> the same over the down rows and the h records: y per (position, row).
//   k_pf_combine  out[t] = slot-order sum of (y * down_scale) * w (exec.rs:626-638).
//
// Operands. Weights stay Q4_0 in HBM (the packed nibble and scale planes of pack.cuh); a stage
// of 8 K-blocks of a tile's 128 rows (16 KB of nibbles) is brought in by one TMA tensor copy and
// split by the producer warp into unsigned bytes n in the canonical no-swizzle K-major layout
// tcgen05 reads (8-row x 16-byte core matrices); a second MMA against a constant tile of -8
// adds -8 * sum(q), so D_b = sum (n - 8) q exactly. Activation tiles (128 tokens x 8 blocks) are
// TMA tensor copies straight into that layout: the tensor map's dimensions are ordered
// (16 bytes, rows, 16-byte chunks) so that a chunk's 128 rows land contiguously.
//
// Epilogue arithmetic. The accumulators start each block at the bits of 1.5 * 2^23, so D_b reads
// as a float offset by that constant and one exact subtraction replaces the int-to-float
// conversion; the products and sums run two tokens at a time on the f32x2 instructions of
// sm_100. That is 4 f32 operations per (row, token, block) against 64 tensor-core operations:
// the CUDA cores, not the tensor cores, bound this kernel (exact per-block scales cost that).
//
// Pipeline (one CTA per tile, 17 warps): warp 16 is the producer and MMA issuer (lane 0 issues
// the TMA copies and the MMAs, all lanes unpack); warps 0-15 are the epilogue, warp w reading
// tensor-memory lanes 32 (w % 4) .. + 31 (tile rows) and columns 32 (w / 4) .. + 31 (tokens);
// warps whose 32 columns hold no token of the tile stay idle. Three shared-memory stages of
// activations, one nibble buffer, four tensor-memory accumulators of 128 columns, mbarriers
// between the roles; every wait is bounded (a timeout ends in the status word, never in a hang).
#pragma once
#include "common.cuh"
#include "pack.cuh"

#include <cuda.h>

namespace rvc {

constexpr int PF_M = 128;          // rows per tile (tensor-memory lanes)
constexpr int PF_N = 128;          // tokens per tile (accumulator columns)
constexpr int PF_KB = 8;           // K-blocks per stage
constexpr int PF_STAGES = 3;
constexpr int PF_TBUF = 4;         // tensor-memory accumulators
constexpr int PF_EPI_WARPS = 8;
constexpr int PF_THREADS = (PF_EPI_WARPS + 1) * 32;
constexpr int PF_TMEM_COLS = PF_TBUF * PF_N;  // 512: the whole tensor memory of the SM

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
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The wait with the loaded registers as operands: the compiler cannot move their uses above it
// (tcgen05.ld writes them asynchronously; plain register uses are not ordered by a memory clobber).
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
                 :
                 : "memory");
}
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
// Q8_0 of x, once per token: warp task (token t, block b) quantises the block and writes it into
// the records of the token's `used` plan positions pos_of[t used + j], with the block scale also
// in the block-major plane xd[b][position] the GEMM's scale tiles come from.
template <typename XT>
__global__ void __launch_bounds__(256) k_pf_quant(const XT *__restrict__ x, int n_embd, int n_tok, int used,
                                                  const int32_t *__restrict__ pos_of, uint8_t *__restrict__ xperm,
                                                  float *__restrict__ xd, int ppad) {
    const int nb = n_embd / QK, xrb = q8rec_bytes(nb);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = n_tok * nb;
    for (int i = blockIdx.x * 8 + warp; i < total; i += gridDim.x * 8) {
        const int t = i / nb, b = i - t * nb;
        const float v = ld_val<XT>(x, (size_t)t * n_embd + (size_t)b * QK + lane);
        uint16_t dbits;
        int qsum;
        const int8_t q = quant_q8_lane(v, &dbits, &qsum);
        const float d = f16_bits_to_f32(dbits);
        for (int j = 0; j < used; ++j) {
            const int k = __ldg(pos_of + t * used + j);
            q8rec_store(xperm + (size_t)k * xrb, nb, b, lane, q, dbits, qsum);
            if (lane == 0) xd[(size_t)b * ppad + k] = d;
        }
    }
}

// ------------------------------------------------------------------ combine
// out[t][r] = slot-order sum over j of (y[pos_of[t used + j]][r] * down_scale[e]) * w[t][j].
__global__ void __launch_bounds__(256) k_pf_combine(const float *__restrict__ y, const int32_t *__restrict__ pos_of,
                                                    const int32_t *__restrict__ ids, const float *__restrict__ wts,
                                                    const float *__restrict__ down_scale, int used, int n_embd,
                                                    int n_tok, float *__restrict__ out) {
    const long long total = (long long)n_tok * n_embd;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / n_embd), r = (int)(i - (long long)t * n_embd);
        float o = 0.0f;
        for (int j = 0; j < used; ++j) {
            const int p = t * used + j;
            const int e = __ldg(ids + p);
            const float ds = down_scale ? __ldg(down_scale + e) : 1.0f;
            const float v = __fmul_rn(__fmul_rn(__ldg(y + (size_t)__ldg(pos_of + p) * n_embd + r), ds), __ldg(wts + p));
            o = j == 0 ? v : __fadd_rn(o, v);
        }
        out[i] = o;
    }
}

// ------------------------------------------------------------------ grouped GEMM
struct PfArgs {
    const int2 *tiles;    // per tile: (expert | tokens << 8, first plan position), from k_plan
    const int *n_tiles;
    int rows_per_expert;  // 2 ff (gate/up) or n_embd (down)
    int nblk;             // K blocks (n_embd / 32 or ff / 32)
    int swizzled;         // the nibble plane's blocks are XOR-swizzled per row (gate/up)
    const uint16_t *scl;  // weight scales [E][rows][nblk] (f16 bits)
    int nh;               // (gate/up) h blocks per pair (ff / 32): the h record geometry
    uint8_t *hrec;        // (gate/up) out: h records by plan position
    float *hd;            // (gate/up) out: h block scales, block-major [nh][ppad]
    int ppad;
    float *y;             // (down) out: [positions][n_embd]
    int n_embd;
    int *status;
    uint64_t negzero2;    // two f32 -0 (0x80000000 each): see f2_prod
};

constexpr int PF_GU = 0, PF_DN = 1;

// Shared memory of one stage: unpacked A (8 blocks x 2 halves x 128 rows x 16 B), B (same for
// 128 tokens), the tokens' block scales (8 blocks x 128 tokens f32); after the stages one
// buffer for the nibbles of A (128 rows x 8 blocks x 16 B), refilled as soon as they are
// unpacked, and the constant A tile of -8 (one block).
constexpr int PF_A_BYTES = PF_KB * 2 * PF_M * 16;  // 32 KB
constexpr int PF_B_BYTES = PF_KB * 2 * PF_N * 16;  // 32 KB
constexpr int PF_NIB_BYTES = PF_M * PF_KB * 16;    // 16 KB
constexpr int PF_DX_BYTES = PF_N * PF_KB * 4;      // 4 KB
constexpr int PF_C_BYTES = 2 * PF_M * 16;          // 4 KB
constexpr int PF_STAGE_BYTES = PF_A_BYTES + PF_B_BYTES + PF_DX_BYTES;
constexpr int PF_SMEM_BYTES = PF_STAGES * PF_STAGE_BYTES + PF_NIB_BYTES + PF_C_BYTES + 1024;  // + alignment slack

// The tensor-memory accumulators start every block at the bits of 1.5 * 2^23: the int32 sum
// C + D of a block dot D (|D| < 2^22) then reads as the float 1.5 * 2^23 + D exactly, and one
// exact subtraction gives (float)D.
constexpr uint32_t PF_MAGIC_BITS = 0x4B400000u;
constexpr float PF_MAGIC = 12582912.0f;

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
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(((uint64_t)__float_as_uint(a.y) << 32) | __float_as_uint(a.x)),
          "l"(((uint64_t)__float_as_uint(b.y) << 32) | __float_as_uint(b.x)));
    return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}

// 32 lanes x 32 columns of tensor memory set to one value; tcgen05.wait::st before reuse.
__device__ __forceinline__ void tmem_fill32(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void named_sync_n(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// One (expert, 128 weight rows, up to 128 plan positions) tile per CTA. Per 32-column block b:
//   D = C + u8(n) . q     (tcgen05.mma kind::i8, A unsigned: the nibbles as stored)
//   D = D + (-8) . q      (A signed: a constant tile), so D = C + sum (n - 8) q exactly;
// the epilogue warps read D, put C back for block b + 4, and accumulate
//   acc = acc + ((float)(D - C) * (dw_b * dx_b))   (each operation rounded, as the reference).
template <int MODE>
__global__ void __launch_bounds__(PF_THREADS, 1) k_pf_gemm(const __grid_constant__ CUtensorMap map_nib,
                                                           const __grid_constant__ CUtensorMap map_act,
                                                           const __grid_constant__ CUtensorMap map_dx, PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full_bar[PF_STAGES], stage_free[PF_STAGES], mma_done[PF_TBUF], tmem_free[PF_TBUF], nib_full;
    __shared__ uint32_t taddr_s;
    if ((int)blockIdx.y >= __ldg(a.n_tiles)) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.nblk, rows = a.rows_per_expert;
    const int row0 = blockIdx.x * PF_M;  // tile rows within the expert
    const int2 td = __ldg(a.tiles + blockIdx.y);
    const int e = td.x & 0xFF, nt = td.x >> 8, p0 = td.y;
    const int ncg = (nt + 31) >> 5;  // 32-token column groups holding tokens
    const int nch = (nt + 63) >> 6;  // 64-token column halves holding tokens (epilogue warps 4 ch .. + 3)
    const int nst = (nblk + PF_KB - 1) / PF_KB;
    uint8_t *const sN = smem + (size_t)PF_STAGES * PF_STAGE_BYTES;
    uint8_t *const sC = sN + PF_NIB_BYTES;

    if (warp == 0) {
        tmem_alloc(&taddr_s, PF_TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int s = 0; s < PF_STAGES; ++s) mbar_init(&full_bar[s], 1), mbar_init(&stage_free[s], 1 + 4 * nch);
        for (int s = 0; s < PF_TBUF; ++s) mbar_init(&mma_done[s], 1), mbar_init(&tmem_free[s], 4 * nch);
        mbar_init(&nib_full, 1);
        fence_barrier_init();
    }
    if (warp == PF_EPI_WARPS) {  // the constant tile: int8 -8 everywhere
        for (int i = lane; i < PF_C_BYTES / 16; i += 32)
            reinterpret_cast<uint4 *>(sC)[i] = make_uint4(0xF8F8F8F8u, 0xF8F8F8F8u, 0xF8F8F8F8u, 0xF8F8F8F8u);
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = taddr_s;
    auto stage_ptr = [&](int s) { return smem + (size_t)s * PF_STAGE_BYTES; };

    if (warp == PF_EPI_WARPS) {
        // ------------------------------------------------ producer + MMA issuer
        // B tiles and token scales go out two stages ahead; the nibbles of the next stage as soon
        // as this stage's are unpacked.
        const uint32_t id_u = idesc_i8(PF_M, ncg * 32, false), id_s = idesc_i8(PF_M, ncg * 32, true);
        const uint64_t dC = umma_desc(sC, PF_M * 16, 128);
        const int wrow0 = e * rows + row0;  // first weight row of the tile
        auto issue_nib = [&](int st) {
            mbar_arrive_expect_tx(&nib_full, PF_NIB_BYTES);
            tma_load_3d(sN, &map_nib, 0, st * PF_KB, wrow0, &nib_full);  // [128 rows][8 blocks][16 B]
        };
        auto issue_bx = [&](int st) {
            const int s = st % PF_STAGES;
            uint8_t *sB = stage_ptr(s) + PF_A_BYTES;
            mbar_arrive_expect_tx(&full_bar[s], PF_B_BYTES + PF_DX_BYTES);
            tma_load_3d(sB, &map_act, 0, p0, 2 * st * PF_KB, &full_bar[s]);      // [16 halves][128 tokens][16 B]
            tma_load_2d(sB + PF_B_BYTES, &map_dx, p0, st * PF_KB, &full_bar[s]);  // [8 blocks][128 tokens] f32
        };
        if (lane == 0) {
            issue_nib(0);
            for (int st = 0; st < min(nst, 2); ++st) issue_bx(st);
        }
        bool ok = true;
        for (int st = 0; st < nst && ok; ++st) {
            const int s = st % PF_STAGES;
            uint8_t *sA = stage_ptr(s), *sB = sA + PF_A_BYTES;
            const int kb0 = st * PF_KB, kn = min(PF_KB, nblk - kb0);
            // slot s last held stage st - 3, complete since the previous iteration's wait
            ok &= pf_wait(&nib_full, (uint32_t)st & 1u, a.status);
            if (!__all_sync(0xffffffffu, ok)) break;
            // unpack: task (row r, block j) -> nibble bytes split into halves 0, 1 at
            // sA + (2 j + k) * 2048 + r * 16. The 8 lanes of one 16-byte access phase take 8
            // consecutive rows (distinct write banks) and blocks whose stored positions differ
            // (distinct read banks): the block is fixed when the rows are swizzled (position
            // j ^ (r & 7); the tile's rows start at a multiple of 8), and runs along the diagonal
            // when they are not.
#pragma unroll 2
            for (int i = lane; i < PF_M * PF_KB; i += 32) {
                const int l = i & 7, g = i >> 3, c = g >> 4;
                const int r = (g & 15) * 8 + l;
                const int j = a.swizzled ? c : ((l + c) & 7);
                const int pos = a.swizzled ? (c ^ l) : j;
                const uint4 nb4 = *reinterpret_cast<const uint4 *>(sN + r * (PF_KB * 16) + pos * 16);
                const uint4 lo = make_uint4(nb4.x & 0x0F0F0F0Fu, nb4.y & 0x0F0F0F0Fu, nb4.z & 0x0F0F0F0Fu,
                                            nb4.w & 0x0F0F0F0Fu);
                const uint4 hi = make_uint4((nb4.x >> 4) & 0x0F0F0F0Fu, (nb4.y >> 4) & 0x0F0F0F0Fu,
                                            (nb4.z >> 4) & 0x0F0F0F0Fu, (nb4.w >> 4) & 0x0F0F0F0Fu);
                *reinterpret_cast<uint4 *>(sA + (2 * j) * (PF_M * 16) + r * 16) = lo;
                *reinterpret_cast<uint4 *>(sA + (2 * j + 1) * (PF_M * 16) + r * 16) = hi;
            }
            fence_proxy_async_smem();  // the A tile for the tensor core; the nibble reads before the refill
            __syncwarp();
            if (lane == 0 && st + 1 < nst) issue_nib(st + 1);
            ok &= pf_wait(&full_bar[s], (uint32_t)(st / PF_STAGES) & 1u, a.status);
            if (!__all_sync(0xffffffffu, ok)) break;
            if (lane == 0) {
                for (int j = 0; j < kn && ok; ++j) {
                    const int b = kb0 + j, buf = b % PF_TBUF;
                    // the epilogue has read the accumulator's previous block and put C back
                    ok &= pf_wait(&tmem_free[buf], (b / PF_TBUF) & 1u, a.status);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t dB = umma_desc(sB + j * 2 * (PF_N * 16), PF_N * 16, 128);
                    mma_i8(taddr + buf * PF_N, umma_desc(sA + j * 2 * (PF_M * 16), PF_M * 16, 128), dB, id_u, true);
                    mma_i8(taddr + buf * PF_N, dC, dB, id_s, true);
                    mma_commit(&mma_done[buf]);
                }
                mma_commit(&stage_free[s]);  // the stage's buffers are free once its MMAs are done
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            // B tile of stage st + 2 into the slot of stage st - 1, once that stage is consumed (its
            // MMAs and the epilogue's reads of its scales): the unpack of st + 1 then overlaps the
            // epilogue of st
            const int sa = st + 2;
            if (ok && sa < nst) {
                if (sa >= PF_STAGES) ok &= pf_wait(&stage_free[sa % PF_STAGES], ((sa / PF_STAGES) - 1) & 1u, a.status);
                if (!__all_sync(0xffffffffu, ok)) break;
                if (lane == 0) issue_bx(sa);
            }
        }
        if (!ok) set_status(a.status, STATUS_TIMEOUT);
    } else if ((warp >> 2) < nch) {
        // ------------------------------------------------ epilogue: scale and accumulate
        const int m = 32 * (warp & 3) + lane;  // tile row (tensor-memory lane)
        const int ch = warp >> 2;              // token columns 64 ch .. 64 ch + 63
        const int ng = min(2, ncg - 2 * ch);   // of which 32-column groups hold tokens (1 or 2)
        const uint32_t tw = taddr + ((uint32_t)(32 * (warp & 3)) << 16) + ch * 64;
#pragma unroll 1
        for (int buf = 0; buf < PF_TBUF; ++buf) {
            tmem_fill32(tw + buf * PF_N, PF_MAGIC_BITS);
            if (ng > 1) tmem_fill32(tw + buf * PF_N + 32, PF_MAGIC_BITS);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int buf = 0; buf < PF_TBUF; ++buf) mbar_arrive(&tmem_free[buf]);
        float2 acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.0f, 0.0f);
        // this row's weight scales (f16 pairs), 8 per stage: loaded at the stage's start from L1,
        // where a prefetch one stage earlier has put them (no registers held across the stage)
        const uint32_t *srow = reinterpret_cast<const uint32_t *>(a.scl + ((size_t)e * rows + row0 + m) * nblk);
        const int nw = nblk >> 1;  // f16 pairs per row (nblk is even)
        uint32_t c0 = 0, c1 = 0, c2 = 0, c3 = 0;
        asm volatile("prefetch.global.L1 [%0];" ::"l"(srow));
        const float2 negc = make_float2(-PF_MAGIC, -PF_MAGIC);
        const uint64_t nz2 = a.negzero2;
        bool ok = true;
        for (int b = 0; b < nblk; ++b) {
            const int buf = b % PF_TBUF, st = b / PF_KB, s = st % PF_STAGES, j = b % PF_KB;
            if (j == 0) {
                const int k0 = st * (PF_KB / 2);
                c0 = k0 + 0 < nw ? __ldg(srow + k0 + 0) : 0u;
                c1 = k0 + 1 < nw ? __ldg(srow + k0 + 1) : 0u;
                c2 = k0 + 2 < nw ? __ldg(srow + k0 + 2) : 0u;
                c3 = k0 + 3 < nw ? __ldg(srow + k0 + 3) : 0u;
                if (k0 + PF_KB / 2 < nw) asm volatile("prefetch.global.L1 [%0];" ::"l"(srow + k0 + PF_KB / 2));
                if (k0 + PF_KB / 2 + 3 < nw) asm volatile("prefetch.global.L1 [%0];" ::"l"(srow + k0 + PF_KB / 2 + 3));
            }
            ok &= pf_wait(&mma_done[buf], (b / PF_TBUF) & 1u, a.status);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const float4 *sdx = reinterpret_cast<const float4 *>(stage_ptr(s) + PF_A_BYTES + PF_B_BYTES) +
                                (j * PF_N + ch * 64) / 4;
            const uint32_t wpair = (j >> 1) == 0 ? c0 : (j >> 1) == 1 ? c1 : (j >> 1) == 2 ? c2 : c3;
            const float dw = f16_bits_to_f32((uint16_t)((j & 1) ? (wpair >> 16) : (wpair & 0xFFFFu)));
            const float2 dw2 = make_float2(dw, dw);
            // 16 columns at a time (4 chunks when both groups hold tokens); after the last read
            // C goes back for block b + 4
            const int nck = 2 * ng;
#pragma unroll
            for (int ck = 0; ck < 4; ++ck) {
                if (ck < nck) {
                    uint32_t v[16];
                    tmem_ld16(tw + buf * PF_N + ck * 16, v);
                    tmem_ld_wait(v);
                    if (ck == nck - 1) {
                        tmem_fill32(tw + buf * PF_N, PF_MAGIC_BITS);
                        if (ng > 1) tmem_fill32(tw + buf * PF_N + 32, PF_MAGIC_BITS);
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tmem_free[buf]);
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 dx = sdx[ck * 4 + q];
                        const float2 s0 = f2_mul(dw2, make_float2(dx.x, dx.y));
                        const float2 s1 = f2_mul(dw2, make_float2(dx.z, dx.w));
                        const float2 t0 =
                            f2_add(make_float2(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1])), negc);
                        const float2 t1 =
                            f2_add(make_float2(__uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])), negc);
                        acc[ck * 8 + 2 * q] = f2_add(acc[ck * 8 + 2 * q], f2_prod(t0, s0, nz2));
                        acc[ck * 8 + 2 * q + 1] = f2_add(acc[ck * 8 + 2 * q + 1], f2_prod(t1, s1, nz2));
                    }
                }
            }
            if (j == PF_KB - 1 || b == nblk - 1) {  // done with this stage's token scales
                __syncwarp();
                if (lane == 0) mbar_arrive(&stage_free[s]);
            }
        }
        if (!ok) set_status(a.status, STATUS_TIMEOUT);
        // ------------------------------------------------ outputs
        if (MODE == PF_DN) {
            if (ok) {
                float *yp = a.y + (size_t)(p0 + ch * 64) * a.n_embd + row0 + m;
                const int nv = min(64, nt - ch * 64);
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const float2 v2 = acc[i >> 1];
                    if (i < nv) *yp = (i & 1) ? v2.y : v2.x;
                    yp += a.n_embd;
                }
            }
        } else {
            // rows: unit u = m / 64 of the tile; m % 64 < 32 gate, else up; column m % 32.
            // Both go through shared memory (stage 0, free now): [gate/up][2 units][32 columns]
            // [128 tokens], so that no accumulator is live across the quantisation calls.
            float *sg = reinterpret_cast<float *>(smem);
            const int nthr = nch * 4 * 32;
            named_sync_n(6, nthr);
            const int u = m >> 6, col = m & 31;
            const bool gate = (m & 63) < 32;
            float *mine = sg + ((gate ? 0 : 2) + u) * 32 * PF_N + col * PF_N + ch * 64;
#pragma unroll
            for (int i = 0; i < 32; ++i) reinterpret_cast<float2 *>(mine)[i] = acc[i];
            named_sync_n(6, nthr);
            if (!gate && ok) {
                const int hrb = q8rec_bytes(a.nh);
                const int q = (row0 >> 6) + u;  // h block within the expert's ff columns
                const float *gp = sg + u * 32 * PF_N + col * PF_N, *up = sg + (2 + u) * 32 * PF_N + col * PF_N;
#pragma unroll 1
                for (int i = 0; i < 64; ++i) {
                    const int n = ch * 64 + i;
                    const float hv = __fmul_rn(gelu_tanh(gp[n]), up[n]);
                    uint16_t dbits;
                    int qsum;
                    const int8_t qv = quant_q8_lane(hv, &dbits, &qsum);  // the warp's 32 lanes: one block
                    if (n < nt) {
                        q8rec_store(a.hrec + (size_t)(p0 + n) * hrb, a.nh, q, lane, qv, dbits, qsum);
                        if (lane == 0) a.hd[(size_t)q * a.ppad + p0 + n] = f16_bits_to_f32(dbits);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, PF_TMEM_COLS);
}

}  // namespace rvc
