// prefill_tc.cuh - the grouped expert GEMM of the prefill path on the 5th-generation tensor
// cores: tcgen05.mma into tensor memory, exact per-block scaling on the CUDA cores.
//
// Computes what the reference's CPU-experts Q8_0 path computes for every (weight row, plan
// position) pair of an expert group (runtime/src/expert_pool.rs:86-135 driving
// expert_kernel.rs:147-161):
//
//     acc = 0;  for b in blocks:  acc = acc + (float)sumi_b * (dw_b * dx_b)
//
// with sumi_b the exact int32 dot of block b's Q4_0 nibbles (minus 8) and the activation's Q8_0
// quants, and every f32 operation rounded where the reference rounds it. Then, for gate/up,
// h = gelu(gate) * up and its Q8_0 quants (exec.rs:606-611, ops.rs:95-105); for down, y per
// (position, row), combined afterwards in slot order (k_pf_combine).
//
// The block dots: the integer operands n - 8 (-8..7) and q (-127..127) are held as f16, which
// represents them exactly, and multiplied by tcgen05.mma kind::f16 with f32 accumulation: every
// product and every partial sum is an integer below 2^15 in magnitude, so the tensor core's f32
// accumulation is exact and tensor memory receives (float)sumi_b itself. (An i8 MMA gives the
// same integers as int32, but their conversion to f32 competes with the f32x2 arithmetic for the
// CUDA cores' issue and pipes: measured on B200, 4 conversions + 6 f32x2 operations run at 6.8
// iterations per SM cycle against 9.1 without the conversions, rosevine_b200/micro/tc_probe.cu.)
//
// Design, from measurements on B200 (tc_probe.cu):
//   - per 32-column block two MMAs (M = 128 rows, N = 128 positions, K = 16 each; the second
//     accumulates) write the block's dots to a tensor-memory buffer; four buffers of 128 columns
//     let the MMAs run ahead of the epilogue. The accumulate flag is an immediate: with a runtime
//     predicate an MMA costs 200-280 issue cycles instead of about 80;
//   - tensor-memory loads do not wait for MMAs in flight on other columns; an epilogue warp
//     hands its buffer back as soon as the dots are in registers;
//   - the epilogue's three f32 operations per (row, position, block) bound the kernel.
//
// Roles (one CTA per SM, persistent over the (row tile, position tile) list):
//   warp 0       tensor-memory allocation; the copies of a stage (2 blocks), all by TMA / bulk
//                copy: the weight nibbles of the tile's 128 rows (four 1 KB tensor copies, one per
//                swizzle key pair of the packed plane, below), then the activation quants of 128
//                positions x 128 B (one tensor copy in the 128-byte swizzle layout, which the MMA
//                reads as its K-major B operand: a copy of 16-byte rows instead ran at about 12 B
//                per SM cycle and bounded the kernel), activation scales [2][128] f32 and weight
//                scales [2][128] f32 (the tile-major scale plane). Five stages in shared memory
//                run up to 10 blocks ahead of the MMAs
//   warp 1       MMA issue (the whole warp runs the loop; one elected lane issues)
//   warps 2-3    weight unpack: thread r turns rows r and r + 64's nibbles (shared memory) into
//                f16 n - 8 in the MMA's K-major A layout
//   warps 4-19   epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (one weight row
//                per thread) and positions 32 ((w - 4) / 4) .. + 31; per block and position
//                s = dw * dx, p = t * s (rounded product), acc = acc + p.
// The packed nibble plane stores row R's block b at b ^ (R & 7) within complete groups of 8 blocks
// (pack.cuh). A stage's block pair (2 st, 2 st + 1) of row R = 8 g + 2 k + j then sits in stored
// pair st ^ k with its blocks in order i ^ j: viewed as [g][k][j][pair][32 B], one tensor copy per
// k of box [16 g][2 j][one pair] fetches the stage's nibbles of a whole row tile.
// Every wait is bounded; a wait that runs out records STATUS_TIMEOUT and ends the CTA's work
// (all roles see the abort flag), after the MMAs and copies in flight have completed.
#pragma once
#include "common.cuh"
#include "pack.cuh"
#include "prefill.cuh"

#include <cuda.h>

namespace rvc {

constexpr int TC_M = 128;     // weight rows per tile (tensor-memory lanes)
constexpr int TC_N = 128;     // plan positions per tile (tensor-memory columns per buffer)
constexpr int TC_KB = 2;      // blocks per stage
constexpr int TC_STAGES = 5;  // shared-memory stages: copies and unpacking run up to 6 blocks ahead of the MMAs
constexpr int TC_TBUF = 4;    // tensor-memory buffers of TC_N columns
constexpr int TC_EPI_WARPS = 16;  // four per SM sub-partition: one lane quarter x one 32-position quarter each
constexpr int TC_EPI_POS = TC_N * 4 / TC_EPI_WARPS;  // positions per epilogue warp (32)
constexpr int TC_THREADS = (4 + TC_EPI_WARPS) * 32;  // 640: up to 96 registers a thread
// An operand row holds a block's 32 values as 4 K chunks of 8 f16 (16 B): chunk c = elements
// 8 c .. 8 c + 7. In shared memory a block's operand is [4 chunks][128 rows][16 B]; MMA k (k = 0,
// 1) reads chunks 2 k, 2 k + 1 (lbo 2048 B between them, 8-row groups 128 B apart).
constexpr int TC_BLK_BYTES = 4 * 128 * 16;                 // 8 KB
constexpr int TC_OFF_B = 0;  // activation operands: [128 positions][TC_KB blocks x 64 B], 128-byte swizzle
constexpr int TC_OFF_DX = TC_OFF_B + TC_KB * TC_BLK_BYTES;  // [TC_KB blocks][128 positions] f32 scales
constexpr int TC_OFF_DW = TC_OFF_DX + TC_KB * TC_N * 4;    // [TC_KB blocks][128 rows] f32 weight scales
constexpr int TC_OFF_NIB = TC_OFF_DW + TC_KB * TC_M * 4;   // [4 k][16 g][2 j][2 blocks][16 B] weight nibbles
constexpr int TC_NIB_BYTES = TC_KB * TC_M * 16;            // 4 KB
constexpr int TC_OFF_A = TC_OFF_NIB + TC_NIB_BYTES;        // [TC_KB blocks] weight operands (unpacked)
constexpr int TC_STAGE_BYTES = TC_OFF_A + TC_KB * TC_BLK_BYTES;  // 38 KB
constexpr int TC_FULL_BYTES = TC_OFF_NIB;                  // bytes the copies on full[] write (B, DX, DW)
static_assert(TC_KB == 2, "a stage is one block pair of the swizzled nibble plane");
// gate/up output exchange: per (unit, position half) pair of warps, gate values of 32 positions
// and up values of 32 positions, [32][32 columns] f32 each
constexpr int TC_OFF_STG = TC_STAGES * TC_STAGE_BYTES;
constexpr int TC_STG_PAIR = 2 * (TC_EPI_POS / 2) * 32 * 4;
constexpr int TC_SMEM_BYTES = TC_OFF_STG + 2 * (TC_EPI_WARPS / 4) * TC_STG_PAIR + 1024;  // + alignment slack
static_assert(TC_SMEM_BYTES <= 227 * 1024, "shared memory of k_pf_gemm_tc");
static_assert(TC_STAGE_BYTES % 1024 == 0, "stage alignment");

constexpr int PF_GU = 0, PF_DN = 1, PF_RAW = 2;  // gate/up, down, raw block dots (debug)

struct TcArgs {
    const int2 *tiles;    // per tile: (expert | positions << 8, first plan position), from k_plan
    const int *n_tiles;
    int max_tiles;        // the tile list's capacity (a larger count read from the device is clamped)
    int n_experts;
    int ppos;             // plan positions of the workspace layout (tile entries are checked)
    int rows_per_expert;  // 2 ff (gate/up) or n_embd (down)
    int row_tiles;        // row tiles per position tile (rows_per_expert / TC_M)
    int row_base;         // first weight row of row tile 0 (0; another row tile for the debug check)
    int nblk;             // K blocks (n_embd / 32 or ff / 32), even
    const float *dwp;     // weight scales, tile-major [E * rows / 128][nblk][128] f32 (pack.cuh)
    int nh;               // (gate/up) h blocks per pair (ff / 32)
    uint8_t *hrec;        // (gate/up) out: h quants (pf_rec_bytes per plan position)
    float *hsc;           // (gate/up) out: h block scales, block-major [nh][ppad] f32
    int ppad;
    float *y;             // (down) out: [positions][n_embd]; (raw) out: int32 [nblk][128][128]
    int n_embd;
    int *status;
    uint64_t negzero2;    // two f32 -0 (0x80000000 each): the addend of f2x_prod
};

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

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices; lbo =
// bytes between the two 16-byte K halves of a 32-byte K step, sbo = bytes between consecutive
// 8-row groups (start >> 4 at bits 0-13, lbo >> 4 at 16-29, sbo >> 4 at 32-45, version 1 at
// 46-47, layout type 0 at 61-63).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// The same for a K-major operand in the 128-byte swizzle layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 B (64 f16 of K), 16-byte chunk c of row r stored at
// chunk c ^ (r & 7), 8-row atoms 1024 B apart (sbo), atoms 1024-byte aligned (base offset 0);
// the K step of an MMA inside the row advances the start address by 32 B (layout type 2 at
// bits 61-63; lbo unused, 16 B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: f32 accumulator (bits 4-5 = 1), A and B f16 (bits 7-9 and
// 10-12 = 0), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// A block's two MMAs (D = A0 B0, then D += A1 B1) and the commit that arrives on `bar` once they
// have completed, under one election: the fewest instructions on the MMA warp's loop, which is
// the GEMM's critical path.
__device__ __forceinline__ void mma_block_elect(uint32_t tmem_d, uint64_t da0, uint64_t db0, uint64_t da1, uint64_t db1,
                                                uint32_t idesc, uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e, p0, p1;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p0, 0, 0;\n\t"
        "setp.ne.b32 p1, 1, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %5, p0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %4, %5, p1;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}\n" ::"r"(tmem_d),
        "l"(da0), "l"(db0), "l"(da1), "l"(db1), "r"(idesc), "r"(smem_u32(bar))
        : "memory");
}
// Arrive on `bar` once every tcgen05 operation issued before by this thread has completed
// (elected lane of a converged warp).
__device__ __forceinline__ void mma_commit_elect(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
        : "memory");
}

#define RVC_LD32_OUT                                                                                           \
    "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), \
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),  \
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
#define RVC_LD32_INOUT                                                                                         \
    "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), \
        "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]),  \
        "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), \
        "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])

// 32 lanes x 32 consecutive 32-bit columns from tensor memory, then the wait; the wait names the
// loaded registers so the compiler cannot move their uses above it.
__device__ __forceinline__ void tmem_ld32_sync(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : RVC_LD32_OUT
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" : RVC_LD32_INOUT : : "memory");
}

// The same load with the 32 values delivered as 16 f32x2-ready pairs (column 2 k in the low half):
// the pairs are formed inside the asm, so that the register allocator places each pair's halves
// together instead of copying them afterwards.
__device__ __forceinline__ void tmem_ld32_pairs(uint32_t taddr, uint64_t (&p)[16]) {
    asm volatile(
        "{\n\t.reg .b32 r<32>;\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {r0, r1, r2, r3, r4, r5, r6, r7, r8, r9, r10, r11, r12, r13, r14, r15, "
        "r16, r17, r18, r19, r20, r21, r22, r23, r24, r25, r26, r27, r28, r29, r30, r31}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t"
        "mov.b64 %0, {r0, r1};\n\tmov.b64 %1, {r2, r3};\n\tmov.b64 %2, {r4, r5};\n\tmov.b64 %3, {r6, r7};\n\t"
        "mov.b64 %4, {r8, r9};\n\tmov.b64 %5, {r10, r11};\n\tmov.b64 %6, {r12, r13};\n\tmov.b64 %7, {r14, r15};\n\t"
        "mov.b64 %8, {r16, r17};\n\tmov.b64 %9, {r18, r19};\n\tmov.b64 %10, {r20, r21};\n\tmov.b64 %11, {r22, r23};\n\t"
        "mov.b64 %12, {r24, r25};\n\tmov.b64 %13, {r26, r27};\n\tmov.b64 %14, {r28, r29};\n\tmov.b64 %15, {r30, r31};\n\t}"
        : "=l"(p[0]), "=l"(p[1]), "=l"(p[2]), "=l"(p[3]), "=l"(p[4]), "=l"(p[5]), "=l"(p[6]), "=l"(p[7]), "=l"(p[8]),
          "=l"(p[9]), "=l"(p[10]), "=l"(p[11]), "=l"(p[12]), "=l"(p[13]), "=l"(p[14]), "=l"(p[15])
        : "r"(taddr)
        : "memory");
}

// Two f32x2 pairs (four consecutive f32) from shared memory.
__device__ __forceinline__ void lds_2x2(uint32_t addr, uint64_t &a, uint64_t &b) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}
// One f32 from shared memory in both halves of an f32x2 pair.
__device__ __forceinline__ uint64_t lds_splat(uint32_t addr) {
    uint64_t r;
    asm volatile("{\n\t.reg .b32 t;\n\tld.shared.b32 t, [%1];\n\tmov.b64 %0, {t, t};\n\t}" : "=l"(r) : "r"(addr));
    return r;
}

// 2-D / 3-D TMA tensor copies global -> shared, completion on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
        "%6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
        : "memory");
}
// Contiguous global -> shared copy (16-byte aligned addresses, a multiple of 16 bytes).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ------------------------------------------------------------------ f32x2 arithmetic
// Two f32 values in one 64-bit register (low half: the first). Each operation rounds each lane to
// nearest even. A product that feeds an add comes from f2x_prod, an fma whose -0 addend is held
// in a register loaded from the kernel's arguments: that is the rounded product, sign of zero
// included. The compiler contracts an f32x2 mul followed by an add into one fma (rounding once),
// for the intrinsics and for inline mul.rn/add.rn.f32x2 alike, and turns an fma with a literal -0
// addend back into a mul (both measured on B200); an fma whose addend it cannot see, followed by
// an add, stays two roundings.
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
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2x_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2x_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// gelu_tanh (common.cuh) with tanh inlined, so that independent evaluations overlap: the same
// operations in the same order (ops.rs:145-149), tanh in double rounded once to f32.
__device__ __forceinline__ float gelu_tanh_inl(float x) {
    const float A = 0.044715f;
    const float S = 0.7978846f;
    const float inner = __fmul_rn(__fmul_rn(S, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(A, x), x)));
    const float t = (float)tanh((double)inner);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// Four nibble values n in 0..15 (one per byte of n4) as two f16x2 words of n - 8: a byte
// permute builds the f16 bits 0x6400 | n (the value 1024 + n, exact), and one f16x2 subtraction
// of 1032 leaves n - 8 exactly.
__device__ __forceinline__ uint2 nib_f16x4(uint32_t n4) {
    uint32_t a, b;
    asm("prmt.b32 %0, %1, 0x64646464, 0x4140;" : "=r"(a) : "r"(n4));
    asm("prmt.b32 %0, %1, 0x64646464, 0x4342;" : "=r"(b) : "r"(n4));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(a) : "r"(0x64086408u));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(b) : "r"(0x64086408u));
    return make_uint2(a, b);
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded mbarrier wait that gives up early once another role has aborted the CTA's work. A phase
// that has completed already is seen by one non-blocking test. A role that is ahead of the
// epilogue (TMA copies, unpack, MMA issue) waits with `backoff`: between polls it sleeps, from
// 32 ns doubling up to 512 ns, so that it does not take issue slots from the epilogue warps that
// share its SM sub-partition (measured: spinning waits issued as many instructions as the
// epilogue's arithmetic). The epilogue polls without sleeping.
constexpr long long TC_WAIT_ITERS = 1ll << 22;  // at most about 2 s of polls
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *status,
                                        bool backoff = false) {
    if (mbar_test_wait(bar, parity)) return true;
    uint32_t ns = 32;
    for (long long i = 0; i < TC_WAIT_ITERS; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (backoff) {
            __nanosleep(ns);
            ns = ns < 512 ? 2 * ns : 512;
        }
    }
    set_status(status, STATUS_TIMEOUT);
    *abort = 1;
    return false;
}

// The same wait in every lane of a warp, with one outcome for the whole warp (the warp-wide
// tcgen05 and barrier operations that follow need all its lanes).
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort, int *status,
                                             bool backoff = false) {
    const bool r = tc_wait(bar, parity, abort, status, backoff);
    return __all_sync(0xffffffffu, r);
}

// 16-byte shared-memory load (four f32).
__device__ __forceinline__ float4 lds128(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// The epilogue warps' barrier (named barrier 1, all TC_EPI_WARPS warps). Every epilogue warp runs
// the same sequence of tiles, stages and blocks, so each reaches every such barrier; waits on
// mbarriers stay with one leader warp and are bounded, and their outcome travels through epi_ok.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(TC_EPI_WARPS * 32) : "memory"); }

// A tile entry from k_plan, checked against the layout: false for an entry that does not fit
// (a stale or foreign workspace), which every role then skips alike.
__device__ __forceinline__ bool tc_tile(const TcArgs &a, int L, int &e, int &nt, int &p0, int &row0) {
    const int ti = L / a.row_tiles, rt = L - ti * a.row_tiles;
    const int2 td = __ldg(a.tiles + ti);
    e = td.x & 0xFF, nt = td.x >> 8, p0 = td.y, row0 = a.row_base + rt * TC_M;
    return e < a.n_experts && nt >= 1 && nt <= TC_N && p0 >= 0 && p0 + nt <= a.ppos;
}

// Profiling builds: a timeline of CTA 0's gate/up GEMM (stage events in slot 6, block events in
// slot 5); compiled away otherwise.
#define TC_TRACE(K, I, P)                          \
    do {                                           \
        if (MODE == PF_GU) RVC_TRACE(K, I, P);     \
    } while (0)

// ------------------------------------------------------------------ the kernel
template <int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1) k_pf_gemm_tc(const __grid_constant__ CUtensorMap map_act,
                                                              const __grid_constant__ CUtensorMap map_dx,
                                                              const __grid_constant__ CUtensorMap map_nib, TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, as an offset from the shared array (keeps shared addressing)
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t full[TC_STAGES], wfull[TC_STAGES], empty[TC_STAGES];
    __shared__ uint64_t tfull[TC_TBUF], tempty[TC_TBUF], drain;
    __shared__ int epi_ok;  // the epilogue leader's wait outcome, read by all epilogue warps after bar.sync
    __shared__ uint32_t taddr_s;
    __shared__ int abort_s;
    volatile int *abort = &abort_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.nblk, nst = (nblk + TC_KB - 1) / TC_KB;
    const int total = max(0, min(__ldg(a.n_tiles), a.max_tiles)) * a.row_tiles;
    if (warp == 0) {
        tmem_alloc(&taddr_s, TC_TBUF * TC_N);
        tmem_relinquish();
    }
    if (tid == 32) {
        for (int s = 0; s < TC_STAGES; ++s) {
            // a stage is ready once its copies have landed and both unpack warps are done: one
            // barrier, so that the MMA warp, whose loop is the GEMM's critical path, waits once
            mbar_init(&full[s], 3);                      // the copies' expect_tx arrival + the two unpack warps
            mbar_init(&wfull[s], 1);
            mbar_init(&empty[s], 1 + TC_EPI_WARPS);      // the MMAs' commit and every epilogue warp
        }
        for (int b = 0; b < TC_TBUF; ++b) mbar_init(&tfull[b], 1), mbar_init(&tempty[b], TC_EPI_WARPS);
        mbar_init(&drain, 1);
        abort_s = 0;
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = taddr_s;
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            int sc = 0;
            bool ok = true;
            for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
                int e, nt, p0, row0;
                if (!tc_tile(a, L, e, nt, p0, row0)) continue;
                for (int st = 0; st < nst && ok; ++st, ++sc) {
                    const int s = sc % TC_STAGES;
                    if (sc >= TC_STAGES && !(ok = tc_wait(&empty[s], (uint32_t)((sc / TC_STAGES - 1) & 1), abort,
                                                          a.status, true)))
                        break;
                    TC_TRACE(6, sc, 0);
                    const uint32_t base = sbase + s * TC_STAGE_BYTES;
                    // weight nibbles first (the unpack warps wait for these alone): stored pair
                    // st ^ k of the rows with key pair k, or pair st past the complete 8-block groups
                    const int g0 = (e * a.rows_per_expert + row0) >> 3;
                    const bool swz = 2 * st < (nblk & ~7);
                    mbar_arrive_expect_tx(&wfull[s], TC_NIB_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        tma_load_5d(base + TC_OFF_NIB + k * (TC_NIB_BYTES / 4), &map_nib, 0, swz ? (st ^ k) : st, 0, k, g0,
                                    &wfull[s]);
                    mbar_arrive_expect_tx(&full[s], TC_FULL_BYTES);
                    tma_load_2d(base + TC_OFF_B, &map_act, st * TC_KB * 64, p0, &full[s]);
                    tma_load_2d(base + TC_OFF_DX, &map_dx, p0, st * TC_KB, &full[s]);
                    const float *dws = a.dwp + ((size_t)((e * a.rows_per_expert + row0) / TC_M) * nblk + st * TC_KB) * TC_M;
                    bulk_load(base + TC_OFF_DW, dws, TC_KB * TC_M * 4, &full[s]);
                }
            }
            // copies still in flight after an abort: wait (bounded) for the last stages issued. The
            // unpack warps may have stopped before arriving on those stages: arrive for them, so
            // that only the copies' bytes are waited for (an arrival beyond a phase's count lands
            // in the next phase, which no role uses after an abort)
            if (!ok)
                for (int k = sc - 1; k >= 0 && k >= sc - TC_STAGES; --k) {
                    fd_mbar_wait(&wfull[k % TC_STAGES], (uint32_t)((k / TC_STAGES) & 1), nullptr);
                    mbar_arrive(&full[k % TC_STAGES]);
                    mbar_arrive(&full[k % TC_STAGES]);
                    fd_mbar_wait(&full[k % TC_STAGES], (uint32_t)((k / TC_STAGES) & 1), nullptr);
                }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issue (whole warp)
        const uint32_t idesc = idesc_f16(TC_M, TC_N);
        int sc = 0, bc = 0;
        bool ok = true;
        for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
            int e, nt, p0, row0;
            if (!tc_tile(a, L, e, nt, p0, row0)) continue;
            for (int st = 0; st < nst && ok; ++st, ++sc) {
                const int s = sc % TC_STAGES;
                const uint32_t par = (uint32_t)((sc / TC_STAGES) & 1);
                if (!(ok = tc_wait_warp(&full[s], par, abort, a.status, true))) break;
                if (lane == 0) TC_TRACE(6, sc, 3);
                tc_fence_after();
                const uint32_t base = sbase + s * TC_STAGE_BYTES;
                const int kn = min(TC_KB, nblk - st * TC_KB);
                for (int j = 0; j < kn; ++j, ++bc) {
                    const int tb = bc % TC_TBUF;
                    if (lane == 0) TC_TRACE(5, bc, 0);
                    if (bc >= TC_TBUF &&
                        !(ok = tc_wait_warp(&tempty[tb], (uint32_t)((bc / TC_TBUF - 1) & 1), abort, a.status, true)))
                        break;
                    tc_fence_after();
                    // block j: K chunks 0, 1 then 2, 3 of the weight (A) and activation (B) operands
                    const uint32_t ab = base + TC_OFF_A + j * TC_BLK_BYTES, bb = base + TC_OFF_B + j * 64;
                    const uint32_t d = tmem + (uint32_t)(tb * TC_N);
                    mma_block_elect(d, umma_desc(ab, 2048, 128), umma_desc_sw128(bb), umma_desc(ab + 4096, 2048, 128),
                                    umma_desc_sw128(bb + 32), idesc, &tfull[tb]);
                    if (lane == 0) TC_TRACE(5, bc, 1);
#ifdef RVC_TC_TRACE_MMA_DONE
                    // profiling builds only: the MMA warp itself timestamps the block's completion
                    if (MODE == PF_GU) {
                        while (!mbar_test_wait(&tfull[tb], (uint32_t)((bc / TC_TBUF) & 1))) {
                        }
                        if (lane == 0) TC_TRACE(5, bc, 6);
                    }
#endif
                }
                if (ok) mma_commit_elect(&empty[s]);  // the stage's operands are free once its MMAs complete
            }
        }
        // every MMA issued has completed before the tensor memory is freed
        mma_commit_elect(&drain);
        fd_mbar_wait(&drain, 0, a.status);
    } else if (warp < 4) {
        // ---------------------------------------------------------- weight unpack (rows r, r + 64)
        // Each row's nibbles (copied into the stage by TMA) become f16 n - 8 in the MMA's A layout.
        const int r0 = tid - 64;
        int sc = 0;
        bool ok = true;
        for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
            int e, nt, p0, row0;
            if (!tc_tile(a, L, e, nt, p0, row0)) continue;
            for (int st = 0; st < nst && ok; ++st, ++sc) {
                const int s = sc % TC_STAGES;
                if (!(ok = tc_wait_warp(&wfull[s], (uint32_t)((sc / TC_STAGES) & 1), abort, a.status, true))) break;
                if (tid == 64) TC_TRACE(6, sc, 1);
                uint8_t *base = smem + s * TC_STAGE_BYTES;
                const uint32_t flip = 2 * st < (nblk & ~7) ? 1u : 0u;  // blocks of a swizzled pair in order i ^ j
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = r0 + 64 * h;
                    const int g = r >> 3, k = (r >> 1) & 3, jr = r & 1;
                    const uint8_t *nrow = base + TC_OFF_NIB + k * (TC_NIB_BYTES / 4) + g * 64 + jr * 32;
#pragma unroll
                    for (int j = 0; j < TC_KB; ++j) {
                        // chunk 0: low nibbles of bytes 0..7 (elements 0..7), 1: of bytes 8..15,
                        // 2: high nibbles of bytes 0..7 (elements 16..23), 3: of bytes 8..15
                        const uint4 w = *reinterpret_cast<const uint4 *>(nrow + ((uint32_t)j ^ (flip & (uint32_t)jr)) * 16);
                        uint4 *ablk = reinterpret_cast<uint4 *>(base + TC_OFF_A + j * TC_BLK_BYTES) + r;
                        const uint2 c0a = nib_f16x4(w.x & 0x0F0F0F0Fu), c0b = nib_f16x4(w.y & 0x0F0F0F0Fu);
                        const uint2 c1a = nib_f16x4(w.z & 0x0F0F0F0Fu), c1b = nib_f16x4(w.w & 0x0F0F0F0Fu);
                        const uint2 c2a = nib_f16x4((w.x >> 4) & 0x0F0F0F0Fu), c2b = nib_f16x4((w.y >> 4) & 0x0F0F0F0Fu);
                        const uint2 c3a = nib_f16x4((w.z >> 4) & 0x0F0F0F0Fu), c3b = nib_f16x4((w.w >> 4) & 0x0F0F0F0Fu);
                        ablk[0 * TC_M] = make_uint4(c0a.x, c0a.y, c0b.x, c0b.y);
                        ablk[1 * TC_M] = make_uint4(c1a.x, c1a.y, c1b.x, c1b.y);
                        ablk[2 * TC_M] = make_uint4(c2a.x, c2a.y, c2b.x, c2b.y);
                        ablk[3 * TC_M] = make_uint4(c3a.x, c3a.y, c3b.x, c3b.y);
                    }
                }
                fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's reads
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);  // the stage's A operand is ready
                if (tid == 64) TC_TRACE(6, sc, 2);
            }
        }
    } else {
        // ---------------------------------------------------------- epilogue
        // Warp w (w = 4 .. 19) holds tensor-memory lanes 32 q .. + 31 (q = w % 4: one weight row per
        // thread) and positions pb .. pb + 31 (pb = 32 ((w - 4) / 4)) of every block. Each warp waits
        // for the buffers on its own and hands each one back as soon as its dots are in registers.
        const int q = warp & 3, kq = (warp - 4) >> 2, pb = TC_EPI_POS * kq;
        const bool leader = warp == 4;
        const int r = 32 * q + lane;  // this thread's weight row in the tile
        const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)pb;
        const uint64_t nz2 = a.negzero2;
        int sc = 0, bc = 0;
        bool ok = true;
        // the output exchange's meeting point (named barrier 1 of the epilogue warps); the leader
        // alone reads the abort flag, so every epilogue warp takes the same decision
        auto rendezvous = [&]() -> bool {
            if (leader && lane == 0) epi_ok = *abort ? 0 : 1;
            epi_bar();
            const bool w = *reinterpret_cast<volatile int *>(&epi_ok) != 0;
            epi_bar();
            return w;
        };
        for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
            int e, nt, p0, row0;
            if (!tc_tile(a, L, e, nt, p0, row0)) {
                if (tid == TC_THREADS - 1) set_status(a.status, STATUS_BAD_INDEX);
                continue;
            }
            const bool has = pb < nt;  // this warp's positions hold tokens
            uint64_t acc[TC_EPI_POS / 2];  // positions pb + 2 m, + 1 as f32 pairs
#pragma unroll
            for (int m = 0; m < TC_EPI_POS / 2; ++m) acc[m] = 0ull;
            for (int st = 0; st < nst && ok; ++st, ++sc) {
                const int s = sc % TC_STAGES;
                const uint32_t par = (uint32_t)((sc / TC_STAGES) & 1);
                if (!(ok = tc_wait_warp(&full[s], par, abort, a.status)))
                    break;
                const uint32_t sdx = sbase + s * TC_STAGE_BYTES + TC_OFF_DX + 4 * pb;  // this warp's positions
                const uint32_t sdw = sbase + s * TC_STAGE_BYTES + TC_OFF_DW + 4 * r;   // this row's scales
                const int kn = min(TC_KB, nblk - st * TC_KB);
                for (int j = 0; j < kn; ++j, ++bc) {
                    const int tb = bc & (TC_TBUF - 1);
                    if (!(ok = tc_wait_warp(&tfull[tb], (uint32_t)((bc / TC_TBUF) & 1), abort, a.status))) break;
                    if (lane == 0 && (warp == 4 || warp == 19)) TC_TRACE(5, bc, warp == 4 ? 2 : 4);
                    tc_fence_after();
                    uint64_t t[TC_EPI_POS / 2];  // this block's dots of positions pb + 2 m, + 1 (exact f32 pairs)
                    if (has) tmem_ld32_pairs(trow + (uint32_t)(tb * TC_N), t);
                    // the block's dots are in registers: hand the buffer back to the MMAs before the
                    // arithmetic, so that the next MMA into it overlaps this block's epilogue
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[tb]);
                    if (has) {
                        if (MODE == PF_RAW) {
                            // raw block dots of the first tile: [block][position][row] int32
                            if (L == 0) {
                                int *out = reinterpret_cast<int *>(a.y) + (size_t)(st * TC_KB + j) * TC_N * TC_M;
#pragma unroll
                                for (int m = 0; m < TC_EPI_POS / 2; ++m) {
                                    out[(pb + 2 * m) * TC_M + r] = (int)f2x_lo(t[m]);
                                    out[(pb + 2 * m + 1) * TC_M + r] = (int)f2x_hi(t[m]);
                                }
                            }
                        } else {
                            const uint64_t dw2 = lds_splat(sdw + j * (TC_M * 4));
                            const uint32_t dxj = sdx + j * (TC_N * 4);
#pragma unroll
                            for (int m = 0; m < TC_EPI_POS / 4; ++m) {
                                uint64_t d01, d23;  // the scales of 4 positions (broadcast), as two pairs
                                lds_2x2(dxj + 16 * m, d01, d23);
                                const uint64_t s0 = f2x_mul(dw2, d01);
                                const uint64_t s1 = f2x_mul(dw2, d23);
                                acc[2 * m] = f2x_add(acc[2 * m], f2x_prod(t[2 * m], s0, nz2));
                                acc[2 * m + 1] = f2x_add(acc[2 * m + 1], f2x_prod(t[2 * m + 1], s1, nz2));
                            }
                        }
                    }
                    if (lane == 0 && (warp == 4 || warp == 19)) TC_TRACE(5, bc, warp == 4 ? 3 : 5);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);  // done with the stage's scales
                if (lane == 0 && warp == 4) TC_TRACE(6, sc, 4);
            }
            if (!ok) break;
            // ------------------------------------------------------ tile outputs
            if (MODE == PF_DN) {
                if (has) {
#pragma unroll
                    for (int m = 0; m < TC_EPI_POS / 2; ++m) {
                        const int pos = pb + 2 * m;
                        float *yp = a.y + (size_t)(p0 + pos) * a.n_embd + row0 + r;
                        if (pos < nt) yp[0] = f2x_lo(acc[m]);
                        if (pos + 1 < nt) yp[a.n_embd] = f2x_hi(acc[m]);
                    }
                }
            } else if (MODE == PF_GU) {
                // Rows 64 u .. + 63 of the tile are h block (row0 / 64 + u): gate column i at row
                // 64 u + i (lane quarter 2 u), up column i at 64 u + 32 + i (quarter 2 u + 1), so
                // lane i of the gate warp and of the up warp of a position group hold gate and up of
                // the same column. The gate warp hands the up warp its gate values of the group's
                // last half of the positions, the up warp hands the gate warp its up values of the
                // first half; then each forms h = gelu(gate) * up for its half and quantises each
                // position's 32 columns (one per lane) to a Q8_0 block as quant_q8_lane does
                // (ops.rs:95-105).
                constexpr int HP = TC_EPI_POS / 2;  // positions each of the pair computes
                const int u = q >> 1;
                const bool gate = (q & 1) == 0;
                float *xg = reinterpret_cast<float *>(smem + TC_OFF_STG + (u * (TC_EPI_WARPS / 4) + kq) * TC_STG_PAIR);
                float *xu = xg + HP * 32;  // xg: gate of the last HP positions; xu: up of the first HP
                if (!(ok = rendezvous())) break;  // the exchange area is free
                if (has) {
#pragma unroll
                    for (int m = 0; m < HP / 2; ++m) {
                        const uint64_t v = gate ? acc[HP / 2 + m] : acc[m];
                        float *dst = (gate ? xg : xu) + (2 * m) * 32 + lane;
                        dst[0] = f2x_lo(v);
                        dst[32] = f2x_hi(v);
                    }
                }
                if (!(ok = rendezvous())) break;
                if (has) {
                    const int hrb = pf_rec_bytes(a.nh);
                    const int hb = (row0 >> 6) + u;  // h block within the expert's ff columns
                    const int t0 = pb + (gate ? 0 : HP);
                    for (int i0 = 0; i0 < HP && t0 + i0 < nt; i0 += 8) {  // 8 positions at a time
                        float hv[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint64_t mine = gate ? acc[(i0 + i) >> 1] : acc[HP / 2 + ((i0 + i) >> 1)];
                            const float own = ((i0 + i) & 1) ? f2x_hi(mine) : f2x_lo(mine);
                            const float other = (gate ? xu : xg)[(i0 + i) * 32 + lane];
                            const float g = gate ? own : other, uv = gate ? other : own;
                            hv[i] = __fmul_rn(gelu_tanh(g), uv);
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int tok = t0 + i0 + i;
                            if (tok >= nt) break;  // warp-uniform
                            // the block's largest magnitude: non-negative floats order as their bit patterns
                            const float amax =
                                __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(hv[i]))));
                            const float d = __fdiv_rn(amax, 127.0f);
                            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                            const float rr = roundf(__fmul_rn(hv[i], id));
                            const int qq = rr != rr ? 0 : (rr > 127.0f ? 127 : (rr < -128.0f ? -128 : (int)rr));
                            // the quant as an f16 integer (the down GEMM's B operand), and the block scale
                            uint16_t *rec = reinterpret_cast<uint16_t *>(a.hrec + (size_t)(p0 + tok) * hrb);
                            rec[hb * 32 + lane] = __half_as_ushort(__int2half_rn(qq));
                            if (lane == 0) a.hsc[(size_t)hb * a.ppad + p0 + tok] = f16_bits_to_f32(f32_to_f16_bits(d));
                        }
                    }
                }
            }
        }
    }
    // ------------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, TC_TBUF * TC_N);
}

}  // namespace rvc
