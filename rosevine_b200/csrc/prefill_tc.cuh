// prefill_tc.cuh - the grouped expert GEMM of the prefill path on the 5th-generation tensor
// cores: tcgen05.mma kind::i8 into tensor memory, exact per-block scaling on the CUDA cores.
//
// Computes what the reference's CPU-experts Q8_0 path computes for every (weight row, plan
// position) pair of an expert group (runtime/src/expert_pool.rs:86-135 driving
// expert_kernel.rs:147-161):
//
//     acc = 0;  for b in blocks:  acc = acc + (float)sumi_b * (dw_b * dx_b)
//
// with sumi_b the exact int32 dot of block b's Q4_0 nibbles (minus 8) and the activation's Q8_0
// quants, and every f32 operation rounded where the reference rounds it. Then, for gate/up,
// h = gelu(gate) * up and its Q8_0 records (exec.rs:606-611, ops.rs:95-105); for down, y per
// (position, row), combined afterwards in slot order (k_pf_combine).
//
// Design, from measurements on B200 (rosevine_b200/micro/tc_probe.cu):
//   - one tcgen05.mma (M = 128 rows, N = 128 positions, K = 32) per 32-column block writes the
//     block's int32 dots to a tensor-memory buffer; four buffers of 128 columns let the MMAs run
//     ahead of the epilogue (an MMA completes about 640 cycles after issue);
//   - tensor-memory loads do not wait for MMAs in flight on other columns, so the epilogue
//     drains one buffer while the next blocks' MMAs run;
//   - the epilogue's three f32 operations per (row, position, block) on the 128 f32 lanes of an
//     SM bound the kernel: the tensor cores are idle most of the time by design. One issuing
//     warp (333 cycles per MMA) keeps up with an epilogue of about 390 cycles per block.
//
// Roles (one CTA per SM, persistent over the (row tile, position tile) list):
//   warp 0       tensor-memory allocation; TMA copies of a stage (8 blocks): weight nibbles
//                [128 rows][8 blocks][16 B], activation quants [16 K-halves][128 positions]
//                [16 B] (the MMA's K-major B layout as stored), activation scales [8][128] f32
//   warp 1       MMA issue (the whole warp runs the loop; one elected lane issues)
//   warps 2-5    nibble unpack: thread r turns row r's nibbles into signed bytes n - 8 in the
//                MMA's K-major A layout (the packed plane swizzles blocks within complete groups
//                of 8: nib_pos in pack.cuh)
//   warps 6-13   epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (one weight row
//                per thread) and one half of the 128 positions; per block and position
//                t = (float)D, s = dw * dx, p = t * s (rounded product), acc = acc + p.
// Every wait is bounded; a wait that runs out records STATUS_TIMEOUT and ends the CTA's work
// (all roles see the abort flag), after the MMAs and copies in flight have completed.
#pragma once
#include "common.cuh"
#include "pack.cuh"

#include <cuda.h>

namespace rvc {

constexpr int TC_M = 128;     // weight rows per tile (tensor-memory lanes)
constexpr int TC_N = 128;     // plan positions per tile (tensor-memory columns per buffer)
constexpr int TC_KB = 8;      // blocks per stage
constexpr int TC_STAGES = 2;  // shared-memory stages
constexpr int TC_TBUF = 4;    // tensor-memory buffers of TC_N columns
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_THREADS = (6 + TC_EPI_WARPS) * 32;
// a stage in shared memory
constexpr int TC_OFF_NIB = 0;                              // [128 rows][8 blocks][16 B] raw nibbles
constexpr int TC_OFF_B = TC_OFF_NIB + TC_M * TC_KB * 16;   // [16 halves][128 positions][16 B] quants
constexpr int TC_OFF_DX = TC_OFF_B + 2 * TC_KB * TC_N * 16;  // [8 blocks][128 positions] f32 scales
constexpr int TC_OFF_A = TC_OFF_DX + TC_KB * TC_N * 4;     // [8 blocks][2 halves][128 rows][16 B] s8
constexpr int TC_STAGE_BYTES = TC_OFF_A + TC_KB * 2 * TC_M * 16;  // 84 KB
constexpr int TC_TMA_BYTES = TC_OFF_A;                     // bytes the three copies of a stage write
// gate/up output staging: [2 units][64 positions][65] f32 (one column half at a time)
constexpr int TC_STG_PITCH = 65;
constexpr int TC_OFF_STG = TC_STAGES * TC_STAGE_BYTES;
constexpr int TC_SMEM_BYTES = TC_OFF_STG + 2 * 64 * TC_STG_PITCH * 4 + 1024;  // + alignment slack
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
    int nblk;             // K blocks (n_embd / 32 or ff / 32)
    const uint16_t *scl;  // weight scales [E][rows][nblk] f16 bits
    int nh;               // (gate/up) h blocks per pair (ff / 32)
    uint8_t *hrec;        // (gate/up) out: h Q8_0 records by plan position
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

// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), A and B signed (bits 7-9
// and 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] = A * B, issued by one elected lane of a converged warp (all lanes pass the same,
// warp-uniform operands: issuing from a one-lane branch costs about 100 more cycles per MMA).
__device__ __forceinline__ void mma_i8_elect(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred e, acc;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 acc, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, acc;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(0u)
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

// Signed bytes n - 8 of four nibble values n in 0..15 (one per byte): (n | 0x80) - 8 cannot
// borrow across bytes, and the xor restores the sign bit.
__device__ __forceinline__ uint32_t nib_s8(uint32_t n4) { return ((n4 | 0x80808080u) - 0x08080808u) ^ 0x80808080u; }

// Bounded mbarrier wait that gives up early once another role has aborted the CTA's work.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *status) {
    for (long long i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && *abort) return false;
    }
    set_status(status, STATUS_TIMEOUT);
    *abort = 1;
    return false;
}

// The same wait in every lane of a warp, with one outcome for the whole warp (the warp-wide
// tcgen05 and barrier operations that follow need all its lanes).
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort, int *status) {
    const bool r = tc_wait(bar, parity, abort, status);
    return __all_sync(0xffffffffu, r);
}

// A tile entry from k_plan, checked against the layout: false for an entry that does not fit
// (a stale or foreign workspace), which every role then skips alike.
__device__ __forceinline__ bool tc_tile(const TcArgs &a, int L, int &e, int &nt, int &p0, int &row0) {
    const int ti = L / a.row_tiles, rt = L - ti * a.row_tiles;
    const int2 td = __ldg(a.tiles + ti);
    e = td.x & 0xFF, nt = td.x >> 8, p0 = td.y, row0 = a.row_base + rt * TC_M;
    return e < a.n_experts && nt >= 1 && nt <= TC_N && p0 >= 0 && p0 + nt <= a.ppos;
}

// ------------------------------------------------------------------ the kernel
template <int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1) k_pf_gemm_tc(const __grid_constant__ CUtensorMap map_nib,
                                                              const __grid_constant__ CUtensorMap map_act,
                                                              const __grid_constant__ CUtensorMap map_dx, TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, as an offset from the shared array (keeps shared addressing)
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t full[TC_STAGES], afull[TC_STAGES], empty[TC_STAGES];
    __shared__ uint64_t tfull[TC_TBUF], tempty[TC_TBUF], drain, stg_bar;
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
            mbar_init(&full[s], 1);
            mbar_init(&afull[s], 4);                     // the four unpack warps
            mbar_init(&empty[s], 1 + TC_EPI_WARPS);      // the MMAs' commit and every epilogue warp
        }
        for (int b = 0; b < TC_TBUF; ++b) mbar_init(&tfull[b], 1), mbar_init(&tempty[b], TC_EPI_WARPS);
        mbar_init(&drain, 1);
        mbar_init(&stg_bar, TC_EPI_WARPS);
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
                const int wrow0 = e * a.rows_per_expert + row0;
                for (int st = 0; st < nst && ok; ++st, ++sc) {
                    const int s = sc % TC_STAGES;
                    if (sc >= TC_STAGES && !(ok = tc_wait(&empty[s], (uint32_t)((sc / TC_STAGES - 1) & 1), abort,
                                                          a.status)))
                        break;
                    const uint32_t base = sbase + s * TC_STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], TC_TMA_BYTES);
                    tma_load_3d(base + TC_OFF_NIB, &map_nib, 0, st * TC_KB, wrow0, &full[s]);
                    tma_load_3d(base + TC_OFF_B, &map_act, 0, p0, 2 * st * TC_KB, &full[s]);
                    tma_load_2d(base + TC_OFF_DX, &map_dx, p0, st * TC_KB, &full[s]);
                }
            }
            // copies still in flight after an abort: wait (bounded) for the last stages issued
            if (!ok)
                for (int k = sc - 1; k >= 0 && k >= sc - TC_STAGES; --k)
                    fd_mbar_wait(&full[k % TC_STAGES], (uint32_t)((k / TC_STAGES) & 1), nullptr);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issue (whole warp)
        const uint32_t idesc = idesc_i8(TC_M, TC_N);
        int sc = 0, bc = 0;
        bool ok = true;
        for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
            int e, nt, p0, row0;
            if (!tc_tile(a, L, e, nt, p0, row0)) continue;
            for (int st = 0; st < nst && ok; ++st, ++sc) {
                const int s = sc % TC_STAGES;
                const uint32_t par = (uint32_t)((sc / TC_STAGES) & 1);
                if (!(ok = tc_wait_warp(&full[s], par, abort, a.status) &&
                           tc_wait_warp(&afull[s], par, abort, a.status)))
                    break;
                tc_fence_after();
                const uint32_t base = sbase + s * TC_STAGE_BYTES;
                const int kn = min(TC_KB, nblk - st * TC_KB);
                for (int j = 0; j < kn; ++j, ++bc) {
                    const int tb = bc % TC_TBUF;
                    if (bc >= TC_TBUF &&
                        !(ok = tc_wait_warp(&tempty[tb], (uint32_t)((bc / TC_TBUF - 1) & 1), abort, a.status)))
                        break;
                    tc_fence_after();
                    // A: block j's two K halves of 128 rows x 16 B; B: K halves 2j, 2j + 1 of 128 positions
                    const uint64_t da = umma_desc(base + TC_OFF_A + j * (2 * TC_M * 16), TC_M * 16, 128);
                    const uint64_t db = umma_desc(base + TC_OFF_B + j * (2 * TC_N * 16), TC_N * 16, 128);
                    mma_i8_elect(tmem + (uint32_t)(tb * TC_N), da, db, idesc);
                    mma_commit_elect(&tfull[tb]);
                }
                if (ok) mma_commit_elect(&empty[s]);  // the stage's A and B are free once its MMAs complete
            }
        }
        // every MMA issued has completed before the tensor memory is freed
        mma_commit_elect(&drain);
        fd_mbar_wait(&drain, 0, a.status);
    } else if (warp < 6) {
        // ---------------------------------------------------------- nibble unpack (row r)
        const int r = tid - 64;
        int sc = 0;
        bool ok = true;
        for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
            int e, nt, p0, row0;
            if (!tc_tile(a, L, e, nt, p0, row0)) continue;
            for (int st = 0; st < nst && ok; ++st, ++sc) {
                const int s = sc % TC_STAGES;
                if (!(ok = tc_wait_warp(&full[s], (uint32_t)((sc / TC_STAGES) & 1), abort, a.status))) break;
                uint8_t *base = smem + s * TC_STAGE_BYTES;
                const int kn = min(TC_KB, nblk - st * TC_KB);
                const uint4 *nrow = reinterpret_cast<const uint4 *>(base + TC_OFF_NIB + r * (TC_KB * 16));
#pragma unroll
                for (int j = 0; j < TC_KB; ++j) {
                    if (j < kn) {
                        // a stage of 8 blocks is one complete group, swizzled in the packed plane
                        const uint4 w = nrow[kn == TC_KB ? (j ^ (r & 7)) : j];
                        const uint4 lo = make_uint4(nib_s8(w.x & 0x0F0F0F0Fu), nib_s8(w.y & 0x0F0F0F0Fu),
                                                    nib_s8(w.z & 0x0F0F0F0Fu), nib_s8(w.w & 0x0F0F0F0Fu));
                        const uint4 hi = make_uint4(nib_s8((w.x >> 4) & 0x0F0F0F0Fu), nib_s8((w.y >> 4) & 0x0F0F0F0Fu),
                                                    nib_s8((w.z >> 4) & 0x0F0F0F0Fu), nib_s8((w.w >> 4) & 0x0F0F0F0Fu));
                        uint4 *ablk = reinterpret_cast<uint4 *>(base + TC_OFF_A + j * (2 * TC_M * 16));
                        ablk[r] = lo;          // K half 0: elements 0..15 (low nibbles)
                        ablk[TC_M + r] = hi;   // K half 1: elements 16..31 (high nibbles)
                    }
                }
                fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's reads
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[s]);
            }
        }
    } else {
        // ---------------------------------------------------------- epilogue
        const int ew = warp - 6, q = warp & 3, hh = ew >> 2;  // lane quarter, column half
        const int r = 32 * q + lane;                           // this thread's weight row in the tile
        const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(64 * hh);
        const uint64_t nz2 = a.negzero2;
        float *stg = reinterpret_cast<float *>(smem + TC_OFF_STG);
        int sc = 0, bc = 0, sp = 0;
        bool ok = true;
        // rendezvous of the epilogue warps around the output staging (an mbarrier with a bounded
        // wait, not bar.sync: a warp that aborted must not leave the others waiting forever)
        auto rendezvous = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(&stg_bar);
            const bool r = tc_wait_warp(&stg_bar, (uint32_t)(sp & 1), abort, a.status);
            ++sp;
            return r;
        };
        for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
            int e, nt, p0, row0;
            if (!tc_tile(a, L, e, nt, p0, row0)) {
                if (tid == TC_THREADS - 1) set_status(a.status, STATUS_BAD_INDEX);
                continue;
            }
            const int nch = max(0, min(2, (nt - 64 * hh + 31) >> 5));  // 32-position chunks holding tokens
            // this row's weight scales, one stage ahead (8 f16 = four 32-bit words; a row of the
            // plane is 4-byte aligned, and words past the row's last block are not read)
            const uint32_t *srow =
                reinterpret_cast<const uint32_t *>(a.scl + (size_t)(e * a.rows_per_expert + row0 + r) * nblk);
            uint32_t wn[4];
            auto ld_dw = [&](int st) {
#pragma unroll
                for (int k = 0; k < 4; ++k) wn[k] = st * TC_KB + 2 * k < nblk ? __ldg(srow + (st * TC_KB) / 2 + k) : 0u;
            };
            uint64_t acc[2][16];
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int k = 0; k < 16; ++k) acc[c][k] = 0ull;
            ld_dw(0);
            for (int st = 0; st < nst && ok; ++st, ++sc) {
                const int s = sc % TC_STAGES;
                uint32_t wc[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) wc[k] = wn[k];
                if (st + 1 < nst) ld_dw(st + 1);  // lands during this stage
                if (!(ok = tc_wait_warp(&full[s], (uint32_t)((sc / TC_STAGES) & 1), abort, a.status))) break;
                const float *sdx = reinterpret_cast<const float *>(smem + s * TC_STAGE_BYTES + TC_OFF_DX) + 64 * hh;
                const int kn = min(TC_KB, nblk - st * TC_KB);
                for (int j = 0; j < kn; ++j, ++bc) {
                    const int tb = bc % TC_TBUF;
                    if (!(ok = tc_wait_warp(&tfull[tb], (uint32_t)((bc / TC_TBUF) & 1), abort, a.status))) break;
                    tc_fence_after();
                    const uint32_t hw = wc[j >> 1];
                    const float dw = f16_bits_to_f32((uint16_t)((j & 1) ? (hw >> 16) : (hw & 0xFFFFu)));
                    const uint64_t dw2 = f2_pack(dw, dw);
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        if (c < nch) {
                            uint32_t v[32];
                            tmem_ld32_sync(trow + (uint32_t)(tb * TC_N + 32 * c), v);
                            if (MODE == PF_RAW) {
                                // raw block dots of the first tile: [block][position][row] int32
                                if (L == 0) {
                                    int *out = reinterpret_cast<int *>(a.y) + (size_t)(st * TC_KB + j) * TC_N * TC_M;
#pragma unroll
                                    for (int k = 0; k < 32; ++k) out[(64 * hh + 32 * c + k) * TC_M + r] = (int)v[k];
                                }
                            } else {
                                const float4 *dx4 = reinterpret_cast<const float4 *>(sdx + j * TC_N + 32 * c);
#pragma unroll
                                for (int k = 0; k < 8; ++k) {
                                    const float4 d4 = dx4[k];  // the scales of 4 positions (broadcast)
                                    const uint64_t t0 = f2_pack(__int2float_rn((int)v[4 * k]), __int2float_rn((int)v[4 * k + 1]));
                                    const uint64_t t1 =
                                        f2_pack(__int2float_rn((int)v[4 * k + 2]), __int2float_rn((int)v[4 * k + 3]));
                                    const uint64_t s0 = f2x_mul(dw2, f2_pack(d4.x, d4.y));
                                    const uint64_t s1 = f2x_mul(dw2, f2_pack(d4.z, d4.w));
                                    acc[c][2 * k] = f2x_add(acc[c][2 * k], f2x_prod(t0, s0, nz2));
                                    acc[c][2 * k + 1] = f2x_add(acc[c][2 * k + 1], f2x_prod(t1, s1, nz2));
                                }
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[tb]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);  // done with the stage's scales
            }
            if (!ok) break;
            // ------------------------------------------------------ tile outputs
            if (MODE == PF_DN) {
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int pos = 64 * hh + 32 * c + 2 * k;
                        float *yp = a.y + (size_t)(p0 + pos) * a.n_embd + row0 + r;
                        if (pos < nt) yp[0] = f2x_lo(acc[c][k]);
                        if (pos + 1 < nt) yp[a.n_embd] = f2x_hi(acc[c][k]);
                    }
            } else if (MODE == PF_GU) {
                // rows 64 u .. + 63 of the tile are h block (row0 / 64 + u): gate columns at rows
                // 64 u + i, up at 64 u + 32 + i (pack.cuh interleaving). One column half at a time
                // the half's two warps per unit stage gate and up as [unit][position][64 + 1];
                // then thread (unit, position) forms h = gelu(gate) * up over the block's 32
                // columns and its Q8_0 record, as quant_q8_lane does (ops.rs:95-105).
                const int u = q >> 1, col = (q & 1) * 32 + lane;
                const int hrb = q8rec_bytes(a.nh);
                for (int half = 0; half < 2 && ok; ++half) {
                    if (!(ok = rendezvous())) break;  // the staging area is free
                    if (hh == half) {
#pragma unroll
                        for (int c = 0; c < 2; ++c)
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                float *sp = stg + ((size_t)u * 64 + 32 * c + 2 * k) * TC_STG_PITCH + col;
                                sp[0] = f2x_lo(acc[c][k]);
                                sp[TC_STG_PITCH] = f2x_hi(acc[c][k]);
                            }
                    }
                    if (!(ok = rendezvous())) break;
                    const int item = tid - 6 * 32;  // 0..255: (unit, position) pairs 0..127
                    const int iu = item >> 6, pos = item & 63, tok = 64 * half + pos;
                    if (item < 128 && tok < nt) {
                        const float *g = stg + ((size_t)iu * 64 + pos) * TC_STG_PITCH;
                        float hv[32];
                        float amax = 0.0f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            hv[i] = __fmul_rn(gelu_tanh(g[i]), g[32 + i]);
                            amax = fmaxf(amax, fabsf(hv[i]));
                        }
                        const float d = __fdiv_rn(amax, 127.0f);
                        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                        uint32_t qw[8];
                        int qs = 0;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const float rr = roundf(__fmul_rn(hv[i], id));
                            const int qq = rr != rr ? 0 : (rr > 127.0f ? 127 : (rr < -128.0f ? -128 : (int)rr));
                            qs += qq;
                            if ((i & 3) == 0) qw[i >> 2] = 0u;
                            qw[i >> 2] |= (uint32_t)(uint8_t)(int8_t)qq << (8 * (i & 3));
                        }
                        const float df = f16_bits_to_f32(f32_to_f16_bits(d));
                        const int hb = (row0 >> 6) + iu;  // h block within the expert's ff columns
                        uint8_t *rec = a.hrec + (size_t)(p0 + tok) * hrb;
                        uint4 *qd = reinterpret_cast<uint4 *>(rec + hb * 32);
                        qd[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
                        qd[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
                        reinterpret_cast<float *>(rec + a.nh * 32)[hb] = df;
                        reinterpret_cast<int *>(rec + a.nh * 36)[hb] = qs;
                        a.hsc[(size_t)hb * a.ppad + p0 + tok] = df;
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int k = 0; k < 16; ++k) acc[c][k] = 0ull;
        }
    }
    // ------------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, TC_TBUF * TC_N);
}

}  // namespace rvc
