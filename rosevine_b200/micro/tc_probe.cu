// tc_probe.cu - microbenchmarks behind the prefill GEMM's design on B200 (sm_100a).
//
// The grouped expert GEMM needs, per (weight row, position, 32-column block), one exact int32
// block dot (a tensor-core job) and a few f32 operations on the CUDA cores that scale and
// accumulate it. Which unit bounds that mix depends on four rates this program measures, each
// timed with clock64 inside the kernel and with CUDA events around it, one CTA per SM:
//
//   tmem    tcgen05.mma kind::i8 (M = 128, N = 128 or 256, K = 32) issued back to back by one
//           thread, tcgen05.ld 32x32b.x32 issued in a loop by 4 or 8 warps, and both at once on
//           disjoint tensor-memory columns: does a tensor-memory load wait for the MMAs in
//           flight, or do the two overlap?
//   pipe    the GEMM's skeleton: MMAs into a ring of tensor-memory buffers, epilogue warps that
//           load each buffer (optionally with the per-value scale and accumulate arithmetic)
//           and hand it back; cycles per MMA at steady state.
//   cvt     cvt.rn.f32.s32 (int32 block dot to f32) throughput per SM per clock.
//   f32x2   mul.rn / add.rn / fma.rn .f32x2 throughput (f32 lane operations per SM per clock).
//
// Build and run (on a B200):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -o tc_probe tc_probe.cu
//   ./tc_probe
// Every mbarrier wait is bounded; a wait that runs out sets a flag the host reports.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>

#define CK(x)                                                                                   \
    do {                                                                                        \
        cudaError_t e_ = (x);                                                                   \
        if (e_ != cudaSuccess) {                                                                \
            fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cudaGetErrorString(e_));          \
            exit(1);                                                                            \
        }                                                                                       \
    } while (0)

namespace {

constexpr long long kSpin = 1ll << 24;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t par) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok)
                 : "r"(smem_u32(b)), "r"(par)
                 : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t par, int *flag) {
    for (long long i = 0; i < kSpin; ++i)
        if (mbar_try(b, par)) return true;
    atomicOr(flag, 1);
    return false;
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, no swizzle: 8-row x 16-byte core matrices; lbo = bytes between the two 16-byte K
// halves, sbo = bytes between 8-row groups.
__device__ __forceinline__ uint64_t desc(const void *p, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_u32(p);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}
// kind::i8: s32 accumulator, A and B signed, both K-major
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
// The same MMA issued from a converged warp: every lane executes the instruction's operands
// (warp-uniform values), elect.sync picks the one lane that issues it.
__device__ __forceinline__ void mma_i8_elect(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit_elect(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

#define LD32_OUTS                                                                                              \
    "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), \
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),  \
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
#define LD32_INOUTS                                                                                            \
    "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), \
        "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]),  \
        "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), \
        "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])

__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : LD32_OUTS
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void ld_wait(uint32_t (&v)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : LD32_INOUTS : : "memory");
}

__device__ __forceinline__ uint64_t f2x_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm volatile("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2x_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm volatile("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2x_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm volatile("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}

constexpr int NWARPS = 9;  // warps 0..7: tensor-memory loads; warp 8: MMA issue
constexpr int SMEM_A = 128 * 32, SMEM_B = 256 * 32;
constexpr int SMEM_BYTES = 150 * 1024;  // more than half an SM's shared memory: one CTA per SM

struct ProbeOut {
    long long mma_cyc, ld_cyc;  // cycles of the MMA thread's loop, max over load warps
    long long mma_n, ld_n;      // MMAs issued, loads per load warp
    unsigned long long t0, t1;  // global timer around the CTA's work
    float sink;
    int pad;
};

// mode 1: MMAs only; 2: loads only; 3: both at once (MMAs into columns 256..511, loads from
// 0..255). mode 4: ring pipeline (MMA -> full[b] -> loads -> empty[b]); mode 5: the same with
// the epilogue arithmetic (cvt, scale product, product, sum per value).
__global__ void __launch_bounds__(NWARPS * 32, 1) k_tmem(int mode, int n, int nldw, int iters, ProbeOut *out,
                                                        int *flag) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t full[4], empty[4], done;
    __shared__ uint32_t taddr_s;
    __shared__ __align__(16) float dx_s[256];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < (SMEM_A + SMEM_B) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t *>(smem)[i] = (uint32_t)(i * 2654435761u) ^ 0x5A5A5A5Au;
    for (int i = tid; i < 256; i += blockDim.x) dx_s[i] = 1.0f + i * (1.0f / 1024);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const int nb = 512 / n;  // ring buffers of n columns
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&taddr_s)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int b = 0; b < 4; ++b) mbar_init(&full[b], 1), mbar_init(&empty[b], nldw);
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t taddr = taddr_s;
    const uint64_t da = desc(smem, 128 * 16, 128), db = desc(smem + SMEM_A, (uint32_t)n * 16, 128);
    const uint32_t id = idesc_i8(128, n);
    long long mma_cyc = 0, ld_cyc = 0;
    float sink = 0.0f;
    unsigned long long g0, g1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
    if (warp == 8 && lane == 0 && (mode & 1 || mode >= 4)) {
        const long long c0 = clock64();
        bool ok = true;
        for (int i = 0; i < iters && ok; ++i) {
            uint32_t dcol;
            if (mode >= 4) {
                const int b = i % nb;
                if (i >= nb) ok = mbar_wait(&empty[b], (uint32_t)((i / nb - 1) & 1), flag);
                tc_after();
                dcol = (uint32_t)(b * n);
                mma_i8(taddr + dcol, da, db, id, 0u);
                mma_commit(&full[b]);
            } else {
                dcol = 256u + (n == 256 ? 0u : (uint32_t)((i & 1) * n));
                mma_i8(taddr + dcol, da, db, id, 0u);
            }
        }
        mma_commit(&done);
        mbar_wait(&done, 0, flag);
        mma_cyc = clock64() - c0;
    }
    if (warp < nldw && (mode & 2 || mode >= 4)) {
        const uint32_t lrow = (uint32_t)(32 * (warp & 3)) << 16;
        const long long c0 = clock64();
        uint32_t acc = 0;
        if (mode < 4) {
            for (int i = 0; i < iters; ++i) {
                uint32_t v[32];
                ld32(taddr + lrow + (uint32_t)((i & 7) * 32), v);
                ld_wait(v);
                acc ^= v[0] ^ v[31];
            }
        } else {
            // this warp's columns of a buffer: all n (4 warps) or half (8 warps)
            const int cols = nldw == 8 ? n / 2 : n;
            const int c_off = nldw == 8 ? (warp >> 2) * cols : 0;
            uint64_t accf[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) accf[k] = 0ull;
            const uint64_t dw2 = pack2(0.013f, 0.013f);
            bool ok = true;
            for (int i = 0; i < iters && ok; ++i) {
                const int b = i % nb;
                if (lane == 0) ok = mbar_wait(&full[b], (uint32_t)((i / nb) & 1), flag);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                tc_after();
                for (int c = 0; c < cols; c += 64) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t v[32];
                        ld32(taddr + lrow + (uint32_t)(b * n + c_off + c + 32 * h), v);
                        ld_wait(v);
                        if (mode == 5) {
                            const float2 *dx = reinterpret_cast<const float2 *>(dx_s + c_off + c + 32 * h);
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const float2 d2 = dx[k];
                                const uint64_t t =
                                    pack2(__int2float_rn((int)v[2 * k]), __int2float_rn((int)v[2 * k + 1]));
                                const uint64_t s = f2x_mul(dw2, pack2(d2.x, d2.y));
                                accf[16 * h + k] = f2x_add(accf[16 * h + k], f2x_mul(t, s));
                            }
                        } else {
                            acc ^= v[0] ^ v[31];
                        }
                    }
                }
                tc_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[b]);
            }
#pragma unroll
            for (int k = 0; k < 32; ++k) sink += __uint_as_float((uint32_t)accf[k]);
        }
        ld_cyc = clock64() - c0;
        sink += (float)acc;
    }
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));
    __shared__ long long s_ld;
    if (tid == 0) s_ld = 0;
    __syncthreads();
    if (warp < nldw) atomicMax((unsigned long long *)&s_ld, (unsigned long long)ld_cyc);
    tc_before();
    __syncthreads();
    tc_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(512) : "memory");
    if (warp == 8 && lane == 0) {
        ProbeOut &o = out[blockIdx.x];
        o.mma_cyc = mma_cyc;
        o.ld_cyc = s_ld;
        o.mma_n = (mode & 1 || mode >= 4) ? iters : 0;
        o.ld_n = (mode & 2 || mode >= 4) ? iters : 0;
        o.t0 = g0, o.t1 = g1;
        o.sink = sink;
    }
    if (warp < nldw && lane == 0 && sink == 12345.0f) out[blockIdx.x].pad = 1;
}

// cvt.rn.f32.s32: 8 independent chains per thread (the bits of each result converted again)
__global__ void __launch_bounds__(1024) k_cvt(int iters, long long *cyc, int *sink) {
    int v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = threadIdx.x * 8 + j;
    const long long c0 = clock64();
    for (int i = 0; i < iters; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __float_as_int(__int2float_rn(v[j]));
    const long long c1 = clock64();
    int s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s ^= v[j];
    if (s == 0x12345678) sink[0] = s;
    if (threadIdx.x == 0) cyc[blockIdx.x] = c1 - c0;
}

// f32x2 throughput: OP 0 mul, 1 add, 2 fma; 8 independent chains of f32 pairs per thread
template <int OP>
__global__ void __launch_bounds__(1024) k_f2(int iters, long long *cyc, int *sink) {
    uint64_t a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = pack2(1.0f + threadIdx.x * 1e-6f + j * 1e-3f, 1.0f - j * 1e-3f);
    const uint64_t b = pack2(0.99999f, 1.00001f), c = pack2(1e-7f, -1e-7f);
    const long long c0 = clock64();
    for (int i = 0; i < iters; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = OP == 0 ? f2x_mul(a[j], b) : OP == 1 ? f2x_add(a[j], c) : f2x_fma(a[j], b, c);
    const long long c1 = clock64();
    uint64_t s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s ^= a[j];
    if (s == 0x12345678ull) sink[0] = 1;
    if (threadIdx.x == 0) cyc[blockIdx.x] = c1 - c0;
}

// Shared-memory descriptor with a layout type (0 none, 6 32-byte swizzle, 2 128-byte swizzle)
__device__ __forceinline__ uint64_t desc_l(const void *p, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return desc(p, lbo, sbo) | ((uint64_t)layout << 61);
}
// kind::f16 with f16 A and B, f32 accumulator, both K-major
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}

// MMA rate and latency. kind 0: i8 (K = 32), 1: f16 (K = 16); both read 32 bytes of K per row.
// layout 0: no swizzle (8-row x 16-byte core matrices, K halves lbo apart); 6: 32-byte swizzle
// (32-byte rows, 8-row groups 256 B apart); 2: 128-byte swizzle (128-byte rows, 8-row groups
// 1024 B apart, the MMA reads the first 32 bytes). The operands' contents are arbitrary bytes:
// only the time is measured. lat = 1: one MMA at a time (issue, commit, wait) - its latency.
__global__ void __launch_bounds__(128) k_mma(int kind, int layout, int m, int n, int iters, int lat, int issuers,
                                            int kchain, int tcols, int uni, ProbeOut *out, int *flag) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // swizzle atoms: 1024-aligned
    __shared__ uint64_t done[2];
    __shared__ uint32_t taddr_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pitch = layout == 2 ? 128 : 32;  // row pitch of the swizzled layouts
    uint8_t *sa = smem, *sb = smem + 128 * 128;
    for (int i = tid; i < (128 * 128 + 256 * 128) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t *>(smem)[i] = (uint32_t)(i * 2654435761u) & 0x3C3C3C3Cu;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&taddr_s)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(&done[0], 1), mbar_init(&done[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t taddr = taddr_s;
    if (warp < issuers && (uni || lane == 0)) {
        uint64_t da, db;
        if (layout == 0) {
            da = desc_l(sa, 128 * 16, 128, 0), db = desc_l(sb, (uint32_t)n * 16, 128, 0);
        } else {
            da = desc_l(sa, 16, 8 * pitch, (uint32_t)layout), db = desc_l(sb, 16, 8 * pitch, (uint32_t)layout);
        }
        const uint32_t id = kind == 0 ? idesc_i8(m, n) : idesc_f16(m, n);
        const uint32_t half = (uint32_t)(tcols / 2);  // two D buffers of tcols / 2 columns
        const long long c0 = clock64();
        bool ok = true;
        if (uni) {  // the whole warp runs the loop; one elected lane issues
            for (int i = warp; i < iters && ok; i += issuers) {
                const uint32_t d = taddr + (uint32_t)(((i / kchain) & 1) * half);
                const uint32_t acc = (i % kchain) != 0;
                const uint64_t koff = layout == 2 ? (uint64_t)((i % kchain) & 3) * 2 : 0;
                mma_i8_elect(d, da + koff, db + koff, id, acc);
                if (lat) {
                    mma_commit_elect(&done[warp]);
                    ok = mbar_wait(&done[warp], (uint32_t)((i / issuers) & 1), flag);
                }
            }
            if (!lat) {
                mma_commit_elect(&done[warp]);
                mbar_wait(&done[warp], 0, flag);
            }
        } else {
            for (int i = warp; i < iters && ok; i += issuers) {
                const uint32_t d = taddr + (uint32_t)(((i / kchain) & 1) * half);
                const uint32_t acc = (i % kchain) != 0;
                // successive MMAs of a chain read successive 32-byte K slices of a 128-byte row
                const uint64_t koff = layout == 2 ? (uint64_t)((i % kchain) & 3) * 2 : 0;
                if (kind == 0)
                    mma_i8(d, da + koff, db + koff, id, acc);
                else
                    mma_f16(d, da + koff, db + koff, id, acc);
                if (lat) {
                    mma_commit(&done[warp]);
                    ok = mbar_wait(&done[warp], (uint32_t)((i / issuers) & 1), flag);
                }
            }
            if (!lat) {
                mma_commit(&done[warp]);
                mbar_wait(&done[warp], 0, flag);
            }
        }
        const long long c1 = clock64();
        if (warp == 0 && lane == 0) {
            ProbeOut &o = out[blockIdx.x];
            o.mma_cyc = c1 - c0;
            o.mma_n = iters;
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(tcols) : "memory");
}

int g_sms = 148;

double run_simple(void (*k)(int, long long *, int *), int iters, const char *name, double ops_per_thread_iter) {
    long long *cyc;
    int *sink;
    CK(cudaMalloc(&cyc, g_sms * sizeof(long long)));
    CK(cudaMalloc(&sink, 4));
    k<<<g_sms, 1024>>>(iters / 10, cyc, sink);
    CK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0));
    k<<<g_sms, 1024>>>(iters, cyc, sink);
    CK(cudaEventRecord(e1));
    CK(cudaDeviceSynchronize());
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    long long h[1024];
    CK(cudaMemcpy(h, cyc, g_sms * sizeof(long long), cudaMemcpyDeviceToHost));
    double mean = 0;
    for (int i = 0; i < g_sms; ++i) mean += (double)h[i] / g_sms;
    const double per_clk = 1024.0 * iters * ops_per_thread_iter / mean;
    printf("{\"probe\": \"%s\", \"ops_per_sm_per_clk\": %.1f, \"cycles\": %.0f, \"ms\": %.3f, \"mhz_eff\": %.0f}\n", name,
           per_clk, mean, ms, mean / (ms * 1e3));
    CK(cudaFree(cyc));
    CK(cudaFree(sink));
    return per_clk;
}

void run_tmem(int mode, int n, int nldw, int iters, int *flag) {
    ProbeOut *out;
    CK(cudaMalloc(&out, g_sms * sizeof(ProbeOut)));
    CK(cudaMemset(out, 0, g_sms * sizeof(ProbeOut)));
    k_tmem<<<g_sms, NWARPS * 32, SMEM_BYTES>>>(mode, n, nldw, iters / 10 + 8, out, flag);  // warm-up
    CK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0));
    k_tmem<<<g_sms, NWARPS * 32, SMEM_BYTES>>>(mode, n, nldw, iters, out, flag);
    CK(cudaEventRecord(e1));
    CK(cudaDeviceSynchronize());
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    ProbeOut h[1024];
    CK(cudaMemcpy(h, out, g_sms * sizeof(ProbeOut), cudaMemcpyDeviceToHost));
    int hf = 0;
    CK(cudaMemcpy(&hf, flag, 4, cudaMemcpyDeviceToHost));
    double mma = 0, ld = 0, ns = 0;
    for (int i = 0; i < g_sms; ++i) {
        mma += (double)h[i].mma_cyc / g_sms;
        ld += (double)h[i].ld_cyc / g_sms;
        ns += (double)(h[i].t1 - h[i].t0) / g_sms;
    }
    const double macs = 128.0 * n * 32;
    const double per_mma = iters ? mma / iters : 0, per_ld = iters ? ld / iters : 0;
    printf("{\"probe\": \"tmem\", \"mode\": %d, \"n\": %d, \"ld_warps\": %d, \"iters\": %d, \"cyc_per_mma\": %.1f, "
           "\"int8_macs_per_clk_per_sm\": %.0f, \"cyc_per_ld_iter\": %.1f, \"cta_ns\": %.0f, \"ms\": %.3f, "
           "\"timeout\": %d}\n",
           mode, n, nldw, iters, per_mma, per_mma > 0 ? macs / per_mma : 0.0, per_ld, ns, ms, hf);
    CK(cudaFree(out));
}


void run_mma(int kind, int layout, int m, int n, int iters, int lat, int issuers, int kchain, int ctas_per_sm,
             int *flag, int uni = 0) {
    const int ctas = g_sms * ctas_per_sm, tcols = ctas_per_sm == 1 ? 512 : 256;
    const int smem = ctas_per_sm == 1 ? SMEM_BYTES : 100 * 1024;
    ProbeOut *out;
    CK(cudaMalloc(&out, ctas * sizeof(ProbeOut)));
    CK(cudaMemset(out, 0, ctas * sizeof(ProbeOut)));
    k_mma<<<ctas, 128, smem>>>(kind, layout, m, n, iters / 10 + 4, lat, issuers, kchain, tcols, uni, out, flag);
    CK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0));
    k_mma<<<ctas, 128, smem>>>(kind, layout, m, n, iters, lat, issuers, kchain, tcols, uni, out, flag);
    CK(cudaEventRecord(e1));
    CK(cudaDeviceSynchronize());
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    ProbeOut h[1024];
    CK(cudaMemcpy(h, out, ctas * sizeof(ProbeOut), cudaMemcpyDeviceToHost));
    int hf = 0;
    CK(cudaMemcpy(&hf, flag, 4, cudaMemcpyDeviceToHost));
    double cyc = 0;
    for (int i = 0; i < ctas; ++i) cyc += (double)h[i].mma_cyc / ctas;
    const double per = cyc / iters, macs = (double)m * n * (kind == 0 ? 32 : 16);
    printf("{\"probe\": \"mma\", \"kind\": \"%s\", \"layout\": %d, \"m\": %d, \"n\": %d, \"latency_mode\": %d, "
           "\"issuers\": %d, \"kchain\": %d, \"ctas_per_sm\": %d, \"uniform_warp\": %d, \"cyc_per_mma_per_cta\": %.1f, "
           "\"macs_per_clk_per_sm\": %.0f, \"tops_or_tflops\": %.0f, \"ms\": %.3f, \"timeout\": %d}\n",
           kind == 0 ? "i8" : "f16", layout, m, n, lat, issuers, kchain, ctas_per_sm, uni, per, ctas_per_sm * macs / per,
           2.0 * macs * iters * ctas / (ms * 1e-3) / 1e12, ms, hf);
    CK(cudaFree(out));
}

}  // namespace

int main() {
    int dev = 0;
    CK(cudaSetDevice(dev));
    CK(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev));
    CK(cudaFuncSetAttribute(k_tmem, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    int *flag;
    CK(cudaMalloc(&flag, 4));
    CK(cudaMemset(flag, 0, 4));
    CK(cudaFuncSetAttribute(k_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    // kind, layout, m, n, iters, latency, issuers, kchain, ctas per SM, flag, uniform warp
    for (int n : {64, 128, 256}) run_mma(0, 2, 128, n, 4000, 0, 1, 1, 1, flag, 1);
    run_mma(0, 2, 128, 256, 4000, 0, 1, 4, 1, flag, 1);
    run_mma(0, 2, 128, 256, 4000, 0, 2, 1, 1, flag, 1);
    run_mma(0, 0, 128, 256, 4000, 0, 1, 1, 1, flag, 1);
    run_mma(0, 2, 128, 256, 500, 1, 1, 1, 1, flag, 1);    // latency
    run_mma(0, 2, 128, 128, 500, 1, 1, 1, 1, flag, 1);
    run_mma(0, 2, 128, 256, 4000, 0, 1, 1, 1, flag, 0);   // single-lane branch, for comparison
    CK(cudaFree(flag));
    return 0;
}
