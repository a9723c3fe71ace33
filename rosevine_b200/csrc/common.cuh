// common.cuh - shared device helpers for the sm_100a MoE kernels.
//
// Conventions: every spin on an mbarrier is bounded (kSpinLimit polls); a wait that
// runs out records RVC_STATUS_TIMEOUT in the status word and the kernel returns, so a
// stuck copy can never hang the GPU. Host code reads the status with rvc_status().
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace rvc {

constexpr int QK = 32;          // elements per quant block
constexpr int Q4_BLOCK = 18;    // f16 d + 16 nibble bytes (reference layout)
constexpr int Q8_BLOCK = 34;    // f16 d + 32 int8

// Device status codes (bit flags, OR-ed into the status word).
constexpr int STATUS_TIMEOUT = 1;   // a bounded wait ran out
constexpr int STATUS_BAD_INDEX = 2; // an index read from device memory was out of range
constexpr int STATUS_ROUTE_MISMATCH = 4;  // verified fast ids differ from the exact-order ids

constexpr long long kSpinLimit = 1ll << 22;  // millions of polls: far above any real wait, still bounded

// Phase timestamps for profiling builds (-DRVC_PROFILE): thread 0 of each CTA records the
// global timer (ns) at marked points of a kernel; rvc_profile_dump (profiling builds only)
// copies them out. Ordinary builds compile the marks away.
#ifdef RVC_PROFILE
__device__ unsigned long long g_prof[8][1024][8];
__device__ long long g_prof_clk[8][1024][8];  // SM clock counter at the same marks
#define RVC_MARK(K, P)                                                                             \
    do {                                                                                           \
        const unsigned b_ = blockIdx.x + blockIdx.y * gridDim.x;                                   \
        if (threadIdx.x == 0 && b_ < 1024) {                                                       \
            unsigned long long t_;                                                                 \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                 \
            ::rvc::g_prof[K][b_][P] = t_;                                                          \
            ::rvc::g_prof_clk[K][b_][P] = clock64();                                               \
        }                                                                                          \
    } while (0)
// Event trace of CTA 0 (profiling builds): slot K, index I (a block or stage counter), point P.
#define RVC_TRACE(K, I, P)                                                                         \
    do {                                                                                           \
        const int i_ = (I);                                                                        \
        if (blockIdx.x == 0 && blockIdx.y == 0 && i_ >= 0 && i_ < 1024) {                          \
            unsigned long long t_;                                                                 \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                 \
            ::rvc::g_prof[K][i_][P] = t_;                                                          \
            ::rvc::g_prof_clk[K][i_][P] = clock64();                                               \
        }                                                                                          \
    } while (0)
#else
#define RVC_TRACE(K, I, P) \
    do {                   \
    } while (0)
#define RVC_MARK(K, P) \
    do {               \
    } while (0)
#endif

__device__ __forceinline__ void set_status(int *status, int code) {
    if (status) atomicOr(status, code);
}

// ------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records a timeout) if it runs out.
__device__ __noinline__ bool fd_mbar_wait(uint64_t *bar, uint32_t parity, int *status) {
    for (long long i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    set_status(status, STATUS_TIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar` in bytes.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetch of a global range (bulk), no smem involved.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ------------------------------------------------------------------ numerics
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// Unsigned-bytes x signed-bytes 4-way dot product accumulate (dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a_unsigned, int b_signed, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_unsigned), "r"(b_signed), "r"(c));
    return d;
}

// Exact integer dot of one Q4_0 nibble block (16 bytes as 4 words, low nibbles = elements
// 0..15, high = 16..31) with one Q8_0 block (32 int8 as 8 words), including the -8 offset:
// sum_j (n_j - 8) q_j = sum_j n_j q_j - 8 sum_j q_j, with qsum = sum_j q_j precomputed.
__device__ __forceinline__ int q4q8_sumi(const uint4 nib, const int4 qa, const int4 qb, int qsum) {
    int s = dp4a_us(nib.x & 0x0F0F0F0Fu, qa.x, -8 * qsum);  // two independent chains
    int t = dp4a_us((nib.x >> 4) & 0x0F0F0F0Fu, qb.x, 0);
    s = dp4a_us(nib.y & 0x0F0F0F0Fu, qa.y, s);
    t = dp4a_us((nib.y >> 4) & 0x0F0F0F0Fu, qb.y, t);
    s = dp4a_us(nib.z & 0x0F0F0F0Fu, qa.z, s);
    t = dp4a_us((nib.z >> 4) & 0x0F0F0F0Fu, qb.z, t);
    s = dp4a_us(nib.w & 0x0F0F0F0Fu, qa.w, s);
    t = dp4a_us((nib.w >> 4) & 0x0F0F0F0Fu, qb.w, t);
    return s + t;
}

// ----------------------------------------------------------- Q8_0 row records
// A quantised activation row (x of a token, h of a pair) as one contiguous record, so that a
// row can be staged into shared memory with a single bulk copy:
//   [nblk x 16 int8: quants 0-15 of each block][nblk x 16 int8: quants 16-31 of each block]
//   [nblk x f32 scale (the f16 scale widened)][nblk x int32 sum of quants]
// nblk*40 bytes, a multiple of 16 when nblk is even. The quants' two planes put a block's halves
// 16 bytes after the previous block's: 8 threads reading blocks b0 + 11 l (l = 0..7) of one record
// (the batched gate/up rows of the decode kernel) hit 8 distinct 16-byte bank groups, where
// 32-byte blocks would put them in 4.
__host__ __device__ constexpr int q8rec_bytes(int nblk) { return nblk * 40; }

// Byte offset of quant j (0..31) of block b in a record of nblk blocks.
__host__ __device__ __forceinline__ int q8rec_q_off(int nblk, int b, int j) {
    return (j < 16 ? b * 16 : (nblk + b) * 16) + (j & 15);
}

struct Q8Rec {
    const uint8_t *p;  // start of the record
    int nblk;
    __device__ __forceinline__ int4 qa(int b) const { return *reinterpret_cast<const int4 *>(p + b * 16); }
    __device__ __forceinline__ int4 qb(int b) const { return *reinterpret_cast<const int4 *>(p + (nblk + b) * 16); }
    __device__ __forceinline__ float d(int b) const { return reinterpret_cast<const float *>(p + nblk * 32)[b]; }
    __device__ __forceinline__ int s(int b) const { return reinterpret_cast<const int *>(p + nblk * 36)[b]; }
};

// Store block b of a record from the warp that quantised it (quant_q8_lane below).
__device__ __forceinline__ void q8rec_store(uint8_t *rec, int nblk, int b, int lane, int8_t q, uint16_t dbits,
                                            int qsum) {
    rec[q8rec_q_off(nblk, b, lane)] = (uint8_t)q;
    if (lane == 0) {
        reinterpret_cast<float *>(rec + nblk * 32)[b] = __half2float(__ushort_as_half(dbits));
        reinterpret_cast<int *>(rec + nblk * 36)[b] = qsum;
    }
}

// f32 exp and tanh rounded once from their double-precision values (correctly rounded but for
// double-rounding cases far rarer than the oracle's tolerance cares about). Out of line: one
// copy of each routine per kernel, as the kernels run them only a handful of times per call.
//
// Code placement. An SM starts a kernel with the first 64 KB of its machine code at hand;
// code beyond that is fetched on demand at a few KB/us (measured on B200), which is slow for
// straight-line code that runs once per call. The decode kernels keep their hot paths in the
// first 64 KB: out-of-line device functions are laid out after the kernel body in the order of
// their mangled names, so hot helpers carry names of 10 to 19 characters ("fd_..."), which
// sort first, and rare-path helpers names of fewer than 10 ("x..."), which sort last.
__device__ __noinline__ float fd_exp_f32(float x) { return (float)exp((double)x); }
__device__ __noinline__ float fd_tanh_f32(float x) { return (float)tanh((double)x); }

// tanh-approximation GELU with the reference's constants and evaluation order
// (runtime/src/ops.rs:145-149); tanh evaluated in double and rounded once to f32.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float A = 0.044715f;
    const float S = 0.7978846f;
    float inner = __fmul_rn(__fmul_rn(S, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(A, x), x)));
    float t = fd_tanh_f32(inner);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// Q8_0 quantisation of 32 values held one per lane of a full warp (ops.rs:95-105):
// d = amax/127 (f32), stored f16 RNE; q = roundf(v * (1/d)). Returns this lane's q; the
// f16 bits of d go to *d_bits and sum of q to *qsum (all lanes).
__device__ __noinline__ int8_t quant_q8_lane(float v, uint16_t *d_bits, int *qsum) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float d = __fdiv_rn(amax, 127.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    float r = roundf(__fmul_rn(v, id));
    int q = r != r ? 0 : (r > 127.0f ? 127 : (r < -128.0f ? -128 : (int)r));
    int s = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    *d_bits = f32_to_f16_bits(d);
    *qsum = s;
    return (int8_t)q;
}

}  // namespace rvc
