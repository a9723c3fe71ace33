// rvcuda.cu - C ABI of the B200 MoE backend (include/rvcuda.h).
//
// Host orchestration of the MoE layer, as the reference's HipSession::layer MoE branch
// (runtime/src/hip_exec.rs:780-846) orchestrates its HIP kernels, but with routing, the
// dispatch plan and the combine on the device, all work ordered on the caller's stream,
// and no host synchronisation inside a call.
#include "../../include/rvcuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "experts_decode.cuh"
#include "pack.cuh"
#include "router.cuh"
#include "router_fast.cuh"

using namespace rvc;

namespace {

inline int launched() { return (int)cudaGetLastError(); }
inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Vector-loaded inputs must be 16-byte aligned; TMA-read buffers (packed weights, workspace)
// 256-byte aligned, as rvc_alloc / cudaMalloc return them.
bool dims_ok(const rvc_moe_weights *w) {
    return w && w->router && w->packed && aligned(w->router, 16) && aligned(w->packed, 256) && w->n_embd > 0 && w->n_embd % 256 == 0 && w->ff > 0 && w->ff % 32 == 0 &&
           w->n_experts > 0 && w->n_experts <= MAX_EXPERTS && w->used > 0 && w->used <= MAX_USED &&
           w->used <= w->n_experts && (w->router_dtype == RVC_F32 || w->router_dtype == RVC_BF16);
}

// Byte offsets of the packed planes inside the packed buffer.
struct PackedLayout {
    size_t gu_nib, gu_scl, dn_nib, dn_scl, total;
    PackedLayout(int ne, int n_embd, int ff) {
        const size_t nb = n_embd / QK, nbh = ff / QK;
        size_t o = 0;
        gu_nib = o, o = align256(o + (size_t)ne * 2 * ff * nb * 16);
        gu_scl = o, o = align256(o + (size_t)ne * 2 * ff * nb * 2);
        dn_nib = o, o = align256(o + (size_t)ne * n_embd * nbh * 16);
        dn_scl = o, o = align256(o + (size_t)ne * n_embd * nbh * 2);
        total = o;
    }
};

PackedView packed_view(const rvc_moe_weights *w) {
    PackedLayout L(w->n_experts, w->n_embd, w->ff);
    const uint8_t *b = static_cast<const uint8_t *>(w->packed);
    return PackedView{b + L.gu_nib, reinterpret_cast<const uint16_t *>(b + L.gu_scl), b + L.dn_nib,
                      reinterpret_cast<const uint16_t *>(b + L.dn_scl)};
}

// Workspace carve-up for calls of up to max_tok tokens.
struct Workspace {
    // header (first 256 B, cleared by rvc_workspace_reset): int status at 0, the K0 and K1
    // last-CTA counters at 4 and 8 (each kernel returns its counter to zero), and at 12 the
    // running count of tokens the fast router sent to its exact fallback.
    size_t status, logits, lbound, lexact0, lexact1, ids, ids_exact, wts, xrec, counts, offsets, order, pos_of,
        active, n_active, hrec, ybuf, total;
    Workspace(int max_tok, int n_embd, int ff, int ne, int used) {
        const size_t nb = n_embd / QK, nbh = ff / QK, pairs = (size_t)max_tok * used;
        size_t o = 0;
        auto take = [&](size_t bytes) {
            size_t at = o;
            o = align256(o + bytes);
            return at;
        };
        status = take(256);
        logits = take((size_t)max_tok * ne * 4);
        lbound = take((size_t)max_tok * ne * 4);
        lexact0 = take((size_t)max_tok * ne * 4);
        lexact1 = take((size_t)max_tok * ne * 4);
        ids = take(pairs * 4);
        ids_exact = take(pairs * 4);
        wts = take(pairs * 4);
        xrec = take((size_t)max_tok * q8rec_bytes((int)nb));
        counts = take((size_t)ne * 4);
        offsets = take((size_t)(ne + 1) * 4);
        order = take(pairs * 4);
        pos_of = take(pairs * 4);
        active = take((size_t)ne * 4);
        n_active = take(4);
        hrec = take(pairs * q8rec_bytes((int)nbh));
        ybuf = pairs > (size_t)DN_MAX_PAIRS ? take(pairs * n_embd * 4) : o;  // y of the expert-major path
        total = o;
    }
};

template <typename T>
T *at(void *ws, size_t off) {
    return reinterpret_cast<T *>(static_cast<uint8_t *>(ws) + off);
}

// Largest token count a workspace of `bytes` supports.
int ws_max_tok(size_t bytes, const rvc_moe_weights *w) {
    int lo = 0, hi = 1 << 22;
    while (lo < hi) {
        int mid = lo + (hi - lo + 1) / 2;
        if (Workspace(mid, w->n_embd, w->ff, w->n_experts, w->used).total <= bytes)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

constexpr int DECODE_MAX_PAIRS = 512;  // pairs per call on the decode kernels

// Opt a kernel into the dynamic shared memory it needs beyond the default 48 KB: the opt-in
// limit is the device's per-block maximum minus the kernel's static shared memory. Done once
// per (kernel slot, device); returns a CUDA error code.
template <typename K>
int set_smem_attr(K kernel, int slot) {
    static bool done[40][64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 0 && dev < 64 && done[slot][dev]) return 0;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return (int)e;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return (int)e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 0 && dev < 64) done[slot][dev] = true;
    return 0;
}

int g_num_sms[64] = {};
int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!g_num_sms[dev]) cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    return g_num_sms[dev] > 0 ? g_num_sms[dev] : 148;
}

// Tokens per K0 tile: up to 16 (8 for f32 activations, to fit the staged rows in shared memory).
template <typename XT>
int chains_tpc(int n_tok) {
    return std::min(n_tok, sizeof(XT) == 4 ? 8 : 16);
}

// K0: exact-order router chains -> lexact; with done_cnt set, the last CTA also selects ids/wts.
template <typename XT, typename WT>
int launch_chains_t(RouteArgs a, cudaStream_t st) {
    const int tpc = chains_tpc<XT>(a.n_tok);
    const size_t smem = (size_t)C0_EPC * c0_row_bytes<WT>(a.n_embd) + (size_t)tpc * c0_row_bytes<XT>(a.n_embd);
    int rc = set_smem_attr(k_router_chains<XT, WT>, 2 + 2 * (int)sizeof(XT) / 2 + (int)sizeof(WT) / 4);
    if (rc) return rc;
    dim3 grid((a.n_experts + C0_EPC - 1) / C0_EPC, (a.n_tok + tpc - 1) / tpc);
    const int threads = std::max(32, (C0_EPC * tpc + 31) / 32 * 32);
    k_router_chains<XT, WT><<<grid, threads, smem, st>>>(a, tpc);
    return launched();
}

int launch_chains(const RouteArgs &a, int x_dtype, int w_dtype, cudaStream_t st) {
    const bool xb = x_dtype == RVC_BF16, wb = w_dtype == RVC_BF16;
    if (xb && wb) return launch_chains_t<uint16_t, uint16_t>(a, st);
    if (xb) return launch_chains_t<uint16_t, float>(a, st);
    if (wb) return launch_chains_t<float, uint16_t>(a, st);
    return launch_chains_t<float, float>(a, st);
}

// K1: verified fast router + Q8_0 of x + plan (n_tok <= RF_MAX_TOK), templated on n_embd / 256.
template <typename XT, typename WT, int NB8>
int launch_route_fast_n(RouteArgs a, cudaStream_t st) {
    const size_t smem = (size_t)a.n_embd * sizeof(float);  // fallback: one x row (below 48 KB)
    k_route_fast<XT, WT, NB8><<<std::min(a.n_experts, num_sms()), RF_THREADS, smem, st>>>(a);
    return launched();
}

template <typename XT, typename WT>
int launch_route_fast_t(RouteArgs a, cudaStream_t st) {
    switch (a.n_embd / 256) {
        case 1: return launch_route_fast_n<XT, WT, 1>(a, st);
        case 2: return launch_route_fast_n<XT, WT, 2>(a, st);
        case 4: return launch_route_fast_n<XT, WT, 4>(a, st);
        case 8: return launch_route_fast_n<XT, WT, 8>(a, st);
        case 11: return launch_route_fast_n<XT, WT, 11>(a, st);
        case 16: return launch_route_fast_n<XT, WT, 16>(a, st);
        default: return RVC_ERR_UNSUPPORTED;
    }
}

int launch_route_fast(const RouteArgs &a, int x_dtype, int w_dtype, cudaStream_t st) {
    const bool xb = x_dtype == RVC_BF16, wb = w_dtype == RVC_BF16;
    if (xb && wb) return launch_route_fast_t<uint16_t, uint16_t>(a, st);
    if (xb) return launch_route_fast_t<uint16_t, float>(a, st);
    if (wb) return launch_route_fast_t<float, uint16_t>(a, st);
    return launch_route_fast_t<float, float>(a, st);
}

// Per-device side stream and fork/join events for K0, which runs beside K1 and the gate/up
// GEMV. The mutex keeps one caller's record/wait pairs together.
struct SideLane {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
SideLane g_side[64];

int side_lane(SideLane **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    SideLane &L = g_side[dev];
    if (!L.stream) {
        std::lock_guard<std::mutex> lock(L.mu);
        if (!L.stream) {
            cudaStream_t s;
            if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess) return (int)e;
            if ((e = cudaEventCreateWithFlags(&L.fork, cudaEventDisableTiming)) != cudaSuccess) return (int)e;
            if ((e = cudaEventCreateWithFlags(&L.join, cudaEventDisableTiming)) != cudaSuccess) return (int)e;
            L.stream = s;
        }
    }
    *out = &L;
    return 0;
}

int launch_select(const rvc_moe_weights *w, const float *logits, int n_tok, int32_t *ids, float *wts,
                  cudaStream_t st) {
    k_select<<<(n_tok + 7) / 8, 256, 0, st>>>(logits, n_tok, w->n_experts, w->used, ids, wts, nullptr);
    return launched();
}

}  // namespace

// Quantise rows of x to the Q8 planes (used when ids come from the caller).
namespace rvc {
template <typename XT>
__global__ void __launch_bounds__(256) k_quant_rows(const XT *__restrict__ x, int n_tok, int n_embd,
                                                    uint8_t *__restrict__ xrec) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = n_embd / QK;
    const long long total = (long long)n_tok * nb;
    for (long long i = (long long)blockIdx.x * 8 + warp; i < total; i += (long long)gridDim.x * 8) {
        const long long t = i / nb, b = i % nb;
        const float v = ld_val<XT>(x, (size_t)t * n_embd + (size_t)b * QK + lane);
        uint16_t dbits;
        int qsum;
        const int8_t q = quant_q8_lane(v, &dbits, &qsum);
        q8rec_store(xrec + (size_t)t * q8rec_bytes(nb), nb, (int)b, lane, q, dbits, qsum);
    }
}

// Block sums for the debug hook: one thread per (input, row, block), reading the packed planes
// and the reference-format Q8_0 activation blocks, through the same q4q8_sumi as the kernels.
__global__ void k_debug_block_sums(PackedView pk, int which, int expert, int n_embd, int ff,
                                   const int32_t *__restrict__ rows, int n_rows, const uint8_t *__restrict__ xq8,
                                   int n_in, int32_t *__restrict__ out) {
    const int nblk = which == 0 ? n_embd / QK : ff / QK;
    const long long total = (long long)n_in * n_rows * nblk;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i % nblk);
        const int ri = (int)((i / nblk) % n_rows);
        const int t = (int)(i / ((long long)nblk * n_rows));
        const int row = rows[ri];
        if (row < 0 || row >= (which == 0 ? 2 * ff : n_embd)) {
            out[i] = INT32_MIN;
            continue;
        }
        const uint8_t *nibp;
        if (which == 0) {
            const int s = row / ff, col = row % ff;
            const int prow = (col / 32) * 64 + s * 32 + (col % 32);
            nibp = pk.gu_nib + (((size_t)expert * 2 * ff + prow) * nblk + b) * 16;
        } else {
            nibp = pk.dn_nib + (((size_t)expert * n_embd + row) * nblk + b) * 16;
        }
        const uint4 nib = *reinterpret_cast<const uint4 *>(nibp);
        const uint8_t *xb = xq8 + ((size_t)t * nblk + b) * Q8_BLOCK + 2;
        int qv[8];
        int qsum = 0;
        for (int j = 0; j < 8; ++j) {
            uint32_t wv = 0;
            for (int k = 0; k < 4; ++k) {
                const int8_t q = (int8_t)xb[4 * j + k];
                qsum += q;
                wv |= (uint32_t)(uint8_t)q << (8 * k);
            }
            qv[j] = (int)wv;
        }
        out[i] = q4q8_sumi(nib, make_int4(qv[0], qv[1], qv[2], qv[3]), make_int4(qv[4], qv[5], qv[6], qv[7]), qsum);
    }
}
}  // namespace rvc

namespace {

// Expert GEMVs for n_tok <= 64 tokens: (Q8_0 of x,) plan, gate/up, down + combine.
// quantised: x already in the workspace's Q8 planes; planned: the plan is already built.
// ids_check: exact-order ids the combine verifies against (may be NULL). join: an event the
// stream waits for before the down/combine kernel (the exact weights), or NULL.
int run_experts(const rvc_moe_weights *w, const void *x_expert, int x_dtype, const int32_t *ids,
                const int32_t *ids_check, const float *wts, int n_tok, float *out, void *ws, const Workspace &L,
                bool quantised, bool planned, cudaEvent_t join, cudaStream_t st) {
    const int pairs = n_tok * w->used;
    const int nb = w->n_embd / QK, nbh = w->ff / QK;
    if (pairs > DECODE_MAX_PAIRS || nbh % 2) return RVC_ERR_UNSUPPORTED;
    int rc;
    uint8_t *xrec = at<uint8_t>(ws, L.xrec), *hrec = at<uint8_t>(ws, L.hrec);
    if (!quantised) {
        const int blocks = std::min(1184, (int)(((long long)n_tok * nb + 7) / 8));
        if (x_dtype == RVC_BF16)
            k_quant_rows<uint16_t><<<blocks, 256, 0, st>>>((const uint16_t *)x_expert, n_tok, w->n_embd, xrec);
        else
            k_quant_rows<float><<<blocks, 256, 0, st>>>((const float *)x_expert, n_tok, w->n_embd, xrec);
        if ((rc = launched())) return rc;
    }
    int *status = at<int>(ws, L.status);
    if (!planned) {
        k_plan<<<1, PLAN_THREADS, 0, st>>>(ids, pairs, w->n_experts, at<int32_t>(ws, L.counts),
                                           at<int32_t>(ws, L.offsets), at<int32_t>(ws, L.order),
                                           at<int32_t>(ws, L.pos_of), at<int32_t>(ws, L.active),
                                           at<int32_t>(ws, L.n_active), status);
        if ((rc = launched())) return rc;
    }
    PlanView plan{at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets), at<int32_t>(ws, L.order),
                  at<int32_t>(ws, L.pos_of), at<int32_t>(ws, L.active), at<int32_t>(ws, L.n_active)};
    PackedView pk = packed_view(w);
    const int max_active = std::min(w->n_experts, pairs);
    {
        const size_t smem = gu_smem_bytes(nb);
        dim3 grid(w->ff / 32, max_active);
        switch (nb / 8) {
#define RVC_GU_CASE(NB8)                                                                                  \
    case NB8:                                                                                             \
        if ((rc = set_smem_attr(k_gate_up_decode<NB8>, 16 + NB8))) return rc;                            \
        k_gate_up_decode<NB8><<<grid, 256, smem, st>>>(pk, w->ff, xrec, plan, w->used, hrec, status); \
        break;
            RVC_GU_CASE(1)
            RVC_GU_CASE(2)
            RVC_GU_CASE(4)
            RVC_GU_CASE(8)
            RVC_GU_CASE(11)
            RVC_GU_CASE(16)
#undef RVC_GU_CASE
            default:
                return RVC_ERR_UNSUPPORTED;
        }
        if ((rc = launched())) return rc;
    }
    if (pairs <= DN_MAX_PAIRS) {
        // every h record fits in shared memory: down + slot-order combine in one kernel
        const int nbuf = max_active > DN_BATCH ? 2 : 1;
        const size_t smem = dn_smem_bytes(nbh, nbuf, pairs);
        if ((rc = set_smem_attr(k_down_combine_decode, 1))) return rc;
        if (join && (rc = (int)cudaStreamWaitEvent(st, join, 0))) return rc;
        k_down_combine_decode<<<w->n_embd / DN_ROWS, 256, smem, st>>>(pk, w->n_embd, w->ff, hrec, plan, ids,
                                                                      ids_check, wts, w->down_scale, n_tok, w->used,
                                                                      nbuf, out, status);
        if ((rc = launched())) return rc;
    } else {
        // expert-major down into y, then the slot-order combine
        float *y = at<float>(ws, L.ybuf);
        if ((rc = set_smem_attr(k_down_expert, 2))) return rc;
        k_down_expert<<<dim3(w->n_embd / DE_ROWS, max_active), 256, de_smem_bytes(nbh), st>>>(pk, w->n_embd, w->ff,
                                                                                            hrec, plan, y, status);
        if ((rc = launched())) return rc;
        if (join && (rc = (int)cudaStreamWaitEvent(st, join, 0))) return rc;
        k_combine<<<dim3((w->n_embd + 255) / 256, n_tok), 256, 0, st>>>(y, plan.pos_of, ids, ids_check, wts,
                                                                         w->down_scale, w->used, w->n_embd, out,
                                                                         status);
        if ((rc = launched())) return rc;
    }
    return 0;
}

}  // namespace

extern "C" {

// ----------------------------------------------------------------- runtime
int rvc_init(int device) { return (int)cudaSetDevice(device); }

int rvc_mem_info(size_t *free_bytes, size_t *total_bytes) {
    if (!free_bytes || !total_bytes) return (int)cudaErrorInvalidValue;
    return (int)cudaMemGetInfo(free_bytes, total_bytes);
}

int rvc_alloc(size_t bytes, void **out) {
    if (!out) return (int)cudaErrorInvalidValue;
    *out = nullptr;
    return (int)cudaMalloc(out, bytes ? bytes : 1);
}

int rvc_free(void *ptr) { return ptr ? (int)cudaFree(ptr) : 0; }

int rvc_upload(void *dst, const void *src, size_t bytes) {
    return (int)cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
}

int rvc_download(void *dst, const void *src, size_t bytes) {
    return (int)cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost);
}

int rvc_copy(void *dst, const void *src, size_t bytes) {
    return (int)cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToDevice);
}

int rvc_sync(void) { return (int)cudaDeviceSynchronize(); }

const char *rvc_error_string(int code) {
    switch (code) {
        case RVC_ERR_DEVICE_TIMEOUT: return "rvcuda: a bounded device wait ran out";
        case RVC_ERR_DEVICE_INDEX: return "rvcuda: a device-side index check failed";
        case RVC_ERR_UNSUPPORTED: return "rvcuda: shape not supported by the kernels";
        case RVC_ERR_WORKSPACE: return "rvcuda: workspace too small for this call";
        default: return cudaGetErrorString((cudaError_t)code);
    }
}

int rvc_event_create(void **out) {
    if (!out) return (int)cudaErrorInvalidValue;
    cudaEvent_t e = nullptr;
    cudaError_t r = cudaEventCreate(&e);
    *out = (void *)e;
    return (int)r;
}

int rvc_event_destroy(void *ev) { return ev ? (int)cudaEventDestroy((cudaEvent_t)ev) : 0; }

int rvc_event_record(void *ev) {
    if (!ev) return (int)cudaErrorInvalidValue;
    return (int)cudaEventRecord((cudaEvent_t)ev, 0);
}

int rvc_event_sync(void *ev) {
    if (!ev) return (int)cudaErrorInvalidValue;
    return (int)cudaEventSynchronize((cudaEvent_t)ev);
}

int rvc_event_elapsed(void *start, void *end, float *ms) {
    if (!start || !end || !ms) return (int)cudaErrorInvalidValue;
    return (int)cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end);
}

int rvc_upload_async(void *dst, const void *src, size_t bytes, void *stream) {
    return (int)cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, S(stream));
}

int rvc_download_async(void *dst, const void *src, size_t bytes, void *stream) {
    return (int)cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, S(stream));
}

int rvc_event_record_on(void *ev, void *stream) {
    if (!ev) return (int)cudaErrorInvalidValue;
    return (int)cudaEventRecord((cudaEvent_t)ev, S(stream));
}

int rvc_stream_sync(void *stream) { return (int)cudaStreamSynchronize(S(stream)); }

// --------------------------------------------------------------- MoE layer
size_t rvc_packed_bytes(int n_experts, int n_embd, int ff) {
    if (n_experts <= 0 || n_embd <= 0 || n_embd % QK || ff <= 0 || ff % QK) return 0;
    return PackedLayout(n_experts, n_embd, ff).total;
}

int rvc_pack_experts(const void *gate_up_q4, const void *down_q4, int n_experts, int n_embd, int ff, void *packed,
                     void *stream) {
    if (!gate_up_q4 || !down_q4 || !packed || n_experts <= 0 || n_embd <= 0 || n_embd % QK || ff <= 0 || ff % QK ||
        !aligned(gate_up_q4, 2) || !aligned(down_q4, 2) || !aligned(packed, 256))
        return (int)cudaErrorInvalidValue;
    PackedLayout L(n_experts, n_embd, ff);
    uint8_t *b = static_cast<uint8_t *>(packed);
    k_pack_q4<<<4 * 148, 256, 0, S(stream)>>>((const uint8_t *)gate_up_q4, n_experts, 2 * ff, n_embd / QK, true, ff,
                                               b + L.gu_nib, reinterpret_cast<uint16_t *>(b + L.gu_scl));
    int rc = launched();
    if (rc) return rc;
    k_pack_q4<<<4 * 148, 256, 0, S(stream)>>>((const uint8_t *)down_q4, n_experts, n_embd, ff / QK, false, ff,
                                               b + L.dn_nib, reinterpret_cast<uint16_t *>(b + L.dn_scl));
    return launched();
}

size_t rvc_moe_workspace_bytes(int max_tok, int n_embd, int ff, int n_experts, int used) {
    if (max_tok <= 0 || n_embd <= 0 || n_embd % QK || ff <= 0 || ff % QK || n_experts <= 0 || used <= 0) return 0;
    return Workspace(max_tok, n_embd, ff, n_experts, used).total;
}

int rvc_moe_router(const rvc_moe_weights *w, const void *x, int x_dtype, const float *bias, int bias_stride,
                   int n_tok, int32_t *ids, float *wts, int32_t *hist, int32_t *perm, float *logits, void *workspace,
                   size_t workspace_bytes, void *stream) {
    if (!dims_ok(w) || !x || n_tok <= 0 || !workspace || bias_stride < 0 || !aligned(x, 16) ||
        !aligned(workspace, 256) || (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used);
    cudaStream_t st = S(stream);
    float *lg = logits ? logits : at<float>(workspace, L.logits);
    int32_t *id = ids ? ids : at<int32_t>(workspace, L.ids);
    float *wt = wts ? wts : at<float>(workspace, L.wts);
    RouteArgs a{};
    a.x = x, a.w = w->router, a.bias = bias, a.bias_stride = bias_stride;
    a.n_tok = n_tok, a.n_experts = w->n_experts, a.n_embd = w->n_embd, a.used = w->used;
    a.lexact = lg, a.status = at<int>(workspace, L.status);
    int rc = launch_chains(a, x_dtype, w->router_dtype, st);  // exact-order logits
    if (rc) return rc;
    rc = launch_select(w, lg, n_tok, id, wt, st);
    if (rc) return rc;
    if (hist || perm) {
        const int pairs = n_tok * w->used;
        k_plan<<<1, PLAN_THREADS, 0, st>>>(
            id, pairs, w->n_experts, hist ? hist : at<int32_t>(workspace, L.counts), at<int32_t>(workspace, L.offsets),
            perm ? perm : at<int32_t>(workspace, L.order), at<int32_t>(workspace, L.pos_of),
            at<int32_t>(workspace, L.active), at<int32_t>(workspace, L.n_active), at<int>(workspace, L.status));
        rc = launched();
    }
    return rc;
}

int rvc_moe_experts(const rvc_moe_weights *w, const void *x_expert, int x_dtype, const int32_t *ids,
                    const float *wts, int n_tok, float *out, void *workspace, size_t workspace_bytes, void *stream) {
    if (!dims_ok(w) || !x_expert || !ids || !wts || !out || n_tok <= 0 || !workspace || !aligned(x_expert, 16) ||
        !aligned(workspace, 256) || (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used);
    return run_experts(w, x_expert, x_dtype, ids, nullptr, wts, n_tok, out, workspace, L, false, false, nullptr,
                       S(stream));
}

int rvc_moe_forward(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype,
                    const float *bias, int bias_stride, int n_tok, float *out, int32_t *ids, float *wts,
                    void *workspace, size_t workspace_bytes, void *stream) {
    if (!dims_ok(w) || !x_router || !x_expert || !out || n_tok <= 0 || !workspace || bias_stride < 0 ||
        !aligned(x_router, 16) || !aligned(x_expert, 16) || !aligned(workspace, 256) ||
        (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    if (n_tok * w->used > DECODE_MAX_PAIRS || n_tok > RF_MAX_TOK) return RVC_ERR_UNSUPPORTED;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used);
    cudaStream_t st = S(stream);
    int32_t *id = ids ? ids : at<int32_t>(workspace, L.ids);
    float *wt = wts ? wts : at<float>(workspace, L.wts);
    int *status = at<int>(workspace, L.status);
    uint8_t *hdr = static_cast<uint8_t *>(workspace);
    SideLane *lane = nullptr;
    int rc = side_lane(&lane);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(lane->mu);
    // K0 on the side lane: exact-order logits, selection and the combine weights
    if ((rc = (int)cudaEventRecord(lane->fork, st))) return rc;
    if ((rc = (int)cudaStreamWaitEvent(lane->stream, lane->fork, 0))) return rc;
    RouteArgs a0{};
    a0.x = x_router, a0.w = w->router, a0.bias = bias, a0.bias_stride = bias_stride;
    a0.n_tok = n_tok, a0.n_experts = w->n_experts, a0.n_embd = w->n_embd, a0.used = w->used;
    a0.lexact = at<float>(workspace, L.lexact0);
    a0.done_cnt = reinterpret_cast<unsigned *>(hdr + 4);
    a0.ids = at<int32_t>(workspace, L.ids_exact), a0.wts = wt, a0.status = status;
    if ((rc = launch_chains(a0, x_dtype, w->router_dtype, lane->stream))) return rc;
    if ((rc = (int)cudaEventRecord(lane->join, lane->stream))) return rc;
    // K1 on the caller's stream: verified ids, Q8_0 of x and the plan
    RouteArgs a1 = a0;
    a1.x = x_router;
    a1.lfast = at<float>(workspace, L.logits), a1.lbound = at<float>(workspace, L.lbound);
    a1.lexact = at<float>(workspace, L.lexact1);
    a1.done_cnt = reinterpret_cast<unsigned *>(hdr + 8);
    a1.fallback_cnt = reinterpret_cast<unsigned *>(hdr + 12);
    a1.ids = id, a1.wts = nullptr;
    a1.plan = PlanOut{at<int32_t>(workspace, L.counts), at<int32_t>(workspace, L.offsets),
                      at<int32_t>(workspace, L.order), at<int32_t>(workspace, L.pos_of),
                      at<int32_t>(workspace, L.active), at<int32_t>(workspace, L.n_active)};
    if (x_router == x_expert) a1.xrec = at<uint8_t>(workspace, L.xrec);
    if ((rc = launch_route_fast(a1, x_dtype, w->router_dtype, st))) return rc;
    return run_experts(w, x_expert, x_dtype, id, at<int32_t>(workspace, L.ids_exact), wt, n_tok, out, workspace, L,
                       x_router == x_expert, true, lane->join, st);
}

int rvc_workspace_reset(void *workspace, void *stream) {
    if (!workspace) return (int)cudaErrorInvalidValue;
    return (int)cudaMemsetAsync(workspace, 0, 256, S(stream));
}

int rvc_status(void *workspace, void *stream) {
    if (!workspace) return (int)cudaErrorInvalidValue;
    int rc = (int)cudaStreamSynchronize(S(stream));
    if (rc) return rc;
    int st = 0;
    rc = (int)cudaMemcpy(&st, workspace, sizeof(int), cudaMemcpyDeviceToHost);
    if (rc) return rc;
    if (st) {
        const int zero = 0;
        rc = (int)cudaMemcpy(workspace, &zero, sizeof(int), cudaMemcpyHostToDevice);
        if (rc) return rc;
    }
    if (st & STATUS_TIMEOUT) return RVC_ERR_DEVICE_TIMEOUT;
    if (st & STATUS_BAD_INDEX) return RVC_ERR_DEVICE_INDEX;
    return 0;
}

int rvc_debug_block_sums(const rvc_moe_weights *w, int which, int expert, const int32_t *rows, int n_rows,
                         const void *xq8, int n_in, int32_t *out, void *stream) {
    if (!dims_ok(w) || (which != 0 && which != 1) || expert < 0 || expert >= w->n_experts || !rows || n_rows <= 0 ||
        !xq8 || n_in <= 0 || !out)
        return (int)cudaErrorInvalidValue;
    k_debug_block_sums<<<592, 256, 0, S(stream)>>>(packed_view(w), which, expert, w->n_embd, w->ff, rows, n_rows,
                                                   (const uint8_t *)xq8, n_in, out);
    return launched();
}

}  // extern "C"

// ------------------------------------------------ fixed-scratch layer (no allocation)
// Some hosts cannot hand this library a workspace: their device memory is carved up once at
// start-up by their own allocator, or they must never risk an allocation failing (or
// synchronising the device) in the middle of a decode step. rvc_moe_forward_noalloc serves
// them from this file-scope array instead, sized RVC_NOALLOC_SCRATCH_BYTES per GPU and held
// by every GPU that loads the library until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[RVC_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {};  // device address of g_noalloc_scratch, per device ordinal

// In host code g_noalloc_scratch names a host-side stand-in, not device memory: the device
// address has to be looked up, once per device, with that device current.
int noalloc_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return (int)e;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}
}  // namespace

extern "C" int rvc_moe_forward_noalloc(const rvc_moe_weights *w, const void *x_router, const void *x_expert,
                                       int x_dtype, const float *bias, int bias_stride, int n_tok, float *out,
                                       int32_t *ids, float *wts, void *stream) {
    if (!dims_ok(w) || n_tok <= 0) return (int)cudaErrorInvalidValue;
    if (Workspace(n_tok, w->n_embd, w->ff, w->n_experts, w->used).total > (size_t)RVC_NOALLOC_SCRATCH_BYTES)
        return RVC_ERR_WORKSPACE;
    void *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // The array keeps the previous call's contents; only the status word must start at zero.
    rc = (int)cudaMemsetAsync(scratch, 0, 256, S(stream));
    if (rc) return rc;
    return rvc_moe_forward(w, x_router, x_expert, x_dtype, bias, bias_stride, n_tok, out, ids, wts, scratch,
                           RVC_NOALLOC_SCRATCH_BYTES, stream);
}

#ifdef RVC_PROFILE
// Profiling builds only: copy (and clear) the phase timestamps recorded by RVC_MARK.
extern "C" int rvc_profile_dump(void *host, size_t bytes) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(host, rvc::g_prof, bytes);
    static unsigned long long zero[8][1024][8];
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(rvc::g_prof, zero, sizeof zero);
    return (int)e;
}
#endif
