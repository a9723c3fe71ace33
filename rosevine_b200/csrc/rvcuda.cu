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
    size_t status, logits, ids, wts, xq, xd, xs, counts, offsets, order, pos_of, active, n_active, hq, hd, hs, total;
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
        ids = take(pairs * 4);
        wts = take(pairs * 4);
        xq = take((size_t)max_tok * nb * QK);
        xd = take((size_t)max_tok * nb * 4);
        xs = take((size_t)max_tok * nb * 4);
        counts = take((size_t)ne * 4);
        offsets = take((size_t)(ne + 1) * 4);
        order = take(pairs * 4);
        pos_of = take(pairs * 4);
        active = take((size_t)ne * 4);
        n_active = take(4);
        hq = take(pairs * nbh * QK);
        hd = take(pairs * nbh * 4);
        hs = take(pairs * nbh * 4);
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

constexpr int DECODE_MAX_PAIRS = 512;  // k_down_combine_decode keeps [pairs][16] f32 in smem

// Opt a kernel into the dynamic shared memory it needs beyond the default 48 KB: the opt-in
// limit is the device's per-block maximum minus the kernel's static shared memory. Done once
// per (kernel slot, device); returns a CUDA error code.
template <typename K>
int set_smem_attr(K kernel, int slot) {
    static bool done[16][64] = {};
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

int launch_router_logits(const rvc_moe_weights *w, const void *x, int x_dtype, const float *bias, int bias_stride,
                         int n_tok, float *logits, cudaStream_t st) {
    constexpr int TOK = 8;
    dim3 grid((n_tok + TOK - 1) / TOK, (w->n_experts + 127) / 128);
    const bool xb = x_dtype == RVC_BF16, wb = w->router_dtype == RVC_BF16;
    if (xb && wb)
        k_router_logits_exact<TOK, uint16_t, uint16_t><<<grid, 128, 0, st>>>(
            (const uint16_t *)x, (const uint16_t *)w->router, bias, bias_stride, n_tok, w->n_experts, w->n_embd,
            logits);
    else if (xb)
        k_router_logits_exact<TOK, uint16_t, float><<<grid, 128, 0, st>>>(
            (const uint16_t *)x, (const float *)w->router, bias, bias_stride, n_tok, w->n_experts, w->n_embd, logits);
    else if (wb)
        k_router_logits_exact<TOK, float, uint16_t><<<grid, 128, 0, st>>>(
            (const float *)x, (const uint16_t *)w->router, bias, bias_stride, n_tok, w->n_experts, w->n_embd, logits);
    else
        k_router_logits_exact<TOK, float, float><<<grid, 128, 0, st>>>(
            (const float *)x, (const float *)w->router, bias, bias_stride, n_tok, w->n_experts, w->n_embd, logits);
    return launched();
}

int launch_select_quant(const rvc_moe_weights *w, const float *logits, const void *x_expert, int x_dtype, int n_tok,
                        int32_t *ids, float *wts, int8_t *xq, float *xd, int32_t *xs, cudaStream_t st) {
    dim3 grid((n_tok + 7) / 8);
    if (x_dtype == RVC_BF16)
        k_select_quant<uint16_t><<<grid, 256, 0, st>>>(logits, (const uint16_t *)x_expert, n_tok, w->n_experts,
                                                         w->used, w->n_embd, ids, wts, nullptr, xq, xd, xs);
    else
        k_select_quant<float><<<grid, 256, 0, st>>>(logits, (const float *)x_expert, n_tok, w->n_experts, w->used,
                                                      w->n_embd, ids, wts, nullptr, xq, xd, xs);
    return launched();
}

}  // namespace

// Quantise rows of x to the Q8 planes (used when ids come from the caller).
namespace rvc {
template <typename XT>
__global__ void __launch_bounds__(256) k_quant_rows(const XT *__restrict__ x, int n_tok, int n_embd,
                                                    int8_t *__restrict__ xq, float *__restrict__ xd,
                                                    int32_t *__restrict__ xs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = n_embd / QK;
    const long long total = (long long)n_tok * nb;
    for (long long i = (long long)blockIdx.x * 8 + warp; i < total; i += (long long)gridDim.x * 8) {
        const long long t = i / nb, b = i % nb;
        const float v = ld_val<XT>(x, (size_t)t * n_embd + (size_t)b * QK + lane);
        uint16_t dbits;
        int qsum;
        const int8_t q = quant_q8_lane(v, &dbits, &qsum);
        xq[(size_t)i * QK + lane] = q;
        if (lane == 0) {
            xd[i] = f16_bits_to_f32(dbits);
            xs[i] = qsum;
        }
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

int run_experts(const rvc_moe_weights *w, const void *x_expert, int x_dtype, const int32_t *ids, const float *wts,
                int n_tok, float *out, void *ws, const Workspace &L, bool quantised, cudaStream_t st) {
    const int pairs = n_tok * w->used;
    if (pairs > DECODE_MAX_PAIRS || w->ff / QK > 32) return RVC_ERR_UNSUPPORTED;
    const int nb = w->n_embd / QK;
    int rc;
    if (!quantised) {
        const int blocks = std::min(1184, (int)(((long long)n_tok * nb + 7) / 8));
        if (x_dtype == RVC_BF16)
            k_quant_rows<uint16_t><<<blocks, 256, 0, st>>>((const uint16_t *)x_expert, n_tok, w->n_embd,
                                                           at<int8_t>(ws, L.xq), at<float>(ws, L.xd),
                                                           at<int32_t>(ws, L.xs));
        else
            k_quant_rows<float><<<blocks, 256, 0, st>>>((const float *)x_expert, n_tok, w->n_embd, at<int8_t>(ws, L.xq),
                                                        at<float>(ws, L.xd), at<int32_t>(ws, L.xs));
        if ((rc = launched())) return rc;
    }
    int *status = at<int>(ws, L.status);
    k_plan<<<1, PLAN_THREADS, 0, st>>>(ids, pairs, w->n_experts, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                                       at<int32_t>(ws, L.order), at<int32_t>(ws, L.pos_of), at<int32_t>(ws, L.active),
                                       at<int32_t>(ws, L.n_active), status);
    if ((rc = launched())) return rc;
    PlanView plan{at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets), at<int32_t>(ws, L.order),
                  at<int32_t>(ws, L.pos_of), at<int32_t>(ws, L.active), at<int32_t>(ws, L.n_active)};
    PackedView pk = packed_view(w);
    Q8View xv{at<int8_t>(ws, L.xq), at<float>(ws, L.xd), at<int32_t>(ws, L.xs)};
    {
        const size_t smem = (size_t)GU_UNIT_ROWS * nb * 18;
        if ((rc = set_smem_attr(k_gate_up_decode, 0))) return rc;
        dim3 grid(w->ff / 32, std::min(w->n_experts, pairs));
        k_gate_up_decode<<<grid, 256, smem, st>>>(pk, w->n_embd, w->ff, xv, plan, w->used, at<int8_t>(ws, L.hq),
                                                  at<float>(ws, L.hd), at<int32_t>(ws, L.hs), status);
        if ((rc = launched())) return rc;
    }
    {
        const int nbh = w->ff / QK;
        const size_t stage = ((size_t)DN_ROWS * nbh * 18 + 127) & ~size_t(127);
        const size_t smem = DN_STAGES * stage + (size_t)pairs * DN_ROWS * 4;
        if ((rc = set_smem_attr(k_down_combine_decode, 1))) return rc;
        Q8View hv{at<int8_t>(ws, L.hq), at<float>(ws, L.hd), at<int32_t>(ws, L.hs)};
        k_down_combine_decode<<<w->n_embd / DN_ROWS, 256, smem, st>>>(pk, w->n_embd, w->ff, hv, plan, ids, wts,
                                                                      w->down_scale, n_tok, w->used, out, status);
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
    int rc = launch_router_logits(w, x, x_dtype, bias, bias_stride, n_tok, lg, st);
    if (rc) return rc;
    rc = launch_select_quant(w, lg, x, x_dtype, n_tok, id, wt, nullptr, nullptr, nullptr, st);
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
    return run_experts(w, x_expert, x_dtype, ids, wts, n_tok, out, workspace, L, false, S(stream));
}

int rvc_moe_forward(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype,
                    const float *bias, int bias_stride, int n_tok, float *out, int32_t *ids, float *wts,
                    void *workspace, size_t workspace_bytes, void *stream) {
    if (!dims_ok(w) || !x_router || !x_expert || !out || n_tok <= 0 || !workspace || bias_stride < 0 ||
        !aligned(x_router, 16) || !aligned(x_expert, 16) || !aligned(workspace, 256) ||
        (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    if (n_tok * w->used > DECODE_MAX_PAIRS) return RVC_ERR_UNSUPPORTED;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used);
    cudaStream_t st = S(stream);
    float *lg = at<float>(workspace, L.logits);
    int32_t *id = ids ? ids : at<int32_t>(workspace, L.ids);
    float *wt = wts ? wts : at<float>(workspace, L.wts);
    int rc = launch_router_logits(w, x_router, x_dtype, bias, bias_stride, n_tok, lg, st);
    if (rc) return rc;
    rc = launch_select_quant(w, lg, x_expert, x_dtype, n_tok, id, wt, at<int8_t>(workspace, L.xq),
                             at<float>(workspace, L.xd), at<int32_t>(workspace, L.xs), st);
    if (rc) return rc;
    return run_experts(w, x_expert, x_dtype, id, wt, n_tok, out, workspace, L, true, st);
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
