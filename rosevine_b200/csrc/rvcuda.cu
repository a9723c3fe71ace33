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

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "common.cuh"
#include "decode_fused.cuh"
#include "dense.cuh"
#include "gguf.h"
#include "norm.cuh"
#include "pack.cuh"
#include "prefill.cuh"
#include "prefill_tc.cuh"

#include <cudaTypedefs.h>
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
// The f32 tile-major scale planes exist for shapes the prefill GEMM takes (rows per expert
// multiples of DW_TILE: 2 ff and n_embd), and are empty otherwise.
struct PackedLayout {
    size_t gu_nib, gu_scl, dn_nib, dn_scl, gu_dw, dn_dw, total;
    bool has_dw;
    PackedLayout(int ne, int n_embd, int ff) {
        const size_t nb = n_embd / QK, nbh = ff / QK;
        has_dw = (2 * ff) % DW_TILE == 0 && n_embd % DW_TILE == 0;
        size_t o = 0;
        gu_nib = o, o = align256(o + (size_t)ne * 2 * ff * nb * 16);
        gu_scl = o, o = align256(o + (size_t)ne * 2 * ff * nb * 2);
        dn_nib = o, o = align256(o + (size_t)ne * n_embd * nbh * 16);
        dn_scl = o, o = align256(o + (size_t)ne * n_embd * nbh * 2);
        gu_dw = o, o = align256(o + (has_dw ? (size_t)ne * 2 * ff * nb * 4 : 0));
        dn_dw = o, o = align256(o + (has_dw ? (size_t)ne * n_embd * nbh * 4 : 0));
        total = o;
    }
};

PackedView packed_view(const rvc_moe_weights *w) {
    PackedLayout L(w->n_experts, w->n_embd, w->ff);
    const uint8_t *b = static_cast<const uint8_t *>(w->packed);
    return PackedView{b + L.gu_nib, reinterpret_cast<const uint16_t *>(b + L.gu_scl), b + L.dn_nib,
                      reinterpret_cast<const uint16_t *>(b + L.dn_scl), reinterpret_cast<const float *>(b + L.gu_dw),
                      reinterpret_cast<const float *>(b + L.dn_dw)};
}

// Batches above PF_MIN_TOK tokens take the prefill kernels (grouped GEMMs), smaller ones the
// decode kernels (measured on B200, CUDA graphs, L2 flushed before each call, layer us decode /
// prefill kernels: 32 tokens 389 / 388, 48 tokens 502 / 500, 64 tokens 602 / 865).
constexpr int PF_MIN_TOK = 64;

// Workspace carve-up for calls of up to max_tok tokens.
struct Workspace {
    // header (first 256 B, cleared by rvc_workspace_reset): int status at 0, the router's
    // last-CTA counter at 4, at 12 the running count of tokens routed through the exact
    // fallback, and the decode kernel's grid barrier: arrival count at 64, generation at 128
    // (separate cache lines; the count returns to zero after every barrier).
    size_t status, lfast, lbound, lexact, ids, wts, sel_ids, sel_wts, sel_flag, xrec, hrec, ybuf, xperm, xd, hd,
        tiles, n_tiles, plan, counts, offsets, order, pos_of, active, n_active, total;
    // prefill plan positions: the expert groups start at multiples of 4, so at most 3 unused
    // positions per expert; ppad (a multiple of 4) is the pitch of the block-major scale planes
    size_t ppos, ppad;
    static constexpr size_t HDR_FALLBACK = 12, HDR_BAR_CNT = 64, HDR_BAR_GEN = 128;
    // prefill_above: calls of more tokens than this take the prefill kernels and get their
    // buffers (the layout of a call that goes to the decode kernels anyway has none)
    Workspace(int max_tok, int n_embd, int ff, int ne, int used, int prefill_above = PF_MIN_TOK) {
        const size_t nb = n_embd / QK, nbh = ff / QK, pairs = (size_t)max_tok * used;
        const bool prefill = max_tok > prefill_above;
        ppos = prefill ? pairs + 3 * (size_t)ne : pairs;
        ppad = (ppos + 3) / 4 * 4;
        size_t o = 0;
        auto take = [&](size_t bytes) {
            size_t at = o;
            o = align256(o + bytes);
            return at;
        };
        status = take(256);
        lfast = take((size_t)max_tok * ne * 4);
        lbound = take((size_t)max_tok * ne * 4);
        lexact = take((size_t)max_tok * ne * 4);
        ids = take(pairs * 4);
        wts = take(pairs * 4);
        sel_ids = take(pairs * 4);
        sel_wts = take(pairs * 4);
        sel_flag = take((size_t)max_tok * 4);
        xrec = take((size_t)max_tok * q8rec_bytes((int)nb));
        // h records: the decode kernels' Q8_0 records, or the prefill GEMM's f16 operand
        hrec = take(ppos * std::max(q8rec_bytes((int)nbh), pf_rec_bytes((int)nbh)));
        ybuf = take(ppos * n_embd * 4);
        // prefill calls only
        xperm = prefill ? take(ppos * pf_rec_bytes((int)nb)) : o;
        xd = prefill ? take(nb * ppad * 4) : o;   // x block scales, f32, block-major
        hd = prefill ? take(nbh * ppad * 4) : o;  // h block scales
        tiles = prefill ? take((pairs / 128 + 1 + (size_t)ne) * 8) : o;
        n_tiles = take(4);
        plan = take(fd_plan_words(std::min(max_tok, FD_MAX_TOK) * used, ne) * 4);
        counts = take((size_t)ne * 4);
        offsets = take((size_t)(ne + 1) * 4);
        order = take(ppos * 4);  // indexed by plan position
        pos_of = take(pairs * 4);
        active = take((size_t)ne * 4);
        n_active = take(4);
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
    if (a.n_tok >= C4_T && a.n_embd % C4_CH == 0 && !a.done_cnt) {  // batches: 4 chains per thread
        const size_t smem = 2 * (size_t)c4_buf_bytes<XT, WT>();
        int rc = set_smem_attr(k_router_chains4<XT, WT>, 20 + 2 * ((int)sizeof(XT) / 4) + (int)sizeof(WT) / 4);
        if (rc) return rc;
        dim3 grid((a.n_experts + C4_E - 1) / C4_E, (a.n_tok + C4_T - 1) / C4_T);
        k_router_chains4<XT, WT><<<grid, C4_THREADS, smem, st>>>(a);
        return launched();
    }
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

int launch_select(const rvc_moe_weights *w, const float *logits, int n_tok, int32_t *ids, float *wts,
                  cudaStream_t st) {
    k_select<<<(n_tok + 7) / 8, 256, 0, st>>>(logits, n_tok, w->n_experts, w->used, ids, wts, nullptr);
    return launched();
}

}  // namespace

namespace rvc {
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
            nibp = pk.gu_nib + (((size_t)expert * 2 * ff + prow) * nblk + (b ^ (prow & 7))) * 16;
        } else {
            nibp = pk.dn_nib + (((size_t)expert * n_embd + row) * nblk + nib_pos(b, nblk, row & 7)) * 16;
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

// Shared-memory plans of k_fd_route, k_fd_gate and k_fd_down for a call (FdLayout); false if
// the shapes do not fit. xs, ws: element sizes of the router input and router weight.
// smax_*: the largest dynamic shared memory each kernel may use.
bool fd_layout(int n_tok, int used, int n_embd, int ff, int ne, int G, size_t smax_gate, size_t smax_down, int xs,
               int ws, FdLayout *out) {
    FdLayout L{};
    const int nb = n_embd / QK, nbh = ff / QK, pairs = n_tok * used;
    const int xrb = q8rec_bytes(nb), hrb = q8rec_bytes(nbh);
    auto r128 = [](size_t x) { return (uint32_t)((x + 127) & ~size_t(127)); };
    if (ne > FD_MAX_EXPERTS || used > MAX_USED || n_tok > FD_MAX_TOK || pairs > FD_MAX_PAIRS) return false;
    // k_fd_route: two item buffers (router row + FD_TB x rows)
    L.r_bytes = 2 * r128((size_t)n_embd * (ws + FD_TB * xs));
    // k_fd_gate: ring of gate/up slots, two x-record buffers, a wave's dots, the plan
    L.slot_bytes = FD_ROWS * nb * 18;
    L.act_bytes = r128((size_t)xrb * std::min(n_tok, 2));
    L.act_x = L.act_bytes / xrb;
    const uint32_t gu = r128((size_t)(FD_MAX_SLOTS / 2) * L.act_x * 2 * 32 * 4);
    const uint32_t plan = r128((size_t)pairs * 5 * 4 + (size_t)(3 * ne + 1) * 4);
    const size_t fixed = 2 * (size_t)L.act_bytes + gu + plan;
    if (smax_gate < fixed + 2 * (size_t)L.slot_bytes) return false;
    L.nslot = (int)std::min<size_t>(FD_MAX_SLOTS, (smax_gate - fixed) / L.slot_bytes);
    const size_t ring = (size_t)L.nslot * L.slot_bytes;
    const size_t irow = (size_t)n_embd * (xs + ws) + 32;  // one exact-chain item: both rows, padded
    if (ring < FD_SCRATCH + irow) return false;
    L.chain_items = (int)std::min<size_t>(FD_THREADS, (ring - FD_SCRATCH) / irow);
    uint32_t o = (uint32_t)ring;
    L.off_act = o, o += 2 * L.act_bytes;
    L.off_gu = o, o += gu;
    L.off_plan = o, o += plan;
    L.bytes = o;
    // k_fd_down: ring of down slots (up to eps experts' row tiles each), two h-record buffers,
    // y (if it fits), the plan
    int g = nbh, h = 8;  // down rows per bulk-copy-aligned group: rg * nbh * 2 % 16 == 0
    while (h) {
        const int t = g % h;
        g = h, h = t;
    }
    L.rg = 8 / g;
    if (n_embd % L.rg) return false;
    const int nq = n_embd / L.rg;
    L.rpc_max = L.rg * ((nq + G - 1) / G);
    const size_t tile_max = (size_t)L.rpc_max * nbh * 18;
    L.d_slot_bytes = (int)r128(std::max(tile_max, (size_t)32768));
    L.d_act_bytes = r128((size_t)hrb * std::min(pairs, 16));
    L.act_h = L.d_act_bytes / hrb;
    const uint32_t dplan = r128((size_t)pairs * 3 * 4 + (size_t)(3 * ne + 1) * 4);
    const uint32_t y = r128((size_t)pairs * L.rpc_max * 4);
    const size_t dfixed = 2 * (size_t)L.d_act_bytes + dplan;
    if (smax_down < dfixed + 2 * (size_t)L.d_slot_bytes) return false;
    L.y_in_smem = smax_down >= dfixed + y + 4 * (size_t)L.d_slot_bytes;
    L.d_nslot = (int)std::min<size_t>(FD_MAX_SLOTS, (smax_down - dfixed - (L.y_in_smem ? y : 0)) / L.d_slot_bytes);
    o = (uint32_t)L.d_nslot * L.d_slot_bytes;
    L.d_off_act = o, o += 2 * L.d_act_bytes;
    L.d_off_y = o, o += L.y_in_smem ? y : 0;
    L.d_off_plan = o, o += dplan;
    L.d_bytes = o;
    *out = L;
    return true;
}

// Largest dynamic shared memory a kernel may use: the device's opt-in maximum per block minus
// the kernel's static shared memory. Also opts the kernel in, once per (kernel, device); the
// table of kernels seen is small and guarded by a mutex.
struct SmemOptIn {
    const void *fn;
    int dev;
    size_t dyn;
};
SmemOptIn g_optin[256];
int g_n_optin = 0;
std::mutex g_optin_mu;

template <typename K>
int fd_smem_max(K kernel, size_t *out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    const void *fn = reinterpret_cast<const void *>(kernel);
    std::lock_guard<std::mutex> lock(g_optin_mu);
    for (int i = 0; i < g_n_optin; ++i)
        if (g_optin[i].fn == fn && g_optin[i].dev == dev) {
            *out = g_optin[i].dyn;
            return 0;
        }
    if (g_n_optin == 256) return (int)cudaErrorInvalidValue;
    cudaFuncAttributes fa;
    if ((e = cudaFuncGetAttributes(&fa, kernel)) != cudaSuccess) return (int)e;
    int optin = 0;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return (int)e;
    const int dyn = optin - (int)fa.sharedSizeBytes;
    if ((e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn)) != cudaSuccess)
        return (int)e;
    g_optin[g_n_optin++] = SmemOptIn{fn, dev, (size_t)dyn};
    *out = (size_t)dyn;
    return 0;
}

// The three decode kernels on `st`, each on one CTA per SM: k_fd_route and k_fd_gate cooperative
// (all CTAs resident, for their grid barriers), k_fd_down plain; the last two as programmatic
// dependents of the kernel before them.
template <typename XT, typename WT, int NB8>
int launch_fd_n(FdArgs &a, cudaStream_t st) {
    auto kr = k_fd_route<XT, WT, NB8>;
    auto kg = k_fd_gate<XT, WT, NB8, false>;
    size_t sr = 0, sg = 0, sd = 0;
    int rc;
    size_t sw = 0;
    if ((rc = fd_smem_max(kr, &sr)) || (rc = fd_smem_max(kg, &sg)) || (rc = fd_smem_max(k_fd_gate<XT, WT, NB8, true>, &sw)) ||
        (rc = fd_smem_max(k_fd_down, &sd)))
        return rc;
    sg = std::min(sg, sw);
    const int G = num_sms();
    if (!fd_layout(a.n_tok, a.used, a.n_embd, a.ff, a.n_experts, G, sg, sd, (int)sizeof(XT), (int)sizeof(WT), &a.L) ||
        a.L.r_bytes > sr)
        return RVC_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(FD_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.dynamicSmemBytes = a.L.r_bytes;
    if ((rc = (int)cudaLaunchKernelEx(&cfg, kr, a))) return rc;
    // k_fd_gate and k_fd_down as programmatic dependents: each is launched while its predecessor
    // runs, its CTAs take SMs as the predecessor's CTAs leave, and it waits (griddepcontrol.wait)
    // for the predecessor's completion before reading what that wrote
    cudaLaunchAttribute dep[2];
    dep[0] = attr[0];
    dep[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    dep[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = dep;
    cfg.numAttrs = 2;
    cfg.dynamicSmemBytes = a.L.bytes;
    if (a.n_tok <= a.L.act_x)  // every x record fits one buffer: the small-batch gate/up kernel
        rc = (int)cudaLaunchKernelEx(&cfg, kg, a);
    else
        rc = (int)cudaLaunchKernelEx(&cfg, k_fd_gate<XT, WT, NB8, true>, a);
    if (rc) return rc;
    cfg.attrs = dep + 1;  // k_fd_down: not cooperative
    cfg.numAttrs = 1;
    cfg.dynamicSmemBytes = a.L.d_bytes;
    if ((rc = (int)cudaLaunchKernelEx(&cfg, k_fd_down, a))) return rc;
    return launched();
}

template <typename XT, typename WT>
int launch_fd_t(FdArgs &a, cudaStream_t st) {
    switch (a.n_embd / 256) {
        case 1: return launch_fd_n<XT, WT, 1>(a, st);
        case 2: return launch_fd_n<XT, WT, 2>(a, st);
        case 4: return launch_fd_n<XT, WT, 4>(a, st);
        case 8: return launch_fd_n<XT, WT, 8>(a, st);
        case 11: return launch_fd_n<XT, WT, 11>(a, st);
        case 16: return launch_fd_n<XT, WT, 16>(a, st);
        default: return RVC_ERR_UNSUPPORTED;
    }
}

// ------------------------------------------------------------------ prefill
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;

int tensor_map_encode() {
    std::lock_guard<std::mutex> lock(g_encode_mu);
    if (g_encode) return 0;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return (int)e;
    if (q != cudaDriverEntryPointSuccess || !fn) return (int)cudaErrorNotSupported;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return 0;
}

// A 2-D tensor map of bytes or f32 (d0 innermost, in elements; stride of dim 1 in bytes), box
// b0 x b1 elements, no swizzle, out-of-range elements read as zero.
int map2d(CUtensorMap *m, const void *base, uint64_t d0, uint64_t d1, uint64_t s1, uint32_t b0, uint32_t b1,
          CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8,
          CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE) {
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {s1};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// The packed nibble plane [E * rows][nblk][16 B] viewed as [g][k][j][pair][32 B] (row = 8 g + 2 k
// + j, blocks 2 pair and 2 pair + 1): a packed reshape, so every stride is the product of the
// extents inside it. Box: one pair of 16 groups' rows with key pair k (16 x 2 rows x 32 B).
int map_nibbles(CUtensorMap *m, const uint8_t *nib, uint64_t n_rows, int nblk) {
    const uint64_t row = (uint64_t)nblk * 16;
    const cuuint64_t dims[5] = {32, (cuuint64_t)nblk / 2, 2, 4, n_rows / 8};
    const cuuint64_t strides[4] = {32, row, 2 * row, 8 * row};
    const cuuint32_t box[5] = {32, 1, 2, 1, 16};
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<uint8_t *>(nib), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// The grouped GEMM's tensor maps: activation operands [positions][rec_bytes] in boxes of 128
// positions x 128 B (two blocks of f16 quants) with the 128-byte swizzle (the MMA's K-major B
// layout); activation block scales [blocks][positions] f32; the weight nibbles (map_nibbles).
struct TcMaps {
    CUtensorMap act, dx, nib;
};

int tc_maps(TcMaps *m, const uint8_t *rec, int rec_bytes, int nblk, int ppos, const float *scales, int ppad,
            const uint8_t *nib, uint64_t n_rows) {
    int rc;
    if ((rc = map2d(&m->act, rec, (uint64_t)rec_bytes, ppos, rec_bytes, TC_KB * 64, TC_N, CU_TENSOR_MAP_DATA_TYPE_UINT8,
                    CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (rc = map2d(&m->dx, scales, (uint64_t)ppad, nblk, (uint64_t)ppad * 4, TC_N, TC_KB,
                    CU_TENSOR_MAP_DATA_TYPE_FLOAT32)) ||
        (rc = map_nibbles(&m->nib, nib, n_rows, nblk)))
        return rc;
    return 0;
}

template <int MODE>
int launch_tc(const TcMaps &m, const TcArgs &g, int max_units, cudaStream_t st) {
    size_t smax = 0;
    int rc;
    if ((rc = fd_smem_max(k_pf_gemm_tc<MODE>, &smax))) return rc;
    if (smax < (size_t)TC_SMEM_BYTES) return RVC_ERR_UNSUPPORTED;
    const int grid = std::max(1, std::min(num_sms(), max_units));  // persistent: one CTA per SM
    k_pf_gemm_tc<MODE><<<grid, TC_THREADS, TC_SMEM_BYTES, st>>>(m.act, m.dx, m.nib, g);
    return launched();
}

// Gate/up and down GEMMs over the plan positions already filled (xperm records, x scale plane):
// y [positions][n_embd] in the workspace.
int pf_gemms(const rvc_moe_weights *w, const Workspace &L, void *ws, int n_pairs, cudaStream_t st) {
    int rc;
    const int ne = w->n_experts, nb = w->n_embd / QK, nbh = w->ff / QK;
    const PackedView pk = packed_view(w);
    uint8_t *xperm = at<uint8_t>(ws, L.xperm), *hrec = at<uint8_t>(ws, L.hrec);
    float *xsc = at<float>(ws, L.xd), *hsc = at<float>(ws, L.hd);
    const int ppos = (int)L.ppos, ppad = (int)L.ppad;
    TcMaps mg, md;
    if ((rc = tc_maps(&mg, xperm, pf_rec_bytes(nb), nb, ppos, xsc, ppad, pk.gu_nib, (uint64_t)ne * 2 * w->ff)) ||
        (rc = tc_maps(&md, hrec, pf_rec_bytes(nbh), nbh, ppos, hsc, ppad, pk.dn_nib, (uint64_t)ne * w->n_embd)))
        return rc;
    const int tiles_max = n_pairs / TC_N + 1 + ne;  // an upper bound on the (expert, position tile) count
    TcArgs g{};
    g.tiles = at<int2>(ws, L.tiles), g.n_tiles = at<int32_t>(ws, L.n_tiles), g.max_tiles = tiles_max;
    g.n_experts = ne, g.ppos = ppos, g.ppad = ppad, g.n_embd = w->n_embd, g.status = at<int>(ws, L.status);
    g.rows_per_expert = 2 * w->ff, g.row_tiles = 2 * w->ff / TC_M, g.nblk = nb, g.dwp = pk.gu_dw;
    g.nh = nbh, g.hrec = hrec, g.hsc = hsc;
    g.negzero2 = 0x8000000080000000ull;
    if ((rc = launch_tc<PF_GU>(mg, g, tiles_max * g.row_tiles, st))) return rc;
    TcArgs d = g;
    d.rows_per_expert = w->n_embd, d.row_tiles = w->n_embd / TC_M, d.nblk = nbh, d.dwp = pk.dn_dw;
    d.hrec = nullptr, d.hsc = nullptr, d.y = at<float>(ws, L.ybuf);
    return launch_tc<PF_DN>(md, d, tiles_max * d.row_tiles, st);
}

int pf_supported(const rvc_moe_weights *w) {
    const int nb = w->n_embd / QK, nbh = w->ff / QK;
    if (nb % TC_KB || nbh % TC_KB || (2 * w->ff) % TC_M || w->n_embd % TC_M || w->n_experts > MAX_EXPERTS ||
        w->used > MAX_USED)
        return RVC_ERR_UNSUPPORTED;
    return tensor_map_encode();
}

// Plan of n_pairs (pair -> expert ids; -1 skipped when skip_empty) into expert groups starting
// at multiples of 4 positions, with the tile list; positions within a group in arrival order.
int pf_plan(const int32_t *pair_expert, int n_pairs, int ne, const Workspace &L, void *ws, cudaStream_t st,
            bool skip_empty = false) {
    k_plan<<<1, PLAN_THREADS, 0, st>>>(pair_expert, n_pairs, ne, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                                       at<int32_t>(ws, L.order), at<int32_t>(ws, L.pos_of), at<int32_t>(ws, L.active),
                                       at<int32_t>(ws, L.n_active), at<int>(ws, L.status), 4, at<int2>(ws, L.tiles),
                                       at<int32_t>(ws, L.n_tiles), TC_N, false, skip_empty);
    return launched();
}

// The prefill layer (n_tok > 64): the reference-order router (logits, selection, plan), Q8_0
// of x in plan order, the grouped GEMMs, the slot-order combine.
// The token count of the last prefill call enqueued with each (workspace, weights) pair (host
// side, for rvc_prefill_gemms): the grouped GEMMs may only be re-run on a workspace holding the
// plan, records and scale planes of such a call, at that call's layout.
struct LastPrefill {
    const void *ws;
    const rvc_moe_weights *w;
    int n_tok;
};
std::mutex g_last_mu;
LastPrefill g_last[64];
int g_n_last = 0;

void note_prefill(const void *ws, const rvc_moe_weights *w, int n_tok) {
    std::lock_guard<std::mutex> lock(g_last_mu);
    for (int i = 0; i < g_n_last; ++i)
        if (g_last[i].ws == ws) {
            g_last[i].w = w, g_last[i].n_tok = n_tok;
            return;
        }
    if (g_n_last < 64) g_last[g_n_last++] = LastPrefill{ws, w, n_tok};
}

// Any other use of a workspace (another layout written over it, a reset, a new owner of the
// same address) ends what rvc_prefill_gemms may re-run on it.
void forget_prefill(const void *ws) {
    std::lock_guard<std::mutex> lock(g_last_mu);
    for (int i = 0; i < g_n_last; ++i)
        if (g_last[i].ws == ws) {
            g_last[i] = g_last[--g_n_last];
            return;
        }
}

int last_prefill(const void *ws, const rvc_moe_weights *w) {
    std::lock_guard<std::mutex> lock(g_last_mu);
    for (int i = 0; i < g_n_last; ++i)
        if (g_last[i].ws == ws) return g_last[i].w == w ? g_last[i].n_tok : 0;
    return 0;
}

int run_prefill(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype, const float *bias,
                int bias_stride, int n_tok, float *out, int32_t *ids, float *wts, void *ws, size_t ws_bytes,
                cudaStream_t st) {
    int rc;
    if ((rc = pf_supported(w))) return rc;
    const int ne = w->n_experts, used = w->used, pairs = n_tok * used, nb = w->n_embd / QK;
    Workspace L(n_tok, w->n_embd, w->ff, ne, used);
    int32_t *id = ids ? ids : at<int32_t>(ws, L.ids);
    float *wt = wts ? wts : at<float>(ws, L.wts);
    int32_t *pos_of = at<int32_t>(ws, L.pos_of);
    // 1. router in the reference's order, selection, plan
    if ((rc = rvc_moe_router(w, x_router, x_dtype, bias, bias_stride, n_tok, id, wt, nullptr, nullptr, nullptr, ws,
                             ws_bytes, st)) ||
        (rc = pf_plan(id, pairs, ne, L, ws, st)))
        return rc;
    // 2. Q8_0 of x, once per token, to its plan positions
    uint8_t *xperm = at<uint8_t>(ws, L.xperm);
    float *xsc = at<float>(ws, L.xd);
    const int qblocks = (n_tok * ((nb + 7) / 8) + 7) / 8;  // one warp per 8 blocks of a token
    if (x_dtype == RVC_BF16)
        k_pf_quant<uint16_t><<<qblocks, 256, 0, st>>>((const uint16_t *)x_expert, w->n_embd, n_tok, used, pos_of, xperm,
                                                      xsc, (int)L.ppad);
    else
        k_pf_quant<float><<<qblocks, 256, 0, st>>>((const float *)x_expert, w->n_embd, n_tok, used, pos_of, xperm, xsc,
                                                   (int)L.ppad);
    if ((rc = launched())) return rc;
    // 3. gate/up and down GEMMs
    if ((rc = pf_gemms(w, L, ws, pairs, st))) return rc;
    note_prefill(ws, w, n_tok);
    // 4. slot-order combine
    k_pf_combine<<<n_tok, 256, 0, st>>>(at<float>(ws, L.ybuf), pos_of, id, wt, w->down_scale, used, w->n_embd, n_tok,
                                        out, at<int>(ws, L.status));
    return launched();
}

// Workspace of an expert-parallel call of up to max_pairs (row, slot) pairs: the prefill layout
// for ceil(max_pairs / 8) tokens of 8 pairs (at least the prefill path's 65).
int ep_tokens(int max_pairs) { return std::max(PF_MIN_TOK + 1, (max_pairs + 7) / 8); }

// The decode layer for n_tok <= 64 tokens: routing from x_router (or the caller's ids/wts),
// experts on x_expert, into out.
int run_decode(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype, const float *bias,
               int bias_stride, const int32_t *ids_in, const float *wts_in, int n_tok, float *out, int32_t *ids,
               float *wts, void *ws, cudaStream_t st, int layout_above = PF_MIN_TOK) {
    if (n_tok > FD_MAX_TOK || n_tok * w->used > FD_MAX_PAIRS || w->n_embd % 256 || (w->ff / QK) % 2)
        return RVC_ERR_UNSUPPORTED;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used, layout_above);
    uint8_t *hdr = static_cast<uint8_t *>(ws);
    FdArgs a{};
    a.xr = x_router, a.xe = x_expert, a.wr = w->router, a.bias = bias, a.bias_stride = bias_stride;
    a.pk = packed_view(w);
    a.down_scale = w->down_scale;
    a.n_tok = n_tok, a.n_embd = w->n_embd, a.ff = w->ff, a.n_experts = w->n_experts, a.used = w->used;
    a.ids_in = ids_in, a.wts_in = wts_in;
    a.out = out, a.ids_out = ids, a.wts_out = wts;
    a.lfast = at<float>(ws, L.lfast), a.lbound = at<float>(ws, L.lbound), a.lexact = at<float>(ws, L.lexact);
    a.xrec = at<uint8_t>(ws, L.xrec), a.hrec = at<uint8_t>(ws, L.hrec), a.ybuf = at<float>(ws, L.ybuf);
    a.sel_ids = at<int32_t>(ws, L.sel_ids), a.sel_wts = at<float>(ws, L.sel_wts);
    a.sel_flag = at<int32_t>(ws, L.sel_flag);
    a.bar_cnt = reinterpret_cast<unsigned *>(hdr + Workspace::HDR_BAR_CNT);
    a.bar_gen = reinterpret_cast<unsigned *>(hdr + Workspace::HDR_BAR_GEN);
    a.fallback_cnt = reinterpret_cast<unsigned *>(hdr + Workspace::HDR_FALLBACK);
    a.plan = at<int32_t>(ws, L.plan);
    a.status = at<int>(ws, L.status);
    const bool xb = x_dtype == RVC_BF16, wb = w->router_dtype == RVC_BF16;
    if (xb && wb) return launch_fd_t<uint16_t, uint16_t>(a, st);
    if (xb) return launch_fd_t<uint16_t, float>(a, st);
    if (wb) return launch_fd_t<float, uint16_t>(a, st);
    return launch_fd_t<float, float>(a, st);
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

int rvc_free(void *ptr) {
    forget_prefill(ptr);  // a later allocation may reuse the address: nothing is left to re-run there
    return ptr ? (int)cudaFree(ptr) : 0;
}

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
        default:
            if (code >= RVC_ERR_GGUF && code < RVC_ERR_GGUF + rvc::gguf::kReasons)
                return rvc::gguf::reason(code - RVC_ERR_GGUF);
            return cudaGetErrorString((cudaError_t)code);
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
    if ((rc = launched()) || !L.has_dw) return rc;
    k_pack_dw<<<4 * 148, 256, 0, S(stream)>>>(reinterpret_cast<const uint16_t *>(b + L.gu_scl),
                                               (size_t)n_experts * 2 * ff, n_embd / QK, reinterpret_cast<float *>(b + L.gu_dw));
    if ((rc = launched())) return rc;
    k_pack_dw<<<4 * 148, 256, 0, S(stream)>>>(reinterpret_cast<const uint16_t *>(b + L.dn_scl),
                                               (size_t)n_experts * n_embd, ff / QK, reinterpret_cast<float *>(b + L.dn_dw));
    return launched();
}

size_t rvc_moe_workspace_bytes(int max_tok, int n_embd, int ff, int n_experts, int used) {
    if (max_tok <= 0 || n_embd <= 0 || n_embd % QK || ff <= 0 || ff % QK || n_experts <= 0 || used <= 0) return 0;
    return Workspace(max_tok, n_embd, ff, n_experts, used).total;
}

int rvc_moe_router(const rvc_moe_weights *w, const void *x, int x_dtype, const float *bias, int bias_stride,
                   int n_tok, int32_t *ids, float *wts, int32_t *hist, int32_t *perm, float *logits, void *workspace,
                   size_t workspace_bytes, void *stream) {
    forget_prefill(workspace);
    if (!dims_ok(w) || !x || n_tok <= 0 || !workspace || bias_stride < 0 || !aligned(x, 16) ||
        !aligned(workspace, 256) || (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used);
    cudaStream_t st = S(stream);
    float *lg = logits ? logits : at<float>(workspace, L.lexact);
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
    forget_prefill(workspace);
    if (!dims_ok(w) || !x_expert || !ids || !wts || !out || n_tok <= 0 || !workspace || !aligned(x_expert, 16) ||
        !aligned(workspace, 256) || (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    return run_decode(w, x_expert, x_expert, x_dtype, nullptr, 0, ids, wts, n_tok, out, nullptr, nullptr, workspace,
                      S(stream));
}

int rvc_prefill_gemms(const rvc_moe_weights *w, void *workspace, size_t workspace_bytes, void *stream) {
    if (!dims_ok(w) || !workspace || !aligned(workspace, 256)) return (int)cudaErrorInvalidValue;
    const int n_tok = last_prefill(workspace, w);
    if (n_tok <= PF_MIN_TOK || ws_max_tok(workspace_bytes, w) < n_tok) return (int)cudaErrorInvalidValue;
    Workspace L(n_tok, w->n_embd, w->ff, w->n_experts, w->used);
    return pf_gemms(w, L, workspace, n_tok * w->used, S(stream));
}

int rvc_moe_forward(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype,
                    const float *bias, int bias_stride, int n_tok, float *out, int32_t *ids, float *wts,
                    void *workspace, size_t workspace_bytes, void *stream) {
    forget_prefill(workspace);  // a prefill call notes the workspace again once its GEMMs are enqueued
    if (!dims_ok(w) || !x_router || !x_expert || !out || n_tok <= 0 || !workspace || bias_stride < 0 ||
        !aligned(x_router, 16) || !aligned(x_expert, 16) || !aligned(workspace, 256) ||
        (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (ws_max_tok(workspace_bytes, w) < n_tok) return RVC_ERR_WORKSPACE;
    if (n_tok > PF_MIN_TOK)
        return run_prefill(w, x_router, x_expert, x_dtype, bias, bias_stride, n_tok, out, ids, wts, workspace,
                           workspace_bytes, S(stream));
    return run_decode(w, x_router, x_expert, x_dtype, bias, bias_stride, nullptr, nullptr, n_tok, out, ids, wts,
                      workspace, S(stream));
}

int rvc_workspace_reset(void *workspace, void *stream) {
    forget_prefill(workspace);
    if (!workspace) return (int)cudaErrorInvalidValue;
    return (int)cudaMemsetAsync(workspace, 0, 256, S(stream));
}

// ------------------------------------------------------------------ expert parallelism
size_t rvc_q8_record_bytes(int n_embd) { return n_embd > 0 && n_embd % QK == 0 ? (size_t)q8rec_bytes(n_embd / QK) : 0; }

size_t rvc_ep_row_bytes(int n_embd, int used) {
    return n_embd > 0 && n_embd % QK == 0 && used > 0 && used <= MAX_USED ? (size_t)ep_row_bytes(n_embd / QK, used) : 0;
}

int rvc_quant_q8_rows(const void *x, int x_dtype, int n_rows, int n_embd, void *records, void *stream) {
    if (!x || !records || n_rows < 0 || n_embd <= 0 || n_embd % QK || !aligned(x, 4) ||
        (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    if (n_rows == 0) return 0;
    const long long tasks = (long long)n_rows * (n_embd / QK);
    const int blocks = (int)std::min<long long>(16 * num_sms(), (tasks + 7) / 8);
    if (x_dtype == RVC_BF16)
        k_quant_rows<uint16_t><<<blocks, 256, 0, S(stream)>>>((const uint16_t *)x, n_embd, n_rows, (uint8_t *)records);
    else
        k_quant_rows<float><<<blocks, 256, 0, S(stream)>>>((const float *)x, n_embd, n_rows, (uint8_t *)records);
    return launched();
}

int rvc_ep_pack(const int32_t *ids, const float *wts, const void *records, int n_tok, int used, int n_embd,
                int n_local, int world, int32_t *counts, void *send, int32_t *owner_map, int *status, void *stream) {
    if (n_tok < 0 || used <= 0 || used > MAX_USED || n_embd <= 0 || n_embd % QK || n_local <= 0 || world <= 0 ||
        world > EP_MAX_RANKS || !counts || !status || (n_tok > 0 && (!ids || !wts || !records || !send || !owner_map)) ||
        (records && !aligned(records, 16)) || (send && !aligned(send, 16)))
        return (int)cudaErrorInvalidValue;
    cudaStream_t st = S(stream);
    cudaError_t e = cudaMemsetAsync(counts, 0, 2 * (size_t)world * sizeof(int32_t), st);  // counts, cursors
    if (e != cudaSuccess) return (int)e;
    if (n_tok == 0) return 0;
    k_ep_count<<<(n_tok + 255) / 256, 256, 0, st>>>(ids, n_tok, used, n_local, world, counts, status);
    int rc = launched();
    if (rc) return rc;
    k_ep_pack<<<(n_tok + 7) / 8, 256, 0, st>>>(ids, wts, (const uint8_t *)records, n_embd / QK, n_tok, used, n_local,
                                               world, counts, counts + world, (uint8_t *)send, owner_map);
    return launched();
}

size_t rvc_ep_workspace_bytes(int max_rows, int used, int n_embd, int ff, int n_experts) {
    if (max_rows <= 0 || used <= 0 || used > MAX_USED || n_embd <= 0 || n_embd % QK || ff <= 0 || ff % QK ||
        n_experts <= 0)
        return 0;
    return Workspace(ep_tokens(max_rows * used), n_embd, ff, n_experts, 8).total;
}

int rvc_ep_experts(const rvc_moe_weights *w, const void *rows, int n_rows, int used, float *partial, void *workspace,
                   size_t workspace_bytes, void *stream) {
    forget_prefill(workspace);
    if (!dims_ok(w) || n_rows < 0 || used <= 0 || used > MAX_USED || !workspace || !aligned(workspace, 256) ||
        (n_rows > 0 && (!rows || !partial || !aligned(rows, 16) || !aligned(partial, 16))))
        return (int)cudaErrorInvalidValue;
    int rc;
    if ((rc = pf_supported(w))) return rc;
    if (n_rows == 0) return 0;
    const int n_pairs = n_rows * used;
    Workspace L(ep_tokens(n_pairs), w->n_embd, w->ff, w->n_experts, 8);
    if (L.total > workspace_bytes) return RVC_ERR_WORKSPACE;
    cudaStream_t st = S(stream);
    const int nb = w->n_embd / QK;
    int32_t *slot_e = at<int32_t>(workspace, L.ids);
    float *slot_w = at<float>(workspace, L.wts);
    k_ep_meta<<<std::min(4 * num_sms(), (n_pairs + 255) / 256), 256, 0, st>>>((const uint8_t *)rows, nb, n_rows, used,
                                                                              slot_e, slot_w);
    if ((rc = launched()) || (rc = pf_plan(slot_e, n_pairs, w->n_experts, L, workspace, st, true))) return rc;
    const long long tasks = (long long)n_rows * nb;
    k_ep_scatter<<<(int)std::min<long long>(16 * num_sms(), (tasks + 7) / 8), 256, 0, st>>>(
        (const uint8_t *)rows, nb, n_rows, used, slot_e, at<int32_t>(workspace, L.pos_of), at<uint8_t>(workspace, L.xperm),
        at<float>(workspace, L.xd), (int)L.ppad);
    if ((rc = launched()) || (rc = pf_gemms(w, L, workspace, n_pairs, st))) return rc;
    k_pf_combine<<<n_rows, 256, 0, st>>>(at<float>(workspace, L.ybuf), at<int32_t>(workspace, L.pos_of), slot_e, slot_w,
                                         w->down_scale, used, w->n_embd, n_rows, partial, at<int>(workspace, L.status));
    return launched();
}

int rvc_ep_reduce(const float *back, const int32_t *owner_map, int n_tok, int world, int n_embd, float *out,
                  void *stream) {
    if (n_tok < 0 || world <= 0 || world > EP_MAX_RANKS || n_embd <= 0 || n_embd % 4 ||
        (n_tok > 0 && (!owner_map || !out || !aligned(out, 16))) || (back && !aligned(back, 16)))
        return (int)cudaErrorInvalidValue;
    if (n_tok == 0) return 0;
    k_ep_reduce<<<n_tok, 256, 0, S(stream)>>>(back, owner_map, world, n_embd, out);
    return launched();
}

int rvc_rms_norm(const float *x, float *out, const float *weight, int rows, int width, float eps, float post,
                 void *stream) {
    if (!x || !out || rows <= 0 || width <= 0 || !aligned(x, 4) || !aligned(out, 4) || (weight && !aligned(weight, 4)))
        return (int)cudaErrorInvalidValue;
    const bool vec = width % 4 == 0 && aligned(x, 16) && aligned(out, 16) && (!weight || aligned(weight, 16));
    const int grid = (rows + NORM_WARPS - 1) / NORM_WARPS;
    if (vec)
        k_rms_norm<true><<<grid, NORM_WARPS * 32, 0, S(stream)>>>(x, out, weight, rows, width, eps, post);
    else
        k_rms_norm<false><<<grid, NORM_WARPS * 32, 0, S(stream)>>>(x, out, weight, rows, width, eps, post);
    return launched();
}

// ------------------------------------------------------------------ shared dense MLP
namespace {
int q4_chains(bool gu, const void *w0, const void *w1, const float *x, float *y, int n_out, int k, int n_tok,
              cudaStream_t st) {
    int rc = gu ? set_smem_attr(k_q4_chains<true>, 31) : set_smem_attr(k_q4_chains<false>, 30);
    if (rc) return rc;
    const int rpc = gu ? DN_ROWS / 2 : DN_ROWS;
    const dim3 grid((unsigned)((n_out + rpc - 1) / rpc), (unsigned)((n_tok + DN_T - 1) / DN_T));
    const DenseArgs a{static_cast<const uint8_t *>(w0), static_cast<const uint8_t *>(w1), x, y, n_out, k, n_tok};
    if (gu)
        k_q4_chains<true><<<grid, DN_THREADS, DN_SMEM, st>>>(a);
    else
        k_q4_chains<false><<<grid, DN_THREADS, DN_SMEM, st>>>(a);
    return launched();
}
}  // namespace

int rvc_q4_mm(const void *w, const float *x, float *y, int n_out, int k, int n_in, void *stream) {
    if (!w || !x || !y || n_out <= 0 || k <= 0 || k % QK || n_in <= 0 || n_in > 65535 * DN_T || !aligned(w, 2) ||
        !aligned(x, 16) || !aligned(y, 4))
        return (int)cudaErrorInvalidValue;
    return q4_chains(false, w, nullptr, x, y, n_out, k, n_in, S(stream));
}

int rvc_geglu(const float *g, const float *u, float *out, int n, void *stream) {
    if (!g || !u || !out || n < 0) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    k_geglu<<<(n + 255) / 256, 256, 0, S(stream)>>>(g, u, out, n);
    return launched();
}

size_t rvc_shared_mlp_workspace_bytes(int max_tok, int n_embd, int ff) {
    if (max_tok <= 0 || n_embd <= 0 || ff <= 0) return 0;
    return align256((size_t)max_tok * n_embd * 4) + align256((size_t)max_tok * ff * 4);
}

int rvc_shared_mlp(const void *w_gate, const void *w_up, const void *w_down, const float *ffn_norm,
                   const float *post_norm, const float *x, float *out, int n_tok, int n_embd, int ff, float eps,
                   void *workspace, size_t workspace_bytes, void *stream) {
    if (!w_gate || !w_up || !w_down || !aligned(w_gate, 2) || !aligned(w_up, 2) || !aligned(w_down, 2) || !x ||
        !out || !workspace || !aligned(workspace, 256) || !aligned(out, 16) || n_tok <= 0 || n_embd <= 0 || ff <= 0 ||
        n_embd % QK || ff % QK || n_tok > 65535 * DN_T)
        return (int)cudaErrorInvalidValue;
    if (workspace_bytes < rvc_shared_mlp_workspace_bytes(n_tok, n_embd, ff)) return RVC_ERR_WORKSPACE;
    cudaStream_t st = S(stream);
    float *cur = static_cast<float *>(workspace);
    float *mlp = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + align256((size_t)n_tok * n_embd * 4));
    int rc = rvc_rms_norm(x, cur, ffn_norm, n_tok, n_embd, eps, 1.0f, stream);         // exec.rs:440-443
    if (!rc) rc = q4_chains(true, w_gate, w_up, cur, mlp, ff, n_embd, n_tok, st);      // :444-448
    if (!rc) rc = q4_chains(false, w_down, nullptr, mlp, out, n_embd, ff, n_tok, st);  // :450
    if (!rc) rc = rvc_rms_norm(out, out, post_norm, n_tok, n_embd, eps, 1.0f, stream);  // :451-453
    return rc;
}

int rvc_status(void *workspace, void *stream) {
    if (!workspace) return (int)cudaErrorInvalidValue;
    int rc = (int)cudaStreamSynchronize(S(stream));
    if (rc) return rc;
    int st = 0;
    rc = (int)cudaMemcpy(&st, workspace, sizeof(int), cudaMemcpyDeviceToHost);
    if (rc) return rc;
    if (st) {  // an aborted call can leave the grid barrier mid-way: clear the whole header
        rc = (int)cudaMemset(workspace, 0, 256);
        if (rc) return rc;
    }
    if (st & STATUS_TIMEOUT) return RVC_ERR_DEVICE_TIMEOUT;
    if (st & STATUS_BAD_INDEX) return RVC_ERR_DEVICE_INDEX;
    return 0;
}

int rvc_debug_gemm_block_dots(const rvc_moe_weights *w, int which, int expert, int row_tile, const void *records,
                              int n, int32_t *out, void *scratch, size_t scratch_bytes, void *stream) {
    if (!dims_ok(w) || (which != 0 && which != 1) || expert < 0 || expert >= w->n_experts || !records || n < 1 ||
        n > TC_N || !out || !scratch || !aligned(records, 16) || !aligned(scratch, 256))
        return (int)cudaErrorInvalidValue;
    int rc;
    if ((rc = pf_supported(w))) return rc;
    const int rows = which == 0 ? 2 * w->ff : w->n_embd, nblk = (which == 0 ? w->n_embd : w->ff) / QK;
    if (row_tile < 0 || row_tile >= rows / TC_M) return (int)cudaErrorInvalidValue;
    const int ppad = (n + 3) / 4 * 4;
    // scratch: the one-entry tile list and its count, then an (unused) scale plane
    if (scratch_bytes < 256 + (size_t)nblk * ppad * 4) return RVC_ERR_WORKSPACE;
    cudaStream_t st = S(stream);
    const int2 tile = make_int2(expert | (n << 8), 0);
    const int hdr[4] = {tile.x, tile.y, 1, 0};
    if ((rc = (int)cudaMemcpyAsync(scratch, hdr, sizeof hdr, cudaMemcpyHostToDevice, st))) return rc;
    if ((rc = (int)cudaMemsetAsync(static_cast<uint8_t *>(scratch) + 256, 0, (size_t)nblk * ppad * 4, st))) return rc;
    const PackedView pk = packed_view(w);
    TcMaps m;
    if ((rc = tc_maps(&m, (const uint8_t *)records, pf_rec_bytes(nblk), nblk, n,
                      reinterpret_cast<const float *>(static_cast<uint8_t *>(scratch) + 256), ppad,
                      which == 0 ? pk.gu_nib : pk.dn_nib, (uint64_t)w->n_experts * rows)))
        return rc;
    TcArgs g{};
    g.tiles = static_cast<const int2 *>(scratch), g.n_tiles = static_cast<const int *>(scratch) + 2, g.max_tiles = 1;
    g.n_experts = w->n_experts, g.ppos = n, g.ppad = ppad, g.n_embd = w->n_embd;
    g.status = static_cast<int *>(scratch) + 3;
    g.rows_per_expert = rows, g.row_tiles = 1, g.row_base = row_tile * TC_M, g.nblk = nblk;
    g.dwp = which == 0 ? pk.gu_dw : pk.dn_dw;
    g.y = reinterpret_cast<float *>(out);
    return launch_tc<PF_RAW>(m, g, 1, st);
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

// ------------------------------------------------------------------ GGUF weights (host only)
struct rvc_gguf {
    rvc::gguf::File f;
};

int rvc_gguf_parse(const void *buf, size_t len, rvc_gguf **out) {
    if (!out || (!buf && len)) return (int)cudaErrorInvalidValue;
    *out = nullptr;
    rvc_gguf *g = new (std::nothrow) rvc_gguf();
    if (!g) return (int)cudaErrorMemoryAllocation;
    const int r = rvc::gguf::parse(static_cast<const uint8_t *>(buf), len, &g->f);
    if (r) {
        delete g;
        return RVC_ERR_GGUF + r;
    }
    *out = g;
    return 0;
}

int rvc_gguf_open(const char *path, rvc_gguf **out) {
    if (!path || !out) return (int)cudaErrorInvalidValue;
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return RVC_ERR_GGUF + rvc::gguf::kIo;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        return RVC_ERR_GGUF + (st.st_size == 0 ? rvc::gguf::kTruncated : rvc::gguf::kIo);
    }
    const size_t len = (size_t)st.st_size;
    void *m = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return RVC_ERR_GGUF + rvc::gguf::kIo;
    rvc_gguf *g = nullptr;
    const int r = rvc_gguf_parse(m, len, &g);
    if (r) {
        munmap(m, len);
        return r;
    }
    g->f.map = m, g->f.map_len = len;
    *out = g;
    return 0;
}

void rvc_gguf_close(rvc_gguf *g) {
    if (!g) return;
    if (g->f.map) munmap(g->f.map, g->f.map_len);
    delete g;
}

int rvc_gguf_tensor(const rvc_gguf *g, const char *name, int *dtype, int *n_dims, uint64_t *shape, const void **data,
                    uint64_t *bytes) {
    if (!g || !name) return (int)cudaErrorInvalidValue;
    const rvc::gguf::Tensor *t = g->f.find(name);
    if (!t) return RVC_ERR_GGUF + rvc::gguf::kMissing;
    if (dtype) *dtype = t->dtype;
    if (n_dims) *n_dims = t->n_dims;
    if (shape)
        for (int d = 0; d < 4; ++d) shape[d] = t->shape[d];
    if (data) *data = t->data;
    if (bytes) *bytes = t->bytes;
    return 0;
}

int rvc_gguf_moe_layer(const rvc_gguf *g, int layer, int n_embd, int ff, int n_experts, rvc_gguf_moe *out) {
    using namespace rvc::gguf;
    if (!g || !out || layer < 0 || n_embd <= 0 || ff <= 0 || n_experts <= 0) return (int)cudaErrorInvalidValue;
    const uint64_t E = (uint64_t)n_embd, F = (uint64_t)ff, N = (uint64_t)n_experts;
    struct Want {
        const char *suffix;
        int dtype, n_dims;
        uint64_t s[3];
        const void **dst;
    };
    const void *gu, *dn, *router, *dscale, *giscale, *pre, *post;
    const Want want[] = {
        {"ffn_gate_up_exps.weight", kQ4_0, 3, {E, 2 * F, N}, &gu},  // contract.rs:69
        {"ffn_down_exps.weight", kQ4_0, 3, {F, E, N}, &dn},         // contract.rs:70
        {"ffn_gate_inp.weight", kF32, 2, {E, N, 0}, &router},       // contract.rs:66
        {"ffn_down_exps.scale", kF32, 1, {N, 0, 0}, &dscale},       // contract.rs:68
        {"ffn_gate_inp.scale", kF32, 1, {E, 0, 0}, &giscale},       // contract.rs:67
        {"pre_ffw_norm_2.weight", kF32, 1, {E, 0, 0}, &pre},        // contract.rs:42-51
        {"post_ffw_norm_2.weight", kF32, 1, {E, 0, 0}, &post},
    };
    for (const Want &w : want) {
        const std::string name = "blk." + std::to_string(layer) + "." + w.suffix;
        const Tensor *t = g->f.find(name.c_str());
        if (!t) return RVC_ERR_GGUF + kMissing;
        bool ok = t->dtype == w.dtype && t->n_dims == w.n_dims;
        for (int d = 0; ok && d < w.n_dims; ++d) ok = t->shape[d] == w.s[d];
        if (!ok) return RVC_ERR_GGUF + kContract;
        *w.dst = t->data;
    }
    out->gate_up = gu, out->down = dn;
    out->router = static_cast<const float *>(router);
    out->down_scale = static_cast<const float *>(dscale);
    out->gate_inp_scale = static_cast<const float *>(giscale);
    out->pre_norm = static_cast<const float *>(pre);
    out->post_norm = static_cast<const float *>(post);
    return 0;
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
    if (!dims_ok(w) || !x_router || !x_expert || !out || n_tok <= 0 || bias_stride < 0 || !aligned(x_router, 16) ||
        !aligned(x_expert, 16) || (x_dtype != RVC_F32 && x_dtype != RVC_BF16))
        return (int)cudaErrorInvalidValue;
    // the decode kernels, in their own workspace layout, for every call that fits the array
    if (n_tok > FD_MAX_TOK ||
        Workspace(n_tok, w->n_embd, w->ff, w->n_experts, w->used, FD_MAX_TOK).total > (size_t)RVC_NOALLOC_SCRATCH_BYTES)
        return RVC_ERR_WORKSPACE;
    void *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // The array keeps the previous call's contents; only the header (status word, grid
    // barrier) must start at zero.
    rc = (int)cudaMemsetAsync(scratch, 0, 256, S(stream));
    if (rc) return rc;
    return run_decode(w, x_router, x_expert, x_dtype, bias, bias_stride, nullptr, nullptr, n_tok, out, ids, wts,
                      scratch, S(stream), FD_MAX_TOK);
}

#ifdef RVC_PROFILE
// Profiling builds only: copy (and clear) the phase timestamps recorded by RVC_MARK.
extern "C" int rvc_profile_dump(void *host, size_t bytes, void *host_clk) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(host, rvc::g_prof, bytes);
    if (e == cudaSuccess && host_clk) e = cudaMemcpyFromSymbol(host_clk, rvc::g_prof_clk, bytes);
    static unsigned long long zero[8][1024][8];
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(rvc::g_prof, zero, sizeof zero);
    return (int)e;
}
#endif
