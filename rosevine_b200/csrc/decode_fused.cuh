// decode_fused.cuh - the decode MoE layer (n_tok <= 64) in three kernels (sm_100a).
//
// Replaces, for decode batches, the reference's MoE branch of HipSession::layer
// (runtime/src/hip_exec.rs:786-843: router GEMV, logits download, host select_experts and
// MoePlan, four uploads, per-expert q4_mm / geglu_split / q4_mm, moe_combine) and computes
// what the CPU-experts Q8_0 path computes (runtime/src/exec.rs:493-517, 541-557, 572-640).
//
// Three kernels, one CTA per SM each, 512 threads. Decode is a latency problem: every phase
// spreads its work over whole CTAs so that no single warp runs a long serial instruction
// stream, and the kernel boundaries replace grid-wide barriers where the next phase needs all of
// the previous one's results (an SM also starts a kernel with its first 64 KB of code at hand,
// so three compact kernels run faster than one long persistent one):
//
// k_fd_gate and k_fd_down are launched as programmatic dependents of the kernel before them: their
// CTAs start on SMs the previous kernel's CTAs leave and wait for its completion (griddep_wait)
// before reading what it wrote, which takes most of the launch gap out of each boundary.
//
//  k_fd_route (cooperative launch, so all CTAs are resident)
//   1. router: items of (expert, up to 4 tokens) spread over the CTAs; within an item warp g
//      takes the g-th 256 columns, forming f64 dots (exact products of bf16/f32 operands) and
//      the rigorous bound on the reference's sequential f32 chain (router_fast.cuh). Spare warps
//      write the Q8_0 records of x.                                   -- grid barrier --
//   2. selection: a group of 128 threads per token ranks the experts in two levels (within
//      each warp, then among the warps' candidates), certifies that the fast logits' order is
//      the reference's and forms the softmax / top-k / renormalised weights with the
//      reference's arithmetic on those logits rounded to f32; CTA t selects token t.
//  k_fd_gate
//   3. tokens that could not be certified get the exact sequential chains and an exact
//      selection (rare: a few percent of tokens); every CTA builds the stable (expert, pair)
//      plan of MoePlan::new in shared memory.
//   4. gate/up: the (expert, 32-column) units of all active experts are split over the CTAs
//      (evenly for one or two tokens, by cost for batches: fd_unit_range). Weight rows stream
//      through a ring of shared-memory slots filled by 1-D TMA bulk copies; token records sit
//      beside them; h = gelu(gate)*up is quantised to Q8_0 records. The CTAs also pull the down
//      tiles of the first FD_L2_EXPERTS active experts toward L2.
//  k_fd_down
//   5. down + combine: each CTA owns a range of output rows for every pair, computes
//      y = W_down[rows] . h for all pairs from tiles streamed through its ring and combines the
//      pairs of each token in slot order.
//
// Every expert dot product runs in the reference's scalar order (expert_kernel.rs:147-161):
// int32 block sums, acc = acc + sumi * (dw * dx) with each operation rounded separately.
#pragma once
#include "common.cuh"
#include "pack.cuh"
#include "router.cuh"
#include "router_fast.cuh"

namespace rvc {

constexpr int FD_THREADS = 512;
constexpr int FD_WARPS = FD_THREADS / 32;
constexpr int FD_MAX_TOK = 64;
constexpr int FD_MAX_PAIRS = 512;
constexpr int FD_MAX_SLOTS = 8;
constexpr int FD_MAX_EXPERTS = 128;  // one selection thread per expert in a 128-thread group
constexpr int FD_GROUPS = FD_THREADS / 128;
constexpr int FD_REDUNDANT_TOK = FD_GROUPS;  // up to this many tokens every CTA selects them all
constexpr int FD_ROWS = 32;                  // packed gate/up rows per ring slot
constexpr int FD_TB = 4;                     // tokens per router item
constexpr int FD_SCRATCH = 16384;            // ring bytes lent to phases 1-2 (scratch below)
// Active experts whose down tiles k_fd_gate pulls toward L2 for k_fd_down's first stages (about
// 18 MB at the target's shapes). Prefetching every active expert's tiles at larger batches (127 MB
// at 32 tokens) held up the gate kernel's first weight copies by ~20 us and did not stay in L2
// beside the gate/up stream; the down kernel's own ring covers the later stages.
constexpr int FD_L2_EXPERTS = 16;
constexpr int FD_HB = FD_MAX_SLOTS / 2;  // token chunks whose dots k_fd_gate<..., true> holds for one h phase

// Shared-memory plans of the three kernels, computed on the host (fd_layout), passed by value.
struct FdLayout {
    // k_fd_route
    uint32_t r_bytes;  // two router-item buffers
    // k_fd_gate
    int nslot, slot_bytes;  // gate/up weight ring (also lends space to the selection phase)
    int act_bytes, act_x;   // each of two x-record buffers, records it holds
    int chain_items;        // exact-chain items one CTA stages at once
    uint32_t off_act, off_gu, off_plan, bytes;
    // k_fd_down
    int d_nslot, d_slot_bytes;  // down weight ring
    int d_act_bytes, act_h;     // each of two h-record buffers, records it holds
    int rg;                     // down rows are assigned in groups of rg (bulk-copy alignment)
    int rpc_max;                // most down rows any CTA owns
    int y_in_smem;              // y of the down projection in shared memory (else ybuf)
    uint32_t d_off_act, d_off_y, d_off_plan, d_bytes;
};

struct FdArgs {
    const void *xr, *xe;  // router input, expert input [n_tok][n_embd]
    const void *wr;       // router weight [n_experts][n_embd]
    const float *bias;    // optional per-(token, expert) logit bias
    int bias_stride;
    PackedView pk;
    const float *down_scale;  // optional [n_experts]
    int n_tok, n_embd, ff, n_experts, used;
    const int32_t *ids_in;  // caller routing (experts-only mode), else NULL
    const float *wts_in;
    float *out;
    int32_t *ids_out;  // optional
    float *wts_out;    // optional
    float *lfast, *lbound, *lexact;  // [n_tok][n_experts]
    uint8_t *xrec, *hrec;            // Q8_0 records: [n_tok], [pairs] in plan order
    float *ybuf;                     // [pairs][n_embd] when y is not kept in shared memory
    int32_t *sel_ids, *sel_flag;     // published selection: [pairs], [n_tok]
    float *sel_wts;                  // [pairs]
    unsigned *bar_cnt, *bar_gen;     // grid barrier (count returns to 0 after every barrier)
    unsigned *fallback_cnt;          // running count of tokens routed through the exact chains
    int32_t *plan;  // published plan: [pairs] ids, wts, pos_of, order; [n_experts] counts, offsets,
                    // active; [1] n_active (k_fd_gate writes it, k_fd_down reads it)
    int *status;
    FdLayout L;
};

// Scratch of phases 1-2, in the first FD_SCRATCH bytes of the ring.
struct FdRouteScratch {
    double wsum[FD_WARPS][FD_TB];  // per column-group f64 sums
    float wa[FD_WARPS][FD_TB], wp[FD_WARPS][FD_TB];
};
struct FdSelGroup {
    unsigned long long ck[4 * MAX_USED];  // level-1 candidates (key, index)
    float cl[4 * MAX_USED], cb[4 * MAX_USED], cp[4 * MAX_USED];
    int top_e[MAX_USED];
    float top_l[MAX_USED], top_b[MAX_USED], top_p[MAX_USED];
    float redf[4];
    double redd[4];
    int ok;
};
struct FdScratch {
    FdRouteScratch r;
    FdSelGroup g[FD_GROUPS];
};
static_assert(sizeof(FdScratch) <= FD_SCRATCH, "phase scratch exceeds its share of the ring");

// ------------------------------------------------- programmatic dependent launch
// A kernel launched as a programmatic dependent (cudaLaunchAttributeProgrammaticStreamSerialization)
// may start before the kernel ahead of it in the stream has finished; griddep_wait blocks until
// that kernel has completed and its memory operations are visible. griddep_launch_dependents lets
// the next such kernel launch early (its CTAs still need free SM resources to start). Both are
// no-ops in a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_gpu(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_gpu(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's generic-proxy global writes before later async-proxy (TMA) reads of
// the same addresses by any thread that synchronises with it.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Sense-reversing barrier over all CTAs of the grid: thread 0 reads the generation, makes the
// CTA's writes visible (acq_rel fence, cumulative over the __syncthreads before it), arrives
// on the count, and either (last arrival) resets the count and publishes the next generation
// with a release store, or spins until the generation moves. The spin is bounded; on timeout it
// records STATUS_TIMEOUT and returns false (the caller leaves the kernel).
__device__ __noinline__ bool grid_sync(unsigned *cnt, unsigned *gen, int *status) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned g = ld_acquire_gpu(gen);
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        int ok = 1;
        if (atomicAdd(cnt, 1u) == gridDim.x - 1) {
            st_relaxed_gpu(cnt, 0u);
            st_release_gpu(gen, g + 1);
        } else {
            long long i = 0;
            while (ld_acquire_gpu(gen) == g)
                if (++i > kSpinLimit) {
                    set_status(status, STATUS_TIMEOUT);
                    ok = 0;
                    break;
                }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// named barrier of one 128-thread selection group
__device__ __forceinline__ void group_sync(int grp) { asm volatile("bar.sync %0, 128;" ::"r"(grp + 1) : "memory"); }

// ------------------------------------------------------------ phase 1: logits
// named barrier of the NB8 column-group warps of a router item
__device__ __forceinline__ void dot_sync(int nthreads) { asm volatile("bar.sync 5, %0;" ::"r"(nthreads) : "memory"); }

// Item (expert e, tokens t0 .. t0 + nt - 1) with its router row and x rows staged at `buf`
// ([router row][x row of each token], n_embd elements each). Called by warps 0..NB8-1 only:
// warp g takes columns [256 g, 256 g + 256), 8 per lane, and forms for each token the f64 sum
// of its products and the two terms of the chain's error bound: P = sum |p_i| and A = sum |S_i|
// over the chain's prefix sums S_i (in f32: their own error is far inside the bound's 2%
// margin). Thread 0 then adds the column groups and stores the logit (plus bias) rounded to
// f32 and its bound. Tokens one at a time in a rolled loop (small code).
template <typename XT, typename WT, int NB8>
__device__ __noinline__ void fd_route_item(const uint8_t *buf, int n_embd, int e, int t0, int nt, int ne,
                                           const float *bias, int bias_stride, float *lfast, float *lbound,
                                           FdRouteScratch &R) {
    const int tid = threadIdx.x, lane = tid & 31, g = tid >> 5;
    const WT *wrow = reinterpret_cast<const WT *>(buf);
    const XT *xrows = reinterpret_cast<const XT *>(buf + (size_t)n_embd * sizeof(WT));
    const int k0 = g * 256 + lane * 8;
    float wv[8];
    lds8<WT>(wrow + k0, wv);
#pragma unroll 1
    for (int tt = 0; tt < nt; ++tt) {
        float xv[8];
        lds8<XT>(xrows + (size_t)tt * n_embd + k0, xv);
        double own = 0.0;
        float p = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            own += (double)wv[j] * (double)xv[j];
            p += fabsf(wv[j] * xv[j]);
        }
        double incl = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) R.wsum[g][0] = incl;
        dot_sync(NB8 * 32);
        double woff = 0.0;
        for (int h = 0; h < g; ++h) woff += R.wsum[h][0];
        float r = (float)(woff + incl - own), A = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            r += wv[j] * xv[j];
            A += fabsf(r);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            A += __shfl_xor_sync(0xffffffffu, A, o);
            p += __shfl_xor_sync(0xffffffffu, p, o);
        }
        if (lane == 0) R.wa[g][0] = A, R.wp[g][0] = p;
        dot_sync(NB8 * 32);
        if (tid == 0) {
            const int t = t0 + tt;
            double S = 0.0;
            float As = 0.0f, Ps = 0.0f;
            for (int h = 0; h < NB8; ++h) S += R.wsum[h][0], As += R.wa[h][0], Ps += R.wp[h][0];
            const double b = bias ? (double)__ldg(bias + (size_t)t * bias_stride + e) : 0.0;
            const double bd = 1.02 * RF_U * ((double)As + (double)Ps) + 2.02 * RF_U * (fabs(S) + fabs(b)) + 1e-30;
            lfast[(size_t)t * ne + e] = (float)(S + b);
            lbound[(size_t)t * ne + e] = (float)(bd * 1.001);
        }
        dot_sync(NB8 * 32);  // the scratch is reused
    }
}

// --------------------------------------------------------- phase 2: selection
// A 128-thread group (group grp; thread gl owns expert gl) routes one token.
// Fast mode (lb != NULL): lf are the f32-rounded f64 logits, ranked by logit (ties to the
//   lower index); each pick must be separated from the next (the last from every expert left
//   out) by more than both bounds plus a margin for the softmax's roundings, so that the
//   reference's probabilities have the same strict order. Returns false otherwise.
// Exact mode (lb == NULL): lf are the reference's own logits; ranked by probability, ties to
//   the lower index, exactly as ops.rs:182-187.
// Both: softmax with max subtraction, f32 exp, f64 sum, multiply by (1/sum) rounded to f32;
// weights p_j / max(sum of the picks' p in pick order, 2^-14) (ops.rs:170-179, exec.rs:507-517).
// Lanes j < used of the group's first warp write ids[j] and wts[j].
__device__ __noinline__ bool xselect(const float *lf, const float *lb, int ne, int used, int32_t *ids,
                                            float *wts, FdSelGroup &S, int grp) {
    const int gl = threadIdx.x & 127, q = gl >> 5, lane = threadIdx.x & 31;
    const bool in = gl < ne;
    const float l = in ? __ldcg(lf + gl) : -INFINITY;
    const float b = (in && lb) ? __ldcg(lb + gl) : 0.0f;
    float m = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) S.redf[q] = m;
    group_sync(grp);
    m = fmaxf(fmaxf(S.redf[0], S.redf[1]), fmaxf(S.redf[2], S.redf[3]));
    const float ex = in ? fd_exp_f32(__fsub_rn(l, m)) : 0.0f;
    double sm = (double)ex;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    if (lane == 0) S.redd[q] = sm;
    group_sync(grp);
    const float inv = __double2float_rn(1.0 / (((S.redd[0] + S.redd[1]) + S.redd[2]) + S.redd[3]));
    const float p = __fmul_rn(ex, inv);
    const uint32_t kk = in ? ((uint32_t)total_key(lb ? l : p) ^ 0x80000000u) : 0u;
    const unsigned long long K = ((unsigned long long)kk << 32) | (unsigned)(0xFFFF - gl);
    // level 1: rank within the warp; the warp's top `used` become candidates
    int r = 0;
#pragma unroll 8
    for (int s = 0; s < 32; ++s) r += __shfl_sync(0xffffffffu, K, s) > K;
    if (r < used) {
        const int ci = q * used + r;
        S.ck[ci] = K, S.cl[ci] = l, S.cb[ci] = b, S.cp[ci] = p;
    }
    group_sync(grp);
    // level 2: the first warp ranks the 4 * used candidates
    const int nc = 4 * used;
    if (q == 0) {
        if (nc <= 32) {  // one candidate per lane, ranked by shuffles
            const unsigned long long Kc = lane < nc ? S.ck[lane] : 0ull;
            int rank = 0;
#pragma unroll 8
            for (int cj = 0; cj < 32; ++cj) rank += __shfl_sync(0xffffffffu, Kc, cj) > Kc;
            if (lane < nc && rank < used) {
                S.top_e[rank] = 0xFFFF - (int)(Kc & 0xFFFFu);
                S.top_l[rank] = S.cl[lane], S.top_b[rank] = S.cb[lane], S.top_p[rank] = S.cp[lane];
            }
        } else {
            for (int ci = lane; ci < nc; ci += 32) {
                const unsigned long long Kc = S.ck[ci];
                int rank = 0;
                for (int cj = 0; cj < nc; ++cj) rank += S.ck[cj] > Kc;
                if (rank < used) {
                    S.top_e[rank] = 0xFFFF - (int)(Kc & 0xFFFFu);
                    S.top_l[rank] = S.cl[ci], S.top_b[rank] = S.cb[ci], S.top_p[rank] = S.cp[ci];
                }
            }
        }
    }
    group_sync(grp);
    float mo = -INFINITY;  // every expert left out, with its bound (fast mode)
    if (lb) {
        bool top = false;
        for (int j = 0; j < used; ++j) top |= S.top_e[j] == gl;
        mo = (in && !top) ? l + b : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mo = fmaxf(mo, __shfl_xor_sync(0xffffffffu, mo, o));
        group_sync(grp);  // redf is reused
        if (lane == 0) S.redf[q] = mo;
        group_sync(grp);
        mo = fmaxf(fmaxf(S.redf[0], S.redf[1]), fmaxf(S.redf[2], S.redf[3]));
    }
    if (q == 0) {
        const int j = lane;
        const float pj = j < used ? S.top_p[j] : 0.0f;
        float psum = -0.0f;  // f32 sum in pick order
        for (int jj = 0; jj < used; ++jj) psum = __fadd_rn(psum, __shfl_sync(0xffffffffu, pj, jj));
        psum = fmaxf(psum, ROUTER_SUM_MIN);
        bool bad = false;
        if (lb && j < used) {
            const float l0 = S.top_l[0], lj = S.top_l[j];
            const bool last = j + 1 == used;
            const float hi = last ? mo : S.top_l[j + 1] + S.top_b[j + 1];
            const float nxt = last ? mo : S.top_l[j + 1];
            bad = !(lj - S.top_b[j] > hi + 1e-6f * (1.0f + fabsf(nxt - l0))) || !(lj - l0 > -80.0f);
        }
        const bool ok = __ballot_sync(0xffffffffu, bad) == 0;
        if (ok && j < used) {
            ids[j] = S.top_e[j];
            wts[j] = __fdiv_rn(pj, psum);
        }
        if (lane == 0) S.ok = ok;
    }
    group_sync(grp);
    return S.ok != 0;
}

// Exact logits (the reference's sequential f32 chains, ops.rs:321-326) of the flagged tokens:
// item i = (f-th flagged token, expert e) for i = f * ne + e; this CTA takes items c, c + G, ...
// in rounds of up to `per` items: the router row and the x row of each item are staged into
// shared memory by bulk copies (rows padded by 16 B so that threads reading the same column of
// consecutive rows hit distinct banks), then thread k runs item k's chain.
template <typename XT, typename WT>
__device__ __noinline__ bool xchains(const XT *x, const WT *w, const float *bias, int bias_stride, int n,
                                             int ne, float *lexact, int *status, const int *flag_tok, int nflag,
                                             uint8_t *buf, int per, uint64_t *bar) {
    const int tid = threadIdx.x, G = gridDim.x, c = blockIdx.x;
    uint32_t phase = 0;
    const int wrow = n * (int)sizeof(WT) + 16, xrow = n * (int)sizeof(XT) + 16, irow = wrow + xrow;
    const int items = nflag * ne;
    const int mine = items > c ? (items - c + G - 1) / G : 0;  // items of this CTA
#pragma unroll 1
    for (int k0 = 0; k0 < mine; k0 += per) {
        const int cnt = min(per, mine - k0);
        if (tid == 0) {
            mbar_arrive_expect_tx(bar, (uint32_t)cnt * (uint32_t)(n * (sizeof(WT) + sizeof(XT))));
#pragma unroll 1
            for (int k = 0; k < cnt; ++k) {
                const int i = c + (k0 + k) * G, t = flag_tok[i / ne], e = i % ne;
                bulk_g2s(buf + (size_t)k * irow, w + (size_t)e * n, n * sizeof(WT), bar);
                bulk_g2s(buf + (size_t)k * irow + wrow, x + (size_t)t * n, n * sizeof(XT), bar);
            }
        }
        const bool ok = fd_mbar_wait(bar, phase & 1u, status);
        ++phase;
        if (__syncthreads_or(!ok)) return false;
        if (tid < cnt) {
            const int i = c + (k0 + tid) * G, t = flag_tok[i / ne], e = i % ne;
            const WT *wr = reinterpret_cast<const WT *>(buf + (size_t)tid * irow);
            const XT *xr = reinterpret_cast<const XT *>(buf + (size_t)tid * irow + wrow);
            float s = -0.0f;
#pragma unroll 1
            for (int k = 0; k < n; k += 8) {
                float wv[8], xv[8];
                lds8<WT>(wr + k, wv);
                lds8<XT>(xr + k, xv);
#pragma unroll
                for (int j = 0; j < 8; ++j) s = chain_step<XT, WT>(s, wv[j], xv[j]);
            }
            if (bias) s = __fadd_rn(s, __ldg(bias + (size_t)t * bias_stride + e));
            lexact[(size_t)t * ne + e] = s;
        }
        __syncthreads();  // the buffer is refilled next round
    }
    return true;
}

// --------------------------------------------------------------- gate / up rows
// The 32 packed rows of one ring slot (lane L: row L) against up to two tokens' x records, for
// small batches (k_fd_gate<..., false>). The packed nibble plane stores block b of row R at
// position b ^ (R & 7) (pack.cuh), so the 32 lanes' 16-byte reads of one block index fall in
// distinct bank groups. A task's nb blocks are split into FD_SEG contiguous ranges, one warp
// each (warp w: range w % FD_SEG of task w / FD_SEG), so that a CTA runs 16 warps where one
// warp per task would run a long serial chain. Each warp forms its range's products
// sumi * (dw * dx) in registers; then, in FD_SEG rounds separated by CTA barriers, the warp of
// range r adds its products in block order onto the running sums the warp of range r - 1 left in
// `hand`, so every row's sum is the reference's (expert_kernel.rs:147-161). Every thread of the
// CTA calls it (the barriers); `active` is false for warps without a task.
constexpr int FD_SEG = 4;
template <int NB8>
__device__ __noinline__ void fd_gu_split(const uint8_t *slot, const uint8_t *rec0, const uint8_t *rec1, bool two,
                                         bool active, float *hand, float *dst) {
    constexpr int nb = NB8 * 8, SL = nb / FD_SEG;
    static_assert(nb % FD_SEG == 0, "block ranges must split evenly");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, seg = warp % FD_SEG, sw = lane & 7;
    const uint8_t *nrow = slot + (size_t)lane * nb * 16;
    const uint16_t *srow = reinterpret_cast<const uint16_t *>(slot + FD_ROWS * nb * 16) + lane * nb;
    const Q8Rec xa{rec0, nb}, xb{rec1, nb};
    float p0[SL], p1[SL];
    if (active && two) {
#pragma unroll
        for (int k = 0; k < SL; ++k) {
            const int b = seg * SL + k;
            const uint4 nib = *reinterpret_cast<const uint4 *>(nrow + (b ^ sw) * 16);
            const float dw = f16_bits_to_f32(srow[b]);
            p0[k] = __fmul_rn((float)q4q8_sumi(nib, xa.qa(b), xa.qb(b), xa.s(b)), __fmul_rn(dw, xa.d(b)));
            p1[k] = __fmul_rn((float)q4q8_sumi(nib, xb.qa(b), xb.qb(b), xb.s(b)), __fmul_rn(dw, xb.d(b)));
        }
    } else if (active) {
#pragma unroll
        for (int k = 0; k < SL; ++k) {
            const int b = seg * SL + k;
            const uint4 nib = *reinterpret_cast<const uint4 *>(nrow + (b ^ sw) * 16);
            const float dw = f16_bits_to_f32(srow[b]);
            p0[k] = __fmul_rn((float)q4q8_sumi(nib, xa.qa(b), xa.qb(b), xa.s(b)), __fmul_rn(dw, xa.d(b)));
            p1[k] = 0.0f;
        }
    }
    float *h = hand + (warp / FD_SEG) * 64;
#pragma unroll 1
    for (int r = 0; r < FD_SEG; ++r) {
        if (active && seg == r) {
            float a0 = r ? h[lane] : 0.0f, a1 = r ? h[32 + lane] : 0.0f;
#pragma unroll
            for (int k = 0; k < SL; ++k) a0 = __fadd_rn(a0, p0[k]);
            if (two) {
#pragma unroll
                for (int k = 0; k < SL; ++k) a1 = __fadd_rn(a1, p1[k]);
            }
            if (r + 1 < FD_SEG) {
                h[lane] = a0, h[32 + lane] = a1;
            } else {
                dst[lane] = a0;
                if (two) dst[64 + lane] = a1;
            }
        }
        __syncthreads();
    }
}

// The same rows for batches (k_fd_gate<..., true>): warp w computes row (w & 7) * 4 + lane / 8
// of the slot, the 8 lanes of a row owning contiguous ranges of NB8 blocks, so a whole CTA
// works on one unit whatever the number of tokens. The ordered sum visits the lanes in order
// (one shuffle per lane), so every row's sum still follows the block order. Unrolled: in a
// batch this code runs for every unit and token pair.
template <int NB8>
__device__ __noinline__ float2 fd_gu_wide(const uint8_t *slot, const uint8_t *rec0, const uint8_t *rec1, bool two) {
    constexpr int nb = NB8 * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = (warp & 7) * 4 + (lane >> 3), l8 = lane & 7, b0 = l8 * NB8, sw = r & 7;
    const uint8_t *nrow = slot + (size_t)r * nb * 16;
    const uint16_t *srow = reinterpret_cast<const uint16_t *>(slot + FD_ROWS * nb * 16) + r * nb;
    const Q8Rec xa{rec0, nb}, xb{rec1, nb};
    float t0[NB8], t1[NB8];
#pragma unroll
    for (int k = 0; k < NB8; ++k) {
        const int b = b0 + k;
        const uint4 nib = *reinterpret_cast<const uint4 *>(nrow + (b ^ sw) * 16);
        const float dw = f16_bits_to_f32(srow[b]);
        t0[k] = __fmul_rn((float)q4q8_sumi(nib, xa.qa(b), xa.qb(b), xa.s(b)), __fmul_rn(dw, xa.d(b)));
        t1[k] = 0.0f;
        if (two) t1[k] = __fmul_rn((float)q4q8_sumi(nib, xb.qa(b), xb.qb(b), xb.s(b)), __fmul_rn(dw, xb.d(b)));
    }
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) {
        if (l8 == l) {
#pragma unroll
            for (int k = 0; k < NB8; ++k) a0 = __fadd_rn(a0, t0[k]);
            if (two) {
#pragma unroll
                for (int k = 0; k < NB8; ++k) a1 = __fadd_rn(a1, t1[k]);
            }
        }
        a0 = __shfl_sync(0xffffffffu, a0, (lane & ~7) | l);
        if (two) a1 = __shfl_sync(0xffffffffu, a1, (lane & ~7) | l);
    }
    return make_float2(a0, a1);
}

// One down-projection dot: row `nrow`/`srow` of a staged tile against the h record `hrec`,
// nbh blocks in block order (expert_kernel.rs:147-161); `key` is the low 3 bits of the row's
// index, by which its complete 8-block groups are swizzled in the packed plane (nib_pos).
__device__ __noinline__ float fd_dn_row(const uint8_t *nrow, const uint16_t *srow, const uint8_t *hrec, int nbh,
                                       int key) {
    const Q8Rec hr{hrec, nbh};
    float acc = 0.0f;
#pragma unroll 4
    for (int b = 0; b < nbh; ++b) {
        const uint4 nib = *reinterpret_cast<const uint4 *>(nrow + nib_pos(b, nbh, key) * 16);
        const int sumi = q4q8_sumi(nib, hr.qa(b), hr.qb(b), hr.s(b));
        acc = __fadd_rn(acc, __fmul_rn((float)sumi, __fmul_rn(f16_bits_to_f32(srow[b]), hr.d(b))));
    }
    return acc;
}

// The warp-0 part of the stable plan (MoePlan::new, exec.rs:541-557): rank of each pair among
// the earlier pairs of its expert, counts, offsets (exclusive scan) and the ascending active
// experts; returns their number.
__device__ __noinline__ int fd_plan_warp(const int32_t *p_ids, int pairs, int ne, int32_t *p_cnt, int32_t *p_rank,
                                         int32_t *p_off, int32_t *p_act) {
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int e = lane; e < ne; e += 32) p_cnt[e] = 0;
    __syncwarp();
#pragma unroll 1
    for (int q0 = 0; q0 < pairs; q0 += 32) {
        const int q = q0 + lane;
        const int e = q < pairs ? p_ids[q] : -1 - lane;
        const unsigned m = __match_any_sync(0xffffffffu, e);
        const int before = __popc(m & ((1u << lane) - 1u));
        const int r = q < pairs ? p_cnt[e] + before : 0;
        __syncwarp();
        if (q < pairs && before == 0) p_cnt[e] += __popc(m);
        __syncwarp();
        if (q < pairs) p_rank[q] = r;
    }
    __syncwarp();
    constexpr int PL = FD_MAX_EXPERTS / 32;
    int run = 0, flags = 0;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        const int e = lane * PL + i;
        run += e < ne ? p_cnt[e] : 0;
        flags += (e < ne && p_cnt[e] > 0);
    }
    int incl = run, fin = flags;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o), z = __shfl_up_sync(0xffffffffu, fin, o);
        if (lane >= o) incl += y, fin += z;
    }
    int base = incl - run, slot = fin - flags;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        const int e = lane * PL + i;
        if (e < ne) {
            p_off[e] = base;
            if (p_cnt[e] > 0) p_act[slot++] = e;
            base += p_cnt[e];
        }
    }
    if (lane == 31) p_off[ne] = incl;
    return __shfl_sync(0xffffffffu, fin, 31);
}

// ---------------------------------------------------------------- plan hand-off
// The dispatch plan k_fd_gate publishes for k_fd_down, in the workspace (int32 words).
struct FdPlan {
    int32_t *ids;
    float *wts;
    int32_t *pos, *order, *cnt, *off, *act, *n_act;
};
__host__ __device__ inline FdPlan fd_plan_at(int32_t *base, int pairs, int ne) {
    FdPlan p;
    p.ids = base;
    p.wts = reinterpret_cast<float *>(base + pairs);
    p.pos = base + 2 * pairs;
    p.order = base + 3 * pairs;
    p.cnt = base + 4 * pairs;
    p.off = p.cnt + ne;
    p.act = p.off + ne + 1;
    p.n_act = p.act + ne;
    return p;
}
__host__ __device__ inline size_t fd_plan_words(int pairs, int ne) { return (size_t)4 * pairs + 3 * ne + 2; }

// Per-CTA plan of the gate/up or down stages (shared memory, written by thread 0).
struct FdCtx {
    int n_act, g0, n_units, rows, r0, eps, NS;
    uint32_t dn_nib, tile;
};

// Down rows [r0, r0 + rows) of CTA c (groups of rg rows, so every bulk copy stays aligned).
__device__ __forceinline__ void fd_rows_of(int c, int G, int n_embd, int rg, int &r0, int &rows) {
    const int nq = n_embd / rg;
    r0 = rg * (c * nq / G);  // (all products here stay far below 2^31)
    rows = rg * ((c + 1) * nq / G) - r0;
}

// Bulk copies are issued by several threads at once, one copy each: issuing one takes a
// thread a good fraction of a microsecond, so a single thread issuing a stage's copies in turn
// would put that on the critical path. (An mbarrier's transaction count may run below zero
// until the arrive with its expected bytes, so copies can complete before that arrive.)

// Part `part` (0: nibbles, with the arrive; 1: scales) of gate/up stage j into its ring slot:
// half j & 1 (gate rows, up rows) of unit j / 2 (expert slot g / nbh, 32-column block g % nbh,
// g = g0 + j / 2).
template <int NB8>
__device__ __noinline__ void fd_issue_gate(const FdCtx &C, int j, int part, uint8_t *ring, int slot_bytes, int nslot,
                                           uint64_t *full, const int32_t *p_act, const uint8_t *gu_nib,
                                           const uint16_t *gu_scl, int ff) {
    constexpr int nb = NB8 * 8;
    constexpr uint32_t nbytes = FD_ROWS * nb * 16, sbytes = FD_ROWS * nb * 2;
    const int nbh = ff / QK;
    const int slot = j % nslot, g = C.g0 + (j >> 1);
    uint8_t *dst = ring + (size_t)slot * slot_bytes;
    uint64_t *bar = &full[slot];
    const size_t row0 = (size_t)p_act[g / nbh] * 2 * ff + (size_t)(g % nbh) * 64 + (j & 1) * FD_ROWS;
    if (part == 0) {
        mbar_arrive_expect_tx(bar, nbytes + sbytes);
        bulk_g2s(dst, gu_nib + row0 * nb * 16, nbytes, bar);
    } else {
        bulk_g2s(dst + nbytes, gu_scl + row0 * nb, sbytes, bar);
    }
}

// Expert i of down stage k into its ring slot (a stage: the CTA's output rows of up to eps
// consecutive active experts); the caller with i == 0 also arrives with the stage's bytes.
__device__ __noinline__ void fd_issue_down(const FdCtx &C, int k, int i, uint8_t *ring, int slot_bytes, int nslot,
                                           uint64_t *full, const int32_t *p_act, const uint8_t *dn_nib,
                                           const uint16_t *dn_scl, int n_embd, int nbh) {
    const int slot = k % nslot;
    uint64_t *bar = &full[slot];
    const int alo = k * C.eps, ahi = min(C.n_act, alo + C.eps);
    if (i == 0) mbar_arrive_expect_tx(bar, (uint32_t)(ahi - alo) * C.tile);
    if (alo + i < ahi) {
        const size_t row0 = (size_t)p_act[alo + i] * n_embd + C.r0;
        uint8_t *d = ring + (size_t)slot * slot_bytes + (size_t)i * C.tile;
        bulk_g2s(d, dn_nib + row0 * nbh * 16, C.dn_nib, bar);
        bulk_g2s(d + C.dn_nib, dn_scl + row0 * nbh, C.tile - C.dn_nib, bar);
    }
}

// Pair range [q0, q1) in plan order of down stage k (its experts are consecutive active slots).
__device__ __forceinline__ int2 fd_dn_pairs(const FdCtx &C, int k, const int32_t *p_act, const int32_t *p_off,
                                            const int32_t *p_cnt) {
    const int alo = k * C.eps, ahi = min(C.n_act, alo + C.eps);
    return make_int2(p_off[p_act[alo]], p_off[p_act[ahi - 1]] + p_cnt[p_act[ahi - 1]]);
}

// Activation records into buffer `dst` on `bar`, by the calling threads numbered i = 0, 1, ...
// (others pass i < 0 or beyond n): with h, thread 0 copies n consecutive h records from plan
// position p0; otherwise thread i < n copies the x record of plan position p0 + i (token
// order[p0 + i] / used), thread 0 arriving with all n records' bytes.
__device__ __noinline__ void fd_issue_records(int i, uint8_t *dst, uint64_t *bar, bool h, int p0, int n,
                                              const int32_t *p_order, int used, const uint8_t *xrec, int xrb,
                                              const uint8_t *hrec, int hrb) {
    if (i < 0) return;
    if (h) {
        if (i == 0) {
            mbar_arrive_expect_tx(bar, (uint32_t)n * hrb);
            bulk_g2s(dst, hrec + (size_t)p0 * hrb, (uint32_t)n * hrb, bar);
        }
    } else if (i < n) {
        if (i == 0) mbar_arrive_expect_tx(bar, (uint32_t)n * xrb);
        bulk_g2s(dst + (size_t)i * xrb, xrec + (size_t)(p_order[p0 + i] / used) * xrb, xrb, bar);
    }
}

// Leave after an error: wait (bounded) for the copies this CTA still has in flight.
__device__ __noinline__ void xdrain(uint64_t *full, int nslot, int j_done, int j_issued, uint64_t *actb,
                                      unsigned act_pend, unsigned act_use) {
    if (threadIdx.x != 0) return;
#pragma unroll 1
    for (int j = j_done; j < j_issued; ++j)
        for (int i = 0; i < (1 << 20) && !mbar_try_wait(&full[j % nslot], (uint32_t)(j / nslot) & 1u); ++i) {
        }
#pragma unroll 1
    for (int b = 0; b < 2; ++b)
        if ((act_pend >> b) & 1u)
            for (int i = 0; i < (1 << 20) && !mbar_try_wait(&actb[b], (act_use >> b) & 1u); ++i) {
            }
}

// The exact fallback (rare): the reference's sequential chains for the flagged tokens, spread
// over every CTA (xchains), a grid barrier, the exact selection of flagged token t by
// warps 0-3 of CTA t, another barrier, and every CTA takes the flagged tokens' new ids/weights.
// Returns false if a barrier or a copy timed out (every CTA leaves then).
template <typename XT, typename WT>
__device__ __noinline__ bool xfallbk(const XT *x, const WT *w, const float *bias, int bias_stride, int n_embd,
                                         int ne, int used, float *lexact, int32_t *sel_ids, float *sel_wts,
                                         unsigned *bar_cnt, unsigned *bar_gen, unsigned *fallback_cnt, int *status,
                                         const int *ftok, int nflag, uint8_t *ring, int chain_items, uint64_t *chb,
                                         int32_t *p_ids, float *p_wts, FdSelGroup &S) {
    const int tid = threadIdx.x, warp = tid >> 5, c = blockIdx.x;
    if (!xchains<XT, WT>(x, w, bias, bias_stride, n_embd, ne, lexact, status, ftok, nflag, ring + FD_SCRATCH,
                                 chain_items, chb))
        return false;
    if (!grid_sync(bar_cnt, bar_gen, status)) return false;
    if (c < nflag && warp < 4) {
        const int t = ftok[c];
        xselect(lexact + (size_t)t * ne, nullptr, ne, used, sel_ids + (size_t)t * used,
                       sel_wts + (size_t)t * used, S, 0);
    }
    if (!grid_sync(bar_cnt, bar_gen, status)) return false;
#pragma unroll 1
    for (int f = 0; f < nflag; ++f)
        if (tid < used) {
            const int i = ftok[f] * used + tid;
            p_ids[i] = __ldcg(sel_ids + i), p_wts[i] = __ldcg(sel_wts + i);
        }
    if (c == 0 && tid == 0 && fallback_cnt) atomicAdd(fallback_cnt, (unsigned)nflag);
    __syncthreads();
    return true;
}

// ------------------------------------------------------------- k_fd_route (1 of 3)
// Router logits and bounds, Q8_0 records of x, and the verified selection (cooperative launch:
// every CTA resident, for the grid barrier between the logits and the selection). Router items
// (expert, up to FD_TB tokens) go to CTAs round robin; thread 0 stages each item's router row
// and x rows into one of two buffers by bulk copies; warps 0..NB8-1 form the dots while the
// spare warps write the records (with no spare warp, or no routing to do, every warp writes
// records). After the barrier, warps 0-3 of CTA t select token t and publish its ids, weights
// and whether its order could be certified (k_fd_gate runs the exact fallback for the others).
template <typename XT, typename WT, int NB8>
__global__ void __launch_bounds__(FD_THREADS, 1) k_fd_route(FdArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t rb[2];
    __shared__ FdRouteScratch R;
    __shared__ FdSelGroup SG;
    RVC_MARK(4, 0);
    constexpr int nb = NB8 * 8;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x, T = a.n_tok, ne = a.n_experts;
    const int xrb = q8rec_bytes(nb);
    const bool route = a.ids_in == nullptr;
    const XT *xr = static_cast<const XT *>(a.xr);
    const WT *wr = static_cast<const WT *>(a.wr);
    const int ngrp = (T + FD_TB - 1) / FD_TB;
    const int n_items = route ? ne * ngrp : 0;
    const uint32_t wbytes = a.n_embd * sizeof(WT), xbytes = a.n_embd * sizeof(XT);
    const uint32_t rbytes = wbytes + FD_TB * xbytes;
    if (tid == 0) {
        mbar_init(&rb[0], 1);
        mbar_init(&rb[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    griddep_launch_dependents();  // k_fd_gate may take SMs as this kernel's CTAs leave
    // this CTA's k-th router item into buffer k & 1: part 0 the router row (and the arrive),
    // part 1 + tt the x row of token tt
    auto issue_item = [&](int k, int part) {
        const int it = c + k * G;
        if (it >= n_items) return;
        const int e = it / ngrp, t0 = (it - e * ngrp) * FD_TB, nt = min(FD_TB, T - t0);
        uint8_t *dst = smem + (size_t)(k & 1) * rbytes;
        if (part == 0) {
            mbar_arrive_expect_tx(&rb[k & 1], wbytes + (uint32_t)nt * xbytes);
            bulk_g2s(dst, wr + (size_t)e * a.n_embd, wbytes, &rb[k & 1]);
        } else if (part <= nt) {
            bulk_g2s(dst + wbytes + (part - 1) * xbytes, xr + (size_t)(t0 + part - 1) * a.n_embd, xbytes, &rb[k & 1]);
        }
    };
    if (tid < 2 * 32 && (tid & 31) <= FD_TB) issue_item(tid >> 5, tid & 31);
    if (route && warp < NB8) {
#pragma unroll 1
        for (int k = 0; c + k * G < n_items; ++k) {
            const int it = c + k * G;
            const int e = it / ngrp, t0 = (it - e * ngrp) * FD_TB;
            fd_mbar_wait(&rb[k & 1], (uint32_t)(k >> 1) & 1u, a.status);  // a timeout is in the status word
            fd_route_item<XT, WT, NB8>(smem + (size_t)(k & 1) * rbytes, a.n_embd, e, t0, min(FD_TB, T - t0), ne,
                                       a.bias, a.bias_stride, a.lfast, a.lbound, R);
            if (tid <= FD_TB) issue_item(k + 2, tid);
        }
    }
    const bool spare = route && NB8 < FD_WARPS;
    if (!spare || warp >= NB8) {
        const XT *xe = static_cast<const XT *>(a.xe);
        const int qw0 = spare ? NB8 : 0, nqw = FD_WARPS - qw0, n_q = T * nb;
#pragma unroll 1
        for (int i = c + G * (warp - qw0); i < n_q; i += G * nqw) {
            const int t = i / nb, b = i - t * nb;
            const float v = ld_val<XT>(xe, (size_t)t * a.n_embd + (size_t)b * QK + lane);
            uint16_t dbits;
            int qsum;
            const int8_t q = quant_q8_lane(v, &dbits, &qsum);
            q8rec_store(a.xrec + (size_t)t * xrb, nb, b, lane, q, dbits, qsum);
        }
    }
    if (!route) return;
    if (!grid_sync(a.bar_cnt, a.bar_gen, a.status)) return;
    RVC_MARK(4, 1);
    if (c < T && warp < 4) {
        const bool ok = xselect(a.lfast + (size_t)c * ne, a.lbound + (size_t)c * ne, ne, a.used,
                                       a.sel_ids + (size_t)c * a.used, a.sel_wts + (size_t)c * a.used, SG, 0);
        if (tid == 0) a.sel_flag[c] = !ok;
    }
}

// -------------------------------------------------------------- k_fd_gate (2 of 3)
// Plan and gate/up (cooperative launch: every CTA resident, for the grid barriers of the rare
// exact fallback). Publishes the plan and leaves h records for k_fd_down, whose weight tiles
// it prefetches into L2. WIDE (batches whose x records do not all fit one buffer): each unit
// is computed by the whole CTA (fd_gu_wide) instead of a warp per half and token pair.
// The gate/up units [g0, g1) of CTA c for batches (k_fd_gate<..., true>), called by one whole warp.
// A unit's time grows with its expert's tokens: each chunk of ax tokens costs a pass over the
// unit's rows and an h phase, on top of the unit's fixed cost (its stage waits and hand-back),
// measured at about 3 to 1. Unit weight 1 + 3 * chunks, and CTA c takes the units whose
// cumulative start weight lies in [c W / G, (c + 1) W / G): every CTA computes the same ranges,
// which tile [0, n_act * nbh) exactly.
__device__ __noinline__ int2 fd_unit_range(int c, int G, int n_act, int nbh, int ax, const int32_t *p_cnt,
                                           const int32_t *p_act) {
    const int lane = threadIdx.x & 31;
    constexpr int PL = FD_MAX_EXPERTS / 32;
    int uw[PL], run = 0;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        const int x = lane * PL + i;
        uw[i] = x < n_act ? 1 + 3 * ((p_cnt[p_act[x]] + ax - 1) / ax) : 0;
        run += uw[i] * nbh;
    }
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const long long W = __shfl_sync(0xffffffffu, incl, 31);
    const long long t0 = (long long)c * W / G, t1 = (long long)(c + 1) * W / G;
    // units whose start weight is below t: in expert x (start S), ceil((t - S) / u) of its nbh
    int n0 = 0, n1 = 0;
    long long S = incl - run;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        if (uw[i] > 0) {
            if (t0 > S) n0 += (int)min((long long)nbh, (t0 - S + uw[i] - 1) / uw[i]);
            if (t1 > S) n1 += (int)min((long long)nbh, (t1 - S + uw[i] - 1) / uw[i]);
        }
        S += (long long)uw[i] * nbh;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        n0 += __shfl_xor_sync(0xffffffffu, n0, o);
        n1 += __shfl_xor_sync(0xffffffffu, n1, o);
    }
    return make_int2(n0, n1);
}

template <typename XT, typename WT, int NB8, bool WIDE>
__global__ void __launch_bounds__(FD_THREADS, 1) k_fd_gate(FdArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[FD_MAX_SLOTS], actb[2], chb;
    __shared__ int s_ftok[FD_MAX_TOK];
    __shared__ int s_nflag, s_n_act, s_bad;
    __shared__ FdCtx C;
    __shared__ float s_hand[FD_WARPS / FD_SEG][2][32];  // fd_gu_split's running sums
    RVC_MARK(4, 2);
    const FdLayout &L = a.L;
    constexpr int nb = NB8 * 8;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int T = a.n_tok, ne = a.n_experts, used = a.used, pairs = T * used;
    const int nbh = a.ff / QK;
    const int xrb = q8rec_bytes(nb);

    uint8_t *ring = smem;
    FdScratch &SC = *reinterpret_cast<FdScratch *>(ring);  // selection phase only
    uint8_t *const act0 = smem + L.off_act;                 // x-record buffer b at act0 + b * act_bytes
    float *sgu = reinterpret_cast<float *>(smem + L.off_gu);  // [units of a wave][act_x][2][32] gate, up dots
    int32_t *p_ids = reinterpret_cast<int32_t *>(smem + L.off_plan);
    float *p_wts = reinterpret_cast<float *>(p_ids + pairs);
    int32_t *p_order = reinterpret_cast<int32_t *>(p_wts + pairs);
    int32_t *p_pos = p_order + pairs;
    int32_t *p_rank = p_pos + pairs;
    int32_t *p_cnt = p_rank + pairs;
    int32_t *p_off = p_cnt + ne;
    int32_t *p_act = p_off + ne + 1;

    if (tid == 0) {
        for (int s = 0; s < L.nslot; ++s) mbar_init(&full[s], 1);
        mbar_init(&actb[0], 1);
        mbar_init(&actb[1], 1);
        mbar_init(&chb, 1);
        fence_barrier_init();
        s_bad = 0;
    }
    __syncthreads();

    // k_fd_route's results are complete and visible past this point; k_fd_down may launch
    griddep_wait();
    griddep_launch_dependents();
    // ------------------------------------------------------------ routing
    // the ids and weights k_fd_route published (or the caller's); tokens whose order it could
    // not certify go through the reference's exact chains here, over all CTAs
    const bool route = a.ids_in == nullptr;
    if (route) {
#pragma unroll 1
        for (int i = tid; i < pairs; i += FD_THREADS) p_ids[i] = __ldcg(a.sel_ids + i), p_wts[i] = __ldcg(a.sel_wts + i);
        if (warp == FD_WARPS - 1) {  // the flagged tokens in ascending order, from two ballots (T <= 64)
            static_assert(FD_MAX_TOK <= 64, "two ballots cover the flags");
            const bool f0 = lane < T && __ldcg(a.sel_flag + lane) != 0;
            const bool f1 = lane + 32 < T && __ldcg(a.sel_flag + lane + 32) != 0;
            const unsigned b0 = __ballot_sync(0xffffffffu, f0), b1 = __ballot_sync(0xffffffffu, f1);
            const unsigned below = (1u << lane) - 1u;
            if (f0) s_ftok[__popc(b0 & below)] = lane;
            if (f1) s_ftok[__popc(b0) + __popc(b1 & below)] = lane + 32;
            if (lane == 0) s_nflag = __popc(b0) + __popc(b1);
        }
        __syncthreads();
        if (s_nflag > 0 &&
            !xfallbk<XT, WT>(static_cast<const XT *>(a.xr), static_cast<const WT *>(a.wr), a.bias, a.bias_stride,
                                 a.n_embd, ne, used, a.lexact, a.sel_ids, a.sel_wts, a.bar_cnt, a.bar_gen,
                                 a.fallback_cnt, a.status, s_ftok, s_nflag, ring, L.chain_items, &chb, p_ids, p_wts,
                                 SC.g[0]))
            return;
    } else {
#pragma unroll 1
        for (int i = tid; i < pairs; i += FD_THREADS) {
            const int e = __ldg(a.ids_in + i);
            if (e < 0 || e >= ne) s_bad = 1;
            p_ids[i] = e;
            p_wts[i] = __ldg(a.wts_in + i);
        }
    }
    __syncthreads();
    if (s_bad) {  // every CTA sees the same ids, so every CTA leaves here
        if (c == 0 && tid == 0) set_status(a.status, STATUS_BAD_INDEX);
        return;
    }

    // ------------------------------------------------------------ plan
    // stable plan (MoePlan::new, exec.rs:541-557), published by CTA 0 for k_fd_down
    if (warp == 0) {
        const int n = fd_plan_warp(p_ids, pairs, ne, p_cnt, p_rank, p_off, p_act);
        if (lane == 0) s_n_act = n;
    }
    __syncthreads();
#pragma unroll 1
    for (int q = tid; q < pairs; q += FD_THREADS) {
        const int k = p_off[p_ids[q]] + p_rank[q];
        p_pos[q] = k;
        p_order[k] = q;
    }
    __syncthreads();
    const int n_act = s_n_act;
    if (c == 0) {
        const FdPlan P = fd_plan_at(a.plan, pairs, ne);
#pragma unroll 1
        for (int q = tid; q < pairs; q += FD_THREADS) {
            P.ids[q] = p_ids[q], P.wts[q] = p_wts[q], P.pos[q] = p_pos[q], P.order[q] = p_order[q];
            if (a.ids_out) a.ids_out[q] = p_ids[q];
            if (a.wts_out) a.wts_out[q] = p_wts[q];
        }
#pragma unroll 1
        for (int e = tid; e < ne; e += FD_THREADS) P.cnt[e] = p_cnt[e], P.off[e] = p_off[e], P.act[e] = p_act[e];
        if (tid == 0) P.off[ne] = p_off[ne], *P.n_act = n_act;
    }
    RVC_MARK(4, 3);

    // ------------------------------------------------------------ stage plan
    // (expert, 32-column) units: an even split for small batches (every unit has one or two
    // tokens), split by cost for batches (fd_unit_range)
    if (WIDE && warp == 0) {
        const int2 r = fd_unit_range(c, G, n_act, nbh, L.act_x, p_cnt, p_act);
        if (lane == 0) C.n_act = n_act, C.g0 = r.x, C.n_units = r.y - r.x, C.NS = 2 * (r.y - r.x);
    } else if (!WIDE && tid == 0) {
        const int U = n_act * nbh;
        C.n_act = n_act;
        C.g0 = c * U / G;
        C.n_units = (c + 1) * U / G - C.g0;
        C.NS = 2 * C.n_units;
    }
    __syncthreads();
    const int n_units = C.n_units, NS = C.NS;
    const int AX = L.act_x;
    const bool resident = T <= AX;  // every x record fits one buffer
    // the first stages, by threads s < nslot in parallel
    const int first = min(NS, L.nslot);
    if (tid < 2 * first)
        fd_issue_gate<NB8>(C, tid >> 1, tid & 1, ring, L.slot_bytes, L.nslot, full, p_act, a.pk.gu_nib, a.pk.gu_scl,
                           a.ff);
    // warm L2 with the down tiles k_fd_down's CTA c reads first (its rows of the first
    // FD_L2_EXPERTS active experts)
    {
        int r0, rows;
        fd_rows_of(c, G, a.n_embd, L.rg, r0, rows);
        if (rows > 0 && tid >= 32 && tid - 32 < min(n_act, FD_L2_EXPERTS)) {
            const size_t row0 = (size_t)p_act[tid - 32] * a.n_embd + r0;
            bulk_prefetch_l2(a.pk.dn_nib + row0 * nbh * 16, (uint32_t)rows * nbh * 16);
            bulk_prefetch_l2(a.pk.dn_scl + row0 * nbh, (uint32_t)rows * nbh * 2);
        }
    }
    int j_issued = first;   // stages issued (the same in every thread)
    unsigned act_pend = 0;  // bit b = a load into x-record buffer b not yet waited for
    unsigned act_use = 0;   // bit b = parity of the next wait on buffer b
    int j_done = 0;         // stages consumed
    // chunk tags (when the records are not resident): expert slot x * 4096 + chunk m
    auto gu_chunks = [&](int x) { return (p_cnt[p_act[x]] + AX - 1) / AX; };
    auto issue_gu = [&](int buf, int id, int base) {  // every thread (threads base + i copy record i)
        const int x = id >> 12, m = id & 4095, e = p_act[x];
        fd_issue_records(tid - base, act0 + (size_t)buf * L.act_bytes, &actb[buf], false, p_off[e] + m * AX,
                         min(AX, p_cnt[e] - m * AX), p_order, used, a.xrec, xrb, nullptr, 0);
        act_pend |= 1u << buf;
    };
    auto after_gu = [&](int u, int id) {  // the tag after `id`, which unit u uses (-1: none)
        const int x = id >> 12, m = id & 4095;
        const int M = gu_chunks(x);
        if (m + 1 < M) return (x << 12) | (m + 1);
        if (M > 1) return u + 1 < n_units ? (((C.g0 + u + 1) / nbh) << 12) : -1;
        const int gn = (x + 1) * nbh;  // first unit of the next expert
        return gn < C.g0 + n_units ? ((x + 1) << 12) : -1;
    };
    if (n_units > 0) {
        if (resident) {  // every token's record, by token index
            if (tid == 0) {
                mbar_arrive_expect_tx(&actb[0], (uint32_t)T * xrb);
                bulk_g2s(act0, a.xrec, (uint32_t)T * xrb, &actb[0]);
            }
            act_pend |= 1u;
        } else {
            const int id0 = (C.g0 / nbh) << 12;
            issue_gu(0, id0, 0);
            const int id1 = after_gu(0, id0);
            if (id1 >= 0) issue_gu(1, id1, 0);
        }
    }
    auto wait_act = [&](int b) {
        const bool ok = fd_mbar_wait(&actb[b], (act_use >> b) & 1u, a.status);
        const bool all = !__syncthreads_or(!ok);
        act_use ^= 1u << b;
        act_pend &= ~(1u << b);
        return all;
    };

    // ------------------------------------------------------------ gate / up
    // Waves of W units (W = nslot / 2 when the records are resident, else 1): once a wave's
    // stages are in, each warp takes (unit, half, token pair) tasks, then (unit, token) tasks
    // form h = gelu(gate) * up and its Q8_0 block in the pair's plan-ordered record.
    const int W = resident ? max(1, L.nslot / 2) : 1;
    // Copies are issued by threads of the last warp after the waits, so that their issue overlaps
    // the other warps' work instead of holding up the barrier after it. Batches defer a released
    // slot's refill to the next unit's start: with nslot >= 4 (two units in the ring) the stages
    // of unit u + 1 are then issued at the start of unit u, before anyone waits for them.
    const bool defer = WIDE && L.nslot >= 4;
    int to_issue = 0;  // released stages whose refill is deferred
    int cur_buf = 1, cur_id = -1;
    if (resident && n_units > 0) {
        if (!wait_act(0)) goto fail;
        cur_buf = 0;
    }
#pragma unroll 1
    for (int u0 = 0; u0 < n_units; u0 += W) {
        const int nw = min(W, n_units - u0);
        {
            bool ok = true;
#pragma unroll 1
            for (int j = 2 * u0; j < 2 * (u0 + nw); ++j)
                ok &= fd_mbar_wait(&full[j % L.nslot], (uint32_t)(j / L.nslot) & 1u, a.status);
            if (__syncthreads_or(!ok)) goto fail;
        }
        if (u0 == 0) RVC_MARK(4, 4);
        RVC_TRACE(5, u0, 0);
        const int x_first = (C.g0 + u0) / nbh;
        const int M = resident ? 1 : gu_chunks(x_first);
#pragma unroll 1
        for (int m = 0; m < M; ++m) {
            if (!resident) {
                const int id = (x_first << 12) | m;
                if (id != cur_id) {  // switch buffers; the one left becomes free for the tag after next
                    const int nbuf = cur_id < 0 ? 0 : cur_buf ^ 1;
                    // (the barrier in wait_act also ends every read of cur_buf's records)
                    if (!wait_act(nbuf)) goto fail;
                    if (cur_id >= 0) {
                        const int n = after_gu(u0, id);
                        if (n >= 0) issue_gu(cur_buf, n, FD_THREADS - AX);
                    }
                    cur_buf = nbuf, cur_id = id;
                }
            }
            // (defer only) refill the slots the previous unit released; placed after the record
            // switch's barrier so that no barrier waits for the issuing threads
            for (; to_issue > 0; --to_issue, ++j_issued)
                if (tid >= FD_THREADS - 2)
                    fd_issue_gate<NB8>(C, j_issued, tid - (FD_THREADS - 2), ring, L.slot_bytes, L.nslot, full, p_act,
                                       a.pk.gu_nib, a.pk.gu_scl, a.ff);
            RVC_TRACE(5, u0, 1);
            const uint8_t *recs = act0 + (size_t)cur_buf * L.act_bytes;
            if constexpr (WIDE) {  // one unit per wave: warps 0-7 the gate half, 8-15 the up half
                const int e = p_act[(C.g0 + u0) / nbh], nt = min(AX, p_cnt[e] - m * AX), half = warp >> 3;
                const uint8_t *slot = ring + (size_t)((2 * u0 + half) % L.nslot) * L.slot_bytes;
#pragma unroll 1
                for (int i = 0; i < nt; i += 2) {
                    const bool two = i + 1 < nt;
                    const float2 acc =
                        fd_gu_wide<NB8>(slot, recs + (size_t)i * xrb, recs + (size_t)(two ? i + 1 : i) * xrb, two);
                    if ((lane & 7) == 0) {  // token slot (m % FD_HB) * AX + i of the h phase's batch
                        float *dst = sgu + ((size_t)((m % FD_HB) * AX + i) * 2 + half) * 32 + (warp & 7) * 4 + (lane >> 3);
                        dst[0] = acc.x;
                        if (two) dst[64] = acc.y;
                    }
                }
            } else {
            // tasks (w, half, token pair): unit w of the wave has nt_w tokens in this chunk; each
            // task split over FD_SEG warps (fd_gu_split)
            int ntask = 0;
#pragma unroll 1
            for (int w = 0; w < nw; ++w) {
                const int e = p_act[(C.g0 + u0 + w) / nbh];
                const int nt = resident ? p_cnt[e] : min(AX, p_cnt[e] - m * AX);
                ntask += 2 * ((nt + 1) / 2);
            }
#pragma unroll 1
            for (int t0 = 0; t0 < ntask; t0 += FD_WARPS / FD_SEG) {  // uniform: fd_gu_split syncs the CTA
                const int task = t0 + warp / FD_SEG;
                const bool active = task < ntask;
                const uint8_t *slot = ring, *r0p = recs, *r1p = recs;
                bool two = false;
                float *dst = sgu;
                if (active) {
                    int w = 0, k = task, nt = 0, e = 0;
#pragma unroll 1
                    for (;; ++w) {
                        e = p_act[(C.g0 + u0 + w) / nbh];
                        nt = resident ? p_cnt[e] : min(AX, p_cnt[e] - m * AX);
                        const int n = 2 * ((nt + 1) / 2);
                        if (k < n) break;
                        k -= n;
                    }
                    const int half = k & 1, i = (k >> 1) * 2;  // tokens i, i + 1 of the chunk
                    two = i + 1 < nt;
                    const int pa = p_off[e] + m * AX + i;
                    r0p = resident ? recs + (size_t)(p_order[pa] / used) * xrb : recs + (size_t)i * xrb;
                    r1p = !two ? r0p : (resident ? recs + (size_t)(p_order[pa + 1] / used) * xrb : r0p + xrb);
                    slot = ring + (size_t)((2 * (u0 + w) + half) % L.nslot) * L.slot_bytes;
                    dst = sgu + ((size_t)(w * AX + i) * 2 + half) * 32;
                }
                fd_gu_split<NB8>(slot, r0p, r1p, two, active, &s_hand[0][0][0], dst);
            }
            }
            // h = gelu(gate) * up and its Q8_0 block per (unit, token): after each chunk, or for
            // batches after every FD_HB chunks of the unit and its last one (their dots wait in sgu's
            // FD_HB * AX token slots; the next chunk's record switch is a barrier, and it writes
            // other slots)
            int hm0 = m, nh = 0;
            if constexpr (WIDE) {
                if (m % FD_HB != FD_HB - 1 && m != M - 1) continue;
                hm0 = m - m % FD_HB;
                nh = min(p_cnt[p_act[x_first]], (m + 1) * AX) - hm0 * AX;
            } else {
#pragma unroll 1
                for (int w = 0; w < nw; ++w) {
                    const int e = p_act[(C.g0 + u0 + w) / nbh];
                    nh += resident ? p_cnt[e] : min(AX, p_cnt[e] - m * AX);
                }
            }
            __syncthreads();
            RVC_TRACE(5, u0, 2);
            const int hrb = q8rec_bytes(nbh);
#pragma unroll 1
            for (int task = warp; task < nh; task += FD_WARPS) {
                int w = 0, i = task, e = p_act[x_first];  // batches: token i of chunks hm0.. (slot i)
                if constexpr (!WIDE) {
#pragma unroll 1
                    for (;; ++w) {
                        e = p_act[(C.g0 + u0 + w) / nbh];
                        const int nt = resident ? p_cnt[e] : min(AX, p_cnt[e] - m * AX);
                        if (i < nt) break;
                        i -= nt;
                    }
                }
                const float *g = sgu + ((size_t)(w * AX + i) * 2) * 32;
                const float hv = __fmul_rn(gelu_tanh(g[lane]), g[32 + lane]);
                uint16_t dbits;
                int qsum;
                const int8_t qv = quant_q8_lane(hv, &dbits, &qsum);
                q8rec_store(a.hrec + (size_t)(p_off[e] + hm0 * AX + i) * hrb, nbh, (C.g0 + u0 + w) % nbh, lane, qv,
                            dbits, qsum);
            }
            __syncthreads();
        }
        // release the wave's slots
        __syncthreads();
        RVC_TRACE(5, u0, 3);
#pragma unroll 1
        for (; j_done < 2 * (u0 + nw); ++j_done)
            if (j_issued + to_issue < NS) {
                if (defer) {
                    ++to_issue;
                    continue;
                }
                if (tid < 2)
                    fd_issue_gate<NB8>(C, j_issued, tid, ring, L.slot_bytes, L.nslot, full, p_act, a.pk.gu_nib,
                                       a.pk.gu_scl, a.ff);
                ++j_issued;
            }
    }
    RVC_MARK(4, 5);
    return;
fail:
    xdrain(full, L.nslot, j_done, j_issued, actb, act_pend, act_use);
}

// -------------------------------------------------------------- k_fd_down (3 of 3)
// Down projection and slot-order combine: CTA c owns output rows [r0, r0 + rows) for every
// pair; its tiles of up to eps experts per ring slot (mostly L2 hits: k_fd_gate prefetched
// them), the h records of those experts' pairs double-buffered beside them.
__global__ void __launch_bounds__(FD_THREADS, 1) k_fd_down(FdArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[FD_MAX_SLOTS], actb[2];
    __shared__ FdCtx C;
    RVC_MARK(4, 6);
    griddep_wait();  // k_fd_gate's plan and h records are complete and visible past this point
    const FdLayout &L = a.L;
    const int tid = threadIdx.x;
    const int G = gridDim.x, c = blockIdx.x;
    const int T = a.n_tok, ne = a.n_experts, used = a.used, pairs = T * used;
    const int nbh = a.ff / QK, hrb = q8rec_bytes(nbh);
    uint8_t *ring = smem;
    uint8_t *const act0 = smem + L.d_off_act;
    float *ys = reinterpret_cast<float *>(smem + L.d_off_y);  // [pairs][rpc_max]
    int32_t *p_ids = reinterpret_cast<int32_t *>(smem + L.d_off_plan);
    float *p_wts = reinterpret_cast<float *>(p_ids + pairs);
    int32_t *p_pos = reinterpret_cast<int32_t *>(p_wts + pairs);
    int32_t *p_cnt = p_pos + pairs;
    int32_t *p_off = p_cnt + ne;
    int32_t *p_act = p_off + ne + 1;
    const FdPlan P = fd_plan_at(a.plan, pairs, ne);
    if (tid == 0) {
        for (int s = 0; s < L.d_nslot; ++s) mbar_init(&full[s], 1);
        mbar_init(&actb[0], 1);
        mbar_init(&actb[1], 1);
        fence_barrier_init();
        C.n_act = *P.n_act;
        fd_rows_of(c, G, a.n_embd, L.rg, C.r0, C.rows);
        C.dn_nib = (uint32_t)C.rows * nbh * 16;
        C.tile = C.dn_nib + (uint32_t)C.rows * nbh * 2;
        C.eps = C.rows > 0 ? (int)(L.d_slot_bytes / C.tile) : 1;
        C.NS = C.rows > 0 ? (C.n_act + C.eps - 1) / C.eps : 0;
    }
#pragma unroll 1
    for (int q = tid; q < pairs; q += FD_THREADS) p_ids[q] = P.ids[q], p_wts[q] = P.wts[q], p_pos[q] = P.pos[q];
#pragma unroll 1
    for (int e = tid; e < ne; e += FD_THREADS) p_cnt[e] = P.cnt[e], p_off[e] = P.off[e], p_act[e] = P.act[e];
    __syncthreads();
    const int NS = C.NS, rows = C.rows, AH = L.act_h;
    const int first = min(NS, L.d_nslot);
    if (tid < first * C.eps)
        fd_issue_down(C, tid / C.eps, tid % C.eps, ring, L.d_slot_bytes, L.d_nslot, full, p_act, a.pk.dn_nib,
                      a.pk.dn_scl, a.n_embd, nbh);
    int j_issued = first, j_done = 0;
    unsigned act_pend = 0, act_use = 0;
    // Copies after the first are issued by the highest threads (the tiles by the last eps, the
    // records by the one below them), after the waits that free their buffers, so that issuing
    // overlaps the dot products (a stage's items go to the lowest threads first) instead of
    // holding up a barrier. A released slot is refilled at the next stage's start: with two or
    // more slots, stage k + 1 has been issued before anyone waits for it.
    const int rec_thr = FD_THREADS - 1 - C.eps, tile_thr = FD_THREADS - C.eps;
    int to_issue = 0;
    // h-record tags: down stage k * 4096 + chunk m, each its own load
    auto dn_chunks = [&](int k) {
        const int2 q = fd_dn_pairs(C, k, p_act, p_off, p_cnt);
        return (q.y - q.x + AH - 1) / AH;
    };
    auto issue_dn = [&](int buf, int id, int thr) {  // (thread thr copies)
        const int k = id >> 12, m = id & 4095;
        const int2 q = fd_dn_pairs(C, k, p_act, p_off, p_cnt);
        const int s0 = q.x + m * AH;
        fd_issue_records(tid - thr, act0 + (size_t)buf * L.d_act_bytes, &actb[buf], true, s0, min(AH, q.y - s0), nullptr, used,
                         nullptr, 0, a.hrec, hrb);
        act_pend |= 1u << buf;
    };
    auto next_dn = [&](int id) {
        const int k = id >> 12, m = id & 4095;
        if (m + 1 < dn_chunks(k)) return (k << 12) | (m + 1);
        return k + 1 < NS ? ((k + 1) << 12) : -1;
    };
    int cur_buf = 1, cur_id = -1;
    if (NS > 0) {
        issue_dn(0, 0, rec_thr);
        const int id1 = next_dn(0);
        if (id1 >= 0) issue_dn(1, id1, rec_thr);
    }
#pragma unroll 1
    for (int k = 0; k < NS; ++k) {
        const int alo = k * C.eps, ahi = min(C.n_act, alo + C.eps);
        const int2 qr = fd_dn_pairs(C, k, p_act, p_off, p_cnt);
        RVC_TRACE(6, k, 0);
        if (__syncthreads_or(!fd_mbar_wait(&full[k % L.d_nslot], (uint32_t)(k / L.d_nslot) & 1u, a.status))) goto fail;
        RVC_TRACE(6, k, 1);
        {
            const uint8_t *slot = ring + (size_t)(k % L.d_nslot) * L.d_slot_bytes;
            const int M = (qr.y - qr.x + AH - 1) / AH;
#pragma unroll 1
            for (int m = 0; m < M; ++m) {
                const int id = (k << 12) | m;
                const int nbuf = cur_buf ^ 1;  // every chunk is a new tag
                {  // (the barrier also ends every read of cur_buf's records)
                    const bool ok = fd_mbar_wait(&actb[nbuf], (act_use >> nbuf) & 1u, a.status);
                    act_use ^= 1u << nbuf;
                    act_pend &= ~(1u << nbuf);
                    if (__syncthreads_or(!ok)) goto fail;
                }
                if (cur_id >= 0) {
                    const int n = next_dn(id);
                    if (n >= 0) issue_dn(cur_buf, n, rec_thr);
                }
                // refill the slot the previous stage released (after the barrier above, so that
                // no barrier waits for the issuing threads)
                for (; to_issue > 0; --to_issue, ++j_issued)
                    if (tid >= tile_thr)
                        fd_issue_down(C, j_issued, tid - tile_thr, ring, L.d_slot_bytes, L.d_nslot, full, p_act,
                                      a.pk.dn_nib, a.pk.dn_scl, a.n_embd, nbh);
                cur_buf = nbuf, cur_id = id;
                RVC_TRACE(6, k, 2);
                const uint8_t *recs = act0 + (size_t)cur_buf * L.d_act_bytes;
                const int s0 = qr.x + m * AH, np = min(AH, qr.y - s0);
#pragma unroll 1
                for (int it = tid; it < np * rows; it += FD_THREADS) {
                    const int pl = it / rows, rr = it - pl * rows, pos = s0 + pl;
                    int x = alo;
                    while (x + 1 < ahi && p_off[p_act[x + 1]] <= pos) ++x;
                    const uint8_t *t0 = slot + (size_t)(x - alo) * C.tile;
                    const float acc = fd_dn_row(t0 + (size_t)rr * nbh * 16,
                                                reinterpret_cast<const uint16_t *>(t0 + C.dn_nib) + rr * nbh,
                                                recs + (size_t)pl * hrb, nbh, (C.r0 + rr) & 7);
                    if (L.y_in_smem)
                        ys[(size_t)pos * L.rpc_max + rr] = acc;
                    else
                        a.ybuf[(size_t)pos * a.n_embd + C.r0 + rr] = acc;
                }
            }
        }
        __syncthreads();  // release the slot (refilled at the next stage's start)
        RVC_TRACE(6, k, 3);
        j_done = k + 1;
        if (j_issued + to_issue < NS) ++to_issue;
    }
    // slot-order combine (exec.rs:626-638): o = (y*ds)*w for j = 0, then o = o + (y*ds)*w
#pragma unroll 1
    for (int i = tid; i < T * rows; i += FD_THREADS) {
        const int t = i / rows, rr = i - t * rows;
        float o = 0.0f;
#pragma unroll 1
        for (int jj = 0; jj < used; ++jj) {
            const int p = t * used + jj;
            const int e = p_ids[p];
            const float ds = a.down_scale ? __ldg(a.down_scale + e) : 1.0f;
            const int k = p_pos[p];
            const float y = L.y_in_smem ? ys[(size_t)k * L.rpc_max + rr] : a.ybuf[(size_t)k * a.n_embd + C.r0 + rr];
            const float v = __fmul_rn(__fmul_rn(y, ds), p_wts[p]);
            o = jj == 0 ? v : __fadd_rn(o, v);
        }
        a.out[(size_t)t * a.n_embd + C.r0 + rr] = o;
    }
    RVC_MARK(4, 7);
    return;
fail:
    xdrain(full, L.d_nslot, j_done, j_issued, actb, act_pend, act_use);
}

}  // namespace rvc
