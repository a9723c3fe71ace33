/* rvcuda.h - C ABI of the B200 (sm_100a) MoE-layer backend, librvcuda.so.
 *
 * Drop-in for the expert path of Rosevine's HIP executor. It keeps the conventions of the
 * reference ABI runtime/hip/rvhip.h:1-14: every function returns 0 or a CUDA error code
 * (cudaError_t values; RVC_ERR_* below for backend-specific failures), rvc_error_string()
 * returns a static string, no exception crosses the ABI, scalar arguments are validated
 * here and buffer extents are the caller's contract (the host wrapper range-checks every
 * view against its allocation, as runtime/src/hip.rs:258-263 does).
 *
 * Differences, all additive (the reference's ADR plans stream-taking entry points,
 * docs/adr/0002-expert-residency-and-scheduling.md:353-358):
 *  - compute entry points take a trailing `void *stream` (a cudaStream_t; NULL = the
 *    legacy default stream, which orders work like the reference's null stream);
 *  - compute entry points take a caller-allocated device workspace (rvc_alloc) sized by
 *    rvc_moe_workspace_bytes(); nothing allocates during a call.
 *
 * Layouts:
 *  - Q4_0 expert tensors as bound by runtime/src/model.rs:36-40 (GGUF): gate_up
 *    [n_experts][2*ff rows][n_embd/32 blocks of 18 B] (gate rows then up rows), down
 *    [n_experts][n_embd rows][ff/32 blocks]. rvc_pack_experts turns them into the packed
 *    device planes every MoE entry point reads.
 *  - Router weight [n_experts][n_embd] (ggml dims [n_embd, n_experts],
 *    runtime/src/contract.rs:66), f32 (the reference model) or bf16 (the benchmark).
 *  - Activations row-major [n_tok][n_embd], f32 or bf16; outputs f32.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Element types of activations and router weights. */
#define RVC_F32 0
#define RVC_BF16 1

/* Backend error codes (outside the cudaError_t range). */
#define RVC_ERR_DEVICE_TIMEOUT 10001 /* a bounded device wait ran out (status word) */
#define RVC_ERR_DEVICE_INDEX 10002   /* a device-side index check failed (status word) */
#define RVC_ERR_UNSUPPORTED 10003    /* shape outside what the kernels support */
#define RVC_ERR_WORKSPACE 10004      /* workspace too small for this call */
#define RVC_ERR_GGUF 10100           /* + a reason: malformed or unusable GGUF file (rvc_error_string) */

/* ---------------------------------------------------------------- runtime
 * 1:1 with runtime/hip/rvhip.h:22-38 (rvh_init ... rvh_event_elapsed). */
int rvc_init(int device);                                    /* rvhip.h:22 */
int rvc_mem_info(size_t *free_bytes, size_t *total_bytes);   /* rvhip.h:23 */
int rvc_alloc(size_t bytes, void **out);                     /* rvhip.h:24 */
int rvc_free(void *ptr);                                     /* rvhip.h:25 */
int rvc_upload(void *dst, const void *src, size_t bytes);    /* rvhip.h:26 */
int rvc_download(void *dst, const void *src, size_t bytes);  /* rvhip.h:27 */
int rvc_copy(void *dst, const void *src, size_t bytes);      /* rvhip.h:28, device to device */
int rvc_sync(void);                                          /* rvhip.h:29 */
const char *rvc_error_string(int code);                      /* rvhip.h:30 */
int rvc_event_create(void **out);                            /* rvhip.h:34 */
int rvc_event_destroy(void *ev);                             /* rvhip.h:35 */
int rvc_event_record(void *ev);                              /* rvhip.h:36 */
int rvc_event_sync(void *ev);                                /* rvhip.h:37 */
int rvc_event_elapsed(void *start, void *end, float *ms);    /* rvhip.h:38 */
/* Stream-ordered variants (additive): async copies and events on `stream`. */
int rvc_upload_async(void *dst, const void *src, size_t bytes, void *stream);
int rvc_download_async(void *dst, const void *src, size_t bytes, void *stream);
int rvc_event_record_on(void *ev, void *stream);
int rvc_stream_sync(void *stream);

/* ---------------------------------------------------------------- norms
 * rvh_rms_norm (rvhip.h:43, rvhip.hip:75-90) with a stream: per row of x [rows][width] f32,
 * mean of squares summed in f64 and rounded to f32, scale = 1 / sqrt(mean + eps), out =
 * x * scale (* post when post != 1) (* weight[i] when weight is not NULL). out may be x. The
 * MoE branch's three norms (hip_exec.rs:786, :796, :846) call this. */
int rvc_rms_norm(const float *x, float *out, const float *weight, int rows, int width, float eps, float post,
                 void *stream);

/* ------------------------------------------------------------- MoE layer */

/* Weights of one MoE layer, as runtime/src/model.rs:11-41 binds them (gate_inp,
 * down_exps_scale, gate_up_exps, down_exps), with the experts already packed.
 * Shapes of the target (runtime/src/contract.rs:12-22): n_embd 2816, ff 704,
 * n_experts 128, used 8. Supported: n_embd % 256 == 0, ff % 32 == 0,
 * n_experts <= 256, used <= 16. */
typedef struct rvc_moe_weights {
    int n_embd;
    int ff;
    int n_experts;
    int used;
    int router_dtype;         /* RVC_F32 or RVC_BF16 */
    const void *router;       /* device [n_experts][n_embd] */
    const void *packed;       /* device, from rvc_pack_experts */
    const float *down_scale;  /* device [n_experts], or NULL for all ones */
} rvc_moe_weights;

/* Bytes of the packed expert planes: the GGUF bytes of both tensors (nibble and f16 scale
 * planes) plus, for shapes the prefill GEMM takes (2 ff and n_embd multiples of 128), an f32
 * copy of the scales in 128-row tiles. */
size_t rvc_packed_bytes(int n_experts, int n_embd, int ff);

/* One-time repack at upload, replacing the raw uploads of runtime/src/hip_exec.rs:429-433.
 * gate_up / down: device copies of the GGUF tensors. packed: rvc_packed_bytes() bytes. */
int rvc_pack_experts(const void *gate_up_q4, const void *down_q4, int n_experts, int n_embd, int ff, void *packed,
                     void *stream);

/* Device workspace for calls of up to max_tok tokens. */
size_t rvc_moe_workspace_bytes(int max_tok, int n_embd, int ff, int n_experts, int used);

/* Router: logits = router . x (+ bias), softmax, top-`used`, renormalised weights, and the
 * dispatch plan. Replaces rvh_rms_norm+rvh_f32_mm (hip_exec.rs:786-787, rvhip.h:43,50), the
 * logits download (:789) and the host select_experts / MoePlan::new (runtime/src/exec.rs:
 * 507-558). The caller applies the router-input norm, as the reference does before f32_mm.
 * bias: optional f32 logit bias, bias[t*bias_stride + e] (stride 0 = one row for all tokens).
 * Outputs (device, each may be NULL): ids/wts [n_tok][used] in slot order; hist
 * [n_experts] pairs per expert; perm [n_tok*used] the pair order of MoePlan (pair = t*used+j);
 * logits [n_tok][n_experts]. */
int rvc_moe_router(const rvc_moe_weights *w, const void *x, int x_dtype, const float *bias, int bias_stride,
                   int n_tok, int32_t *ids, float *wts, int32_t *hist, int32_t *perm, float *logits, void *workspace,
                   size_t workspace_bytes, void *stream);

/* Routed experts for given ids/weights: Q8_0 activations, gate/up with GELU-tanh, Q8_0 h,
 * down, and the slot-order weighted combine into out [n_tok][n_embd] f32 (before
 * post_ffw_norm_2). Replaces hip_exec.rs:820-843 (gather_rows, per-expert q4_mm,
 * geglu_split, q4_mm, moe_combine; rvhip.h:44,71,77-80) and computes what experts_cpu
 * (runtime/src/exec.rs:572-640) computes with Activation::Q8_0. */
int rvc_moe_experts(const rvc_moe_weights *w, const void *x_expert, int x_dtype, const int32_t *ids,
                    const float *wts, int n_tok, float *out, void *workspace, size_t workspace_bytes, void *stream);

/* The whole MoE layer: rvc_moe_router on x_router, then rvc_moe_experts on x_expert (the
 * reference's layer() MoE branch, hip_exec.rs:780-843, between its norms). ids/wts may be
 * NULL. x_router and x_expert may be the same buffer. */
int rvc_moe_forward(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype,
                    const float *bias, int bias_stride, int n_tok, float *out, int32_t *ids, float *wts,
                    void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- expert parallelism
 * No reference counterpart: the reference runs every expert on one device. Rank r of N holds
 * experts [r n_local, (r + 1) n_local). A rank routes its own tokens (rvc_moe_router), quantises
 * them once (rvc_quant_q8_rows), packs one row per (token, destination rank) (rvc_ep_pack), runs
 * its resident experts on the rows it receives (rvc_ep_experts) and sums the partial outputs
 * returned for its tokens (rvc_ep_reduce); the exchanges between these calls are the caller's
 * (NCCL all-to-allv of rvc_ep_row_bytes-byte rows, and of n_embd f32 partials back). */

/* Bytes of one Q8_0 row record of this backend: quants 0-15 of every 32-element block (16 int8
 * each), then quants 16-31 of every block, then all blocks' f32 scales, then all blocks' int32
 * quant sums (n_embd / 32 * 40 bytes). */
size_t rvc_q8_record_bytes(int n_embd);

/* Bytes of one sent row: a record, then `used` int32 local expert ids (-1: the slot's expert is on
 * another rank) and `used` f32 routing weights, in the token's slot order. */
size_t rvc_ep_row_bytes(int n_embd, int used);

/* Q8_0 records (quantised as the reference quantises activations) of x [n_rows][n_embd]. */
int rvc_quant_q8_rows(const void *x, int x_dtype, int n_rows, int n_embd, void *records, void *stream);

/* Rows to send, grouped by destination rank (rank order; rows within a group in arrival order):
 * a token goes once to every rank holding one of its experts. counts [2 * world] int32: on
 * return counts[r] = rows for rank r (counts[world ..] is scratch); send holds up to
 * n_tok * world rows; owner_map [n_tok][world] = the row of (token, rank) in send, or -1. */
int rvc_ep_pack(const int32_t *ids, const float *wts, const void *records, int n_tok, int used, int n_embd,
                int n_local, int world, int32_t *counts, void *send, int32_t *owner_map, int *status, void *stream);

/* Workspace for rvc_ep_experts calls of up to max_rows received rows. */
size_t rvc_ep_workspace_bytes(int max_rows, int used, int n_embd, int ff, int n_experts);

/* The resident experts (w: this rank's n_experts, ids local) over n_rows received rows.
 * partial[r] [n_embd] f32 = slot-order sum over the row's occupied slots of (y * down_scale[e])
 * * w, y the expert output of the reference's CPU-experts Q8_0 path (block dots exact, each
 * (row, expert) y bit-identical to that path's). */
int rvc_ep_experts(const rvc_moe_weights *w, const void *rows, int n_rows, int used, float *partial, void *workspace,
                   size_t workspace_bytes, void *stream);

/* out[t] = the partials back[owner_map[t][r]] over the ranks r with owner_map[t][r] >= 0, added in
 * rank order (f32); a token sent nowhere gets zeros. */
int rvc_ep_reduce(const float *back, const int32_t *owner_map, int n_tok, int world, int n_embd, float *out,
                  void *stream);

/* Zero the workspace's status word (call once after allocating a workspace). */
int rvc_workspace_reset(void *workspace, void *stream);

/* Synchronise `stream`, then read and clear the workspace's device status word:
 * returns 0, RVC_ERR_DEVICE_TIMEOUT or RVC_ERR_DEVICE_INDEX. */
int rvc_status(void *workspace, void *stream);

/* rvc_moe_forward without a caller workspace (no counterpart in the reference; added for
 * hosts that cannot allocate device memory per call - their VRAM is pre-carved by their own
 * allocator, or a decode step must never risk a failing or synchronising allocation).
 * Scratch comes from a fixed array of RVC_NOALLOC_SCRATCH_BYTES inside librvcuda.so, which
 * every GPU that loads the library holds until the process exits; that is room for 64
 * tokens at the target's shapes. Calls needing more return RVC_ERR_WORKSPACE. Nothing is
 * allocated. The first call on a device looks up the array's device address (make that
 * first call before any stream capture). All calls share the one array: calls that may
 * overlap on the GPU (other streams, other threads) race and must be serialised by the
 * caller. Device status (bounded-wait timeouts) is cleared at the start of every call and
 * is not reported by this entry point. */
#define RVC_NOALLOC_SCRATCH_BYTES (8u << 20)
int rvc_moe_forward_noalloc(const rvc_moe_weights *w, const void *x_router, const void *x_expert, int x_dtype,
                            const float *bias, int bias_stride, int n_tok, float *out, int32_t *ids, float *wts,
                            void *stream);

/* Measurement hook (no counterpart in the reference): enqueue on `stream`, again, the two
 * grouped expert GEMMs (gate/up with GELU and h quantisation, then down) of the last
 * rvc_moe_forward call of more than 64 tokens enqueued with this workspace and these weights,
 * on the plan, records and scale planes that call left in the workspace. The GEMMs rewrite the
 * same h records and y, so the layer's outputs stay as they were. Lets a caller time the
 * layer's dominant kernels alone with events on `stream`. Returns cudaErrorInvalidValue if no
 * such call was made with this workspace and these weights, or if any other entry point has
 * been given the workspace since (rvc_workspace_reset included). Calls on the workspace from
 * other streams must be ordered by the caller, as for every entry point. */
int rvc_prefill_gemms(const rvc_moe_weights *w, void *workspace, size_t workspace_bytes, void *stream);

/* Test hook: the exact int32 Q4_0 x Q8_0 block sums the expert kernels form, for
 * `n_rows` rows of one expert of the packed weights against Q8_0 activation rows.
 * which: 0 = gate_up (original row numbering), 1 = down. xq8: device [n_in][nblk*34]
 * (reference Q8_0 blocks). out: device int32 [n_in][n_rows][nblk]. */
int rvc_debug_block_sums(const rvc_moe_weights *w, int which, int expert, const int32_t *rows, int n_rows,
                         const void *xq8, int n_in, int32_t *out, void *stream);

/* Test hook (no counterpart in the reference): the integer block dots of one tile of the prefill
 * GEMM, formed by the production kernel (k_pf_gemm_tc: weight unpack, TMA copies, tcgen05.mma
 * into tensor memory with the integer operands held exactly as f16, tensor-memory loads) in a
 * mode whose epilogue writes the dots instead of scaling them. The tile: rows row_tile*128 ..
 * +127 of expert `expert`'s gate_up (which = 0; packed row order, gate and up interleaved per 32
 * rows) or down (which = 1) rows, against n (1..128) activation rows in the GEMM's operand
 * layout: per 32-element block of n_embd (which = 0) or ff (which = 1) columns, the 32 Q8_0
 * quants as f16 integers (64 bytes; device, 16-byte aligned). out: device int32 [nblk][128
 * positions][128 rows]; positions >= n read 0. scratch: device, 256-byte aligned, at least
 * 256 + nblk * 4 * round_up(n, 4) bytes; its int at byte 12 receives the kernel's status bits. */
int rvc_debug_gemm_block_dots(const rvc_moe_weights *w, int which, int expert, int row_tile, const void *records,
                              int n, int32_t *out, void *scratch, size_t scratch_bytes, void *stream);

/* ---------------------------------------------------------------- shared dense MLP
 * The layer's dense gated MLP beside the experts (runtime/src/exec.rs:438-453 on the CPU,
 * runtime/src/hip_exec.rs:770-778 on the device), Q4_0 weights in the GGUF layout as bound by
 * runtime/src/model.rs:30-32 (ffn_gate / ffn_up [ff rows][n_embd/32 blocks of 18 B], ffn_down
 * [n_embd rows][ff/32 blocks]) and F32 activations. Every dot is the CPU reference's sequential
 * f32 sum of rounded products (ops.rs:249-266), so results equal the CPU reference's bit for bit
 * and do not depend on the batch. */

/* y[t][r] = W[r] . x[t]; W Q4_0 n_out x k (k a multiple of 32), x n_in x k (16-byte aligned).
 * rvhip.h:45 (rvh_q4_mm) with a stream. */
int rvc_q4_mm(const void *w, const float *x, float *y, int n_out, int k, int n_in, void *stream);
/* out[i] = gelu(g[i]) * u[i] (rvhip.h:65, rvh_geglu). */
int rvc_geglu(const float *g, const float *u, float *out, int n, void *stream);
/* Workspace of rvc_shared_mlp calls of up to max_tok tokens. */
size_t rvc_shared_mlp_workspace_bytes(int max_tok, int n_embd, int ff);
/* out = rms_norm(Wd . (gelu(Wg . c) * (Wu . c))) * post_norm with c = rms_norm(x) * ffn_norm
 * (exec.rs:438-453): x, out [n_tok][n_embd] f32 (out 16-byte aligned); gate and up fused in
 * one kernel with the GELU product. Four launches on `stream`. */
int rvc_shared_mlp(const void *w_gate, const void *w_up, const void *w_down, const float *ffn_norm,
                   const float *post_norm, const float *x, float *out, int n_tok, int n_embd, int ff, float eps,
                   void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- GGUF weights (host only)
 * The reference reads the model with its own GGUF parser (runtime/src/gguf.rs, Gguf::parse) and
 * binds tensors by name (runtime/src/model.rs:61-107, Weights::bind). These calls do the same for
 * the MoE layer: the file is mapped read-only, validated with the reference parser's checks
 * (a file it rejects is rejected here, the reason as its message: rvc_error_string of the
 * RVC_ERR_GGUF + reason code), and tensors are views into the mapping, valid until
 * rvc_gguf_close. Tensor types: F32 and Q4_0, as the reference accepts. */
typedef struct rvc_gguf rvc_gguf;

/* Map and validate a GGUF v3 file (gguf.rs:272-383 replaces). */
int rvc_gguf_open(const char *path, rvc_gguf **out);
/* The same over a caller's buffer (not copied: it must outlive the handle). */
int rvc_gguf_parse(const void *buf, size_t len, rvc_gguf **out);
void rvc_gguf_close(rvc_gguf *g);
/* A tensor by name (gguf.rs, Gguf::tensor): ggml type (0 F32, 2 Q4_0), rank, shape[4] (ggml
 * order: shape[0] is the innermost dimension; unused dimensions 1), its bytes in the mapping. */
int rvc_gguf_tensor(const rvc_gguf *g, const char *name, int *dtype, int *n_dims, uint64_t *shape, const void **data,
                    uint64_t *bytes);

/* Host views of one layer's MoE tensors, each checked against the target contract's shape and
 * type (runtime/src/contract.rs:42-51, 66-70): gate_up and down are rvc_pack_experts' inputs. */
typedef struct {
    const void *gate_up;          /* Q4_0 ggml [n_embd, 2 ff, n_experts]: blk.L.ffn_gate_up_exps.weight */
    const void *down;             /* Q4_0 ggml [ff, n_embd, n_experts]: blk.L.ffn_down_exps.weight */
    const float *router;          /* F32 [n_experts][n_embd]: blk.L.ffn_gate_inp.weight */
    const float *down_scale;      /* [n_experts]: blk.L.ffn_down_exps.scale */
    const float *gate_inp_scale;  /* [n_embd]: blk.L.ffn_gate_inp.scale (router input norm) */
    const float *pre_norm;        /* [n_embd]: blk.L.pre_ffw_norm_2.weight (expert input norm) */
    const float *post_norm;       /* [n_embd]: blk.L.post_ffw_norm_2.weight (output norm) */
} rvc_gguf_moe;
/* model.rs:61-107 (Weights::bind) for one layer's MoE branch. */
int rvc_gguf_moe_layer(const rvc_gguf *g, int layer, int n_embd, int ff, int n_experts, rvc_gguf_moe *out);

#ifdef __cplusplus
}
#endif
