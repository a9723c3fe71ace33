/* rv_oracle.h - CPU restatement of Rosevine's Q8_0 CPU-experts MoE path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * product path and the timed CPU baseline ("port") of bench.py. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * may load it. The product library (librvcuda.so) never links or calls it.
 *
 * Every function restates the reference algorithm it names (paths relative to
 * the Rosevine project root). Arithmetic order follows the reference so that
 * results are bit-identical to the Rust code on the same glibc: f32 operations
 * are never contracted (built with -ffp-contract=off); f32 exp/tanh are the correctly
 * rounded results of the libm functions Rust's f32::exp / f32::tanh call (rv_oracle.c).
 *
 * Parity pins: tests/test_oracle_golden.py checks this code against the
 * reference's own known-answer tests (ops.rs, expert_kernel.rs, exec.rs tests)
 * and against fixtures generated from the reference's binary64 scalar oracle
 * (scripts/correctness_oracle.py) by tests/golden/make_golden.py.
 *
 * Layouts (the reference's, model.rs:31-40, contract.rs:66-70):
 *   Q4_0 block: 18 B = f16 d (LE) + 16 B nibbles; element j (j<16) is
 *     (qs[j] & 15) - 8, element j+16 is (qs[j] >> 4) - 8, times d.
 *   Q8_0 block: 34 B = f16 d + 32 x int8.
 *   gate_up: [n_experts][2*ff rows][k/32 blocks] (gate rows first, then up).
 *   down:    [n_experts][n_embd rows][ff/32 blocks].
 *   router:  [n_experts rows][n_embd] (f32 in the reference, bf16 in the
 *            benchmark configs).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

enum { RVO_F32 = 0, RVO_BF16 = 1 };
enum { RVO_KERNEL_SCALAR = 0, RVO_KERNEL_AVX2 = 1, RVO_KERNEL_BEST = 2 };

/* ops.rs:7-24 */
float rvo_f16_to_f32(uint16_t h);
/* ops.rs:27-59 */
uint16_t rvo_f32_to_f16(float f);
float rvo_bf16_to_f32(uint16_t b);
/* ops.rs:95-105: x has k (multiple of 32) values; out gets k/32 * 34 bytes. */
void rvo_quantize_q8_0(const float *x, int k, uint8_t *out);
/* f32 exp / tanh, correctly rounded (see rv_oracle.c) */
float rvo_expf(float x);
float rvo_tanhf(float x);
/* ops.rs:145-149 */
float rvo_gelu(float x);
/* ops.rs:170-179 (in place) */
void rvo_softmax(float *x, int n);
/* ops.rs:182-187: indices of the k largest, descending, ties to lower index. */
void rvo_top_k(const float *x, int n, int k, int32_t *idx);
/* ops.rs:321-326 / exec.rs:493-503: logits[t][e] = sum_k w[e][k] * x[t][k],
 * sequential f32, plus bias[t * bias_stride + e] when bias != NULL. */
void rvo_router_logits(const void *x, int x_dtype, const void *w, int w_dtype, const float *bias, int bias_stride,
                       int n_tok, int n_embd, int n_experts, float *logits);
/* RMS norm of `rows` rows of `width` f32 (ops.rs:131-139; the HIP executor's rvh_rms_norm
 * contract, runtime/hip/rvhip.h:43 and rvhip.hip:75-90, adds `post`): sum of squares in f64,
 * mean rounded to f32, scale = 1 / sqrt(mean + eps) in f32, out = x * scale (* post when
 * post != 1) (* weight[i] when weight is given), each product rounded. out may equal x. */
void rvo_rms_norm(const float *x, float *out, const float *weight, int rows, int width, float eps, float post);
/* ops.rs:249-266 (matmul_q4_0): y[t][r] = dequant(W[r]) . x[t], Q4_0 rows of k, F32 x, each
 * dot the sequential f32 sum of rounded products from -0. */
void rvo_matmul_q4_0(const uint8_t *w, int k, const float *x, int n_in, float *y, int n_out);
/* exec.rs:438-453: the shared dense MLP with its two norms (out [n_tok][n_embd]). */
void rvo_shared_mlp(const uint8_t *gate, const uint8_t *up, const uint8_t *down, const float *ffn_norm,
                    const float *post_norm, const float *x, int n_tok, int n_embd, int ff, float eps, float *out);
/* exec.rs:507-517: softmax, top `used`, renormalise with the 2^-14 clamp.
 * logits are overwritten by probabilities. */
void rvo_select_experts(float *logits, int n_tok, int n_experts, int used, int32_t *ids, float *weights);
/* expert_kernel.rs:147-161 (generic order) and :163-191 (AVX2 int8 routine). */
float rvo_dot_q8_scalar(const uint8_t *row_q4, const uint8_t *xq8, int k);
float rvo_dot_q8_avx2(const uint8_t *row_q4, const uint8_t *xq8, int k);
int rvo_have_avx2(void);
/* The exact integer sum of one Q4_0 block times one Q8_0 block
 * (expert_kernel.rs:152-157). */
int32_t rvo_block_sumi(const uint8_t *blk_q4, const uint8_t *blk_q8);

/* exec.rs:541-557: stable order of pairs by (expert, pair); pos_of[pair];
 * counts[e] pairs per expert. */
void rvo_moe_plan(const int32_t *ids, int n_pairs, int n_experts, int32_t *order, int32_t *pos_of, int32_t *counts);

/* Persistent expert worker pool (expert_pool.rs:179-447): parked workers,
 * 16-row atomic chunks, caller-side Q8_0 quantisation. */
typedef struct rvo_pool rvo_pool;
rvo_pool *rvo_pool_new(int threads, int kernel);
void rvo_pool_free(rvo_pool *p);
int rvo_pool_threads(const rvo_pool *p);

/* exec.rs:572-640 with Activation::Q8_0 (expert_pool.rs:282-355): routed
 * experts for n_tok tokens given ids/weights, out[t][n_embd] f32 before
 * post_ffw_norm_2. x_expert is f32 or bf16 [n_tok][n_embd]. down_scale may be
 * NULL (all 1.0). Optional debug outputs (may be NULL): h[pos][ff] f32 and
 * y[pos][n_embd] f32 in plan order. Returns 0 or -1 on bad shapes. */
int rvo_experts_q8(rvo_pool *pool, const void *x_expert, int x_dtype, const uint8_t *gate_up, const uint8_t *down,
                   const float *down_scale, const int32_t *ids, const float *weights, int n_tok, int n_embd, int ff,
                   int n_experts, int used, float *out, float *h_dbg, float *y_dbg);

/* The whole MoE layer: router logits, selection and routed experts, as the
 * reference's CPU executor layer (exec.rs:456-475) computes it for a given
 * router input and expert input. logits_out, ids_out, w_out may be NULL. */
int rvo_moe_layer(rvo_pool *pool, const void *x_router, const void *x_expert, int x_dtype, const void *w_router,
                  int w_dtype, const float *bias, int bias_stride, const uint8_t *gate_up, const uint8_t *down,
                  const float *down_scale, int n_tok, int n_embd, int ff, int n_experts, int used, float *logits_out,
                  int32_t *ids_out, float *w_out, float *out);

#ifdef __cplusplus
}
#endif
