/*
 * fence_oracle.h — CPU restatement of the reference's batch-1 token loop, used ONLY as the checker
 * by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg. Nothing in the product
 * library links or calls it.
 *
 * Every function names the reference code it restates. Arithmetic is done in double and rounded
 * to float at the points where the reference stores fp32 activations, and to fp16 where the
 * reference converts (f32_to_f16 before each Q6_K GEMV; the KV cache). Transcendentals are the
 * exact library functions (the reference's device build uses --use_fast_math approximations).
 *
 * Pinning: the Q6_K path is checked against the reference's own fp64 host oracle
 * (tests/test_gemv_q6k.cu:78-128, compiled from the reference sources into oracle/_ref) and its
 * golden blocks (tests/test_q6k_dot.cu:242-332); the rest against fixtures produced by the
 * reference's CUDA forward (tests/golden/).
 */
#ifndef FENCE_ORACLE_H
#define FENCE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float oracle_h2f(uint16_t h);
uint16_t oracle_f2h(float f);     /* round to nearest even */
float oracle_bf2f(uint16_t h);
uint16_t oracle_f2bf(float f);    /* round to nearest even */

/* one Q6_K super-block (210 B) dequantised: w[i] = d * scales[i/16] * (q6[i] - 32) */
void oracle_q6k_dequant(const uint8_t* blk, double* w256);
/* cpu_q6k_dot_block, tests/test_gemv_q6k.cu:78-114 */
double oracle_q6k_dot_block(const uint8_t* blk, const uint16_t* x_f16);
/* cpu_gemv_q6k, tests/test_gemv_q6k.cu:117-128 (threaded over rows) */
void oracle_gemv_q6k(const uint8_t* W, const uint16_t* x_f16, double* y, int M, int K, int nthreads);
/* gemv_q8_0 semantics, src/kernels/gemv_q8_0.cuh:40-97: y = sum_b d_b * sum_i qs_i x_i, fp32 x */
void oracle_gemv_q8_0(const uint8_t* W, const float* x, double* y, int M, int K, int nthreads);
/* embed_q8_0, src/kernels/gemv_q8_0.cuh:12-29 */
void oracle_embed_q8_0(float* out, const uint8_t* W, int token, int dim);
/* rms_norm, src/kernels/ops.cuh:17-45 (out may alias x) */
void oracle_rms_norm(float* out, const float* x, const float* w, int n, float eps);
/* rms_norm_per_head, src/kernels/ops.cuh:66-95 */
void oracle_rms_norm_per_head(float* x, const float* w, int n_heads, int hd, float eps);
/* apply_rope (NeoX pairs), src/kernels/ops.cuh:115-167 */
void oracle_rope(float* q, float* k, int hd, int nq, int nkv, int pos, float base);
/* silu_elementwise_mul, src/kernels/ops.cuh:183-195 */
void oracle_silu_mul(float* out, const float* g, const float* u, int n);
/* softmax, src/kernels/ops.cuh:207-246 */
void oracle_softmax(float* x, int n);
/* gqa_attention, src/kernels/ops.cuh:320-403; cache elements fp16 (kv_bf16 = 0) or bf16 */
void oracle_attention(float* out, const float* q, const uint16_t* kc, const uint16_t* vc, int kv_bf16,
                      long stride_t, long stride_h, int hd, int nq, int nkv, int seq_len);
/* argmax, src/kernels/ops.cuh:467-499: strided scan + tree, ties to the smaller index mod 256 */
int oracle_argmax(const float* x, int n);

/* Qwen3Model::sample_nucleus, src/model/qwen3.cu:351-460, in the reference's float arithmetic
 * (sequential sums, penalty once per history occurrence, min-p, entropy-scaled temperature,
 * descending sort with ties to the smaller index, top-k then top-p) with the random draw made
 * explicit: u in [0, 1) plays the part of the one generate_canonical<double> draw that
 * std::discrete_distribution makes, and the id is the first kept entry whose cumulative
 * normalised weight (double) is >= u (the last one if none). Returns the token id; *cut_margin
 * (if not NULL) receives the distance of the top-p cumulative from top_p at the cut and *u_margin
 * the distance of u from the nearest cumulative boundary, so a test can skip draws that rounding
 * could move. */
int oracle_sample_nucleus(const float* logits, int vocab, const int* history, int n_history, float temperature,
                          float top_p, int top_k, float rep_penalty, float min_p, int dynamic_temp, double u,
                          double* cut_margin, double* u_margin);

/* ---- full model (src/model/qwen3.cu:116-341) ---- */
typedef struct oracle_model oracle_model;
/* kv_bf16: 0 = fp16 cache (reference), 1 = bf16 (engine option). */
oracle_model* oracle_model_open(const char* path, int max_ctx, int kv_bf16, int nthreads);
void oracle_model_close(oracle_model* m);
/* dims[0..9] = layers, embed, ff, heads, kv_heads, head_dim, vocab, max_ctx, linear_type, qk_norm */
void oracle_model_dims(const oracle_model* m, int* dims);
int oracle_model_fill_kv(oracle_model* m, int n_pos, uint64_t seed);
/* Qwen3Model::forward (qwen3.cu:241-265): logits[vocab] for `token` at `pos`. 0 = ok. */
int oracle_forward(oracle_model* m, int token, int pos, float* logits);
/* Sparse MoE models (ffn_gate_inp + ffn_*_exps tensors, {arch}.expert_count / expert_used_count):
 * the forward replaces the dense FFN by the routed experts (see moe_ffn in the source; no reference
 * counterpart, parity unpinned). oracle_model_moe gives (n_exp, n_used), 0 for dense models;
 * oracle_last_route copies the experts chosen per layer at the last forward ([L][n_used]) and
 * returns the smallest router-logit gap between the last chosen expert and the best unchosen one
 * (a tie there lets rounding pick either expert). */
void oracle_model_moe(const oracle_model* m, int* n_exp, int* n_used);
float oracle_last_route(const oracle_model* m, int* sel);
/* Hidden state after the final norm of the last forward (embed_dim floats). */
void oracle_last_hidden(const oracle_model* m, float* out);
/* Test hook: the sparse-MoE FFN of layer l on a given normed input (out[H] before the residual add,
 * sel[n_used] the chosen experts); 0 on success. */
int oracle_moe_ffn_apply(oracle_model* m, int l, const float* normed, float* out, int* sel);

#ifdef __cplusplus
}
#endif
#endif
