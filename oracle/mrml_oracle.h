/*
 * mrml_oracle.h — CPU restatement of the MRML mixture-of-experts FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels in libmrml_moe_b200.so and the timed CPU baseline of bench.py.
 * Nothing in the shipped product links, loads or calls it.
 *
 * Every function restates the arithmetic of the reference Rust CPU path of
 * mitchellrenouf/QT_llama.cpp (crate mrml-tensor), operation for operation,
 * in the same evaluation order and with the same glibc libm calls
 * (expf, tanhf, roundf, sqrtf — the functions crates/mrml-math/src/lib.rs:3-22
 * links).  Compile without fast-math and with -ffp-contract=off so that no
 * multiply-add is fused: the Rust code never contracts.
 *
 * Parity pinning: the reference cannot be compiled in this container (it is a
 * nightly-Rust workspace and no Rust toolchain is installed), so the oracle is
 * pinned against the reference's own known-answer tests, restated in
 * tests/test_oracle.py from crates/mrml-tensor/tests/quant_test.rs,
 * tests/ops_test.rs and src/cuda.rs (router test).  Those tests are
 * tolerance-based; no binary golden vector ships with the reference.
 */
#ifndef MRML_ORACLE_H
#define MRML_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, crates/mrml-tensor/src/types.rs:7-27. */
enum { ORACLE_Q4_0 = 2, ORACLE_Q8_0 = 8 };

/* quant.rs:47-77 (subnormals expanded, Inf/NaN kept). */
float oracle_f16_to_f32(uint16_t h);
/* quant.rs:81-104 (mantissa truncated, exponent underflow flushed to +0). */
uint16_t oracle_f32_to_f16(float f);

/* quant.rs:193-228.  n must be a multiple of 32; dst holds n/32 * 34 bytes. */
void oracle_quantize_q8_0(const float *src, size_t n, uint8_t *dst);
/* quant.rs:372-389.  n must be a multiple of 32; dst holds n/32 * 18 bytes. */
void oracle_quantize_q4_0(const float *src, size_t n, uint8_t *dst);
/* quant.rs:135-190. */
void oracle_dequantize_q4_0(const uint8_t *src, size_t n_blocks, float *out);
void oracle_dequantize_q8_0(const uint8_t *src, size_t n_blocks, float *out);

/* quant.rs:335-369 (scalar; the AVX2 and AVX-VNNI paths at 272-332 and
 * 443-479 give the same bits: exact integer block sums, then the same f32
 * update sum += (float)isum * (d_w * d_a) in block order). */
float oracle_vec_dot_q4_0_q8_0(const uint8_t *w, const uint8_t *a, int n);
/* quant.rs:564-577 (scalar; identical bits to the VNNI path 499-530). */
float oracle_vec_dot_q8_0_q8_0(const uint8_t *w, const uint8_t *a, int n);

/* ops.rs:221-260 (rows of `wtype` blocks against a Q8_0 vector). */
void oracle_mat_vec_q8(int wtype, const uint8_t *w, const uint8_t *x_q8,
                       float *y, int n_rows, int n_cols);
/* ops.rs:162-180: quantise x to Q8_0 first, then as above. */
void oracle_mat_vec_f32(int wtype, const uint8_t *w, const float *x, float *y,
                        int n_rows, int n_cols);

/* ops.rs:99-114. */
float oracle_gelu_approx(float x);
void oracle_geglu(const float *gate, const float *up, float *out, int n);
/* ops.rs:24-49 (weight may be NULL). */
void oracle_rms_norm(const float *x, const float *weight, float eps, float *out,
                     int n);

/* FFN prologue of a MoE layer, model.rs:1719-1784 for T rows of H:
 * attn_res = hidden + rms_norm(attn, post_attn_norm) (attn NULL: hidden),
 * x_shared = rms_norm(attn_res, ffn_norm), x_moe = rms_norm(attn_res,
 * pre_ffw_norm_2), router_x[i] = rms_norm(attn_res, none)[i] * (1 / sqrtf(H))
 * * router_scale[i].  A NULL output is skipped; a NULL weight means 1. */
void oracle_ffn_prologue(const float *hidden, const float *attn, const float *post_attn_norm,
                         const float *ffn_norm, const float *pre_ffw_norm_2, const float *router_scale,
                         float *attn_res, float *x_shared, float *x_moe, float *router_x, int H, int T, float eps);

/* FFN epilogue, model.rs:2176-2196 for T rows of H:
 * hidden = (attn_res + rms_norm(rms_norm(mlp_raw, post_ffw_norm_1)
 *          + rms_norm(moe_raw, post_ffw_norm_2), post_ffw_norm)) * out_scale.
 * mlp_raw NULL reads as zeros; hidden may alias attn_res. */
void oracle_ffn_epilogue(const float *attn_res, const float *mlp_raw, const float *moe_raw,
                         const float *post_ffw_norm_1, const float *post_ffw_norm_2, const float *post_ffw_norm,
                         float out_scale, float *hidden, int H, int T, float eps);

/* Router, model.rs:1804-1829 generalised from (E=128, K=8) to (E, K):
 * logits[t,e] = sequential f32 sum of x[t,i]*W[e,i] (mul then add, i
 * ascending); experts sorted by logit descending, ties to the lower expert id;
 * p_k = expf(l_k - l_0) summed in k order; probs[t,k] = p_k / max(sum, 1e-6). */
void oracle_moe_router(const float *W, const float *x, float *logits,
                       int32_t *ids, float *probs, int H, int E, int K, int T);

/* Top-k and softmax only (model.rs:1816-1829), for callers that supply
 * logits directly. */
void oracle_moe_route_from_logits(const float *logits, int32_t *ids,
                                  float *probs, int E, int K, int T);

/* Experts and combine, model.rs:2111-2165 generalised to (H, I, E, K, T) and
 * to Q8_0 expert weights.  Per token: x -> Q8_0; for k ascending, skip
 * alpha <= 1e-4; gate = rows [0, I), up = rows [I, 2I) of expert e's
 * gate_up slab; act = geglu(gate, up); down = W_down[e] . Q8_0(act);
 * out[i] += alpha * down[i] * scale[e] (scale 1 when down_scale is NULL).
 * gate_up is [E][2I][H/32] blocks, down is [E][H][I/32] blocks.
 * n_threads > 1 runs each GEMV row-parallel like parallel.rs:73-116 with
 * a minimum chunk of 64 rows (ops.rs:236-259); results do not depend on it. */
void oracle_moe_experts(int wtype, const uint8_t *gate_up, const uint8_t *down,
                        const int32_t *ids, const float *probs,
                        const float *down_scale, const float *x, float *out,
                        int H, int I, int E, int K, int T, int n_threads);

/* Intermediate values of one (token, slot) for debugging parity:
 * gate[I], up[I], act[I], down[H] (unscaled). */
void oracle_moe_expert_trace(int wtype, const uint8_t *gate_up,
                             const uint8_t *down, int expert, const float *x,
                             int H, int I, float *gate, float *up, float *act,
                             float *down_out);

#ifdef __cplusplus
}
#endif
#endif
