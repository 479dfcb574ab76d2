/*
 * CPU oracle for the f32 training-step hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C11 compiled with -ffp-contract=off, the
 * arithmetic of eshkol-transformer's serial CPU providers on the training
 * step: A2 attention + RoPE, N2 linear / LayerNorm / GELU / residual /
 * embedding, L2 indexed cross-entropy, L3S mean reduction and O2 AdamW.
 * Every function keeps the reference's summation order and rounding points,
 * so its outputs are bit-identical to the reference providers (checked
 * against oracle/_ref, the reference sources compiled unmodified, and against
 * the reference's golden fixtures under tests/golden).
 *
 * Only tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py
 * may load this library.  The product path (libet_b200.so) never calls it.
 */
#ifndef ESHKOL_B200_ORACLE_H
#define ESHKOL_B200_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs (identical definition in the product host) */
uint64_t orc_splitmix64(uint64_t x);
void orc_fill_normal(uint64_t seed, uint64_t stream, size_t count, double mean,
                     double stddev, float *out);
void orc_fill_tokens(uint64_t seed, uint64_t stream, size_t count,
                     uint64_t vocabulary, int64_t *out);

/* ---- A2 attention [N,Hq,Hkv,Tq,Tk,Dh] (a2_attention_provider.c:669-790) */
void orc_attention_forward(const int64_t shape[6], const float *q,
                           const float *k, const float *v,
                           const int64_t *query_positions,
                           const int64_t *key_positions, const uint8_t *mask,
                           float *output);
void orc_attention_backward(const int64_t shape[6], const float *q,
                            const float *k, const float *v,
                            const int64_t *query_positions,
                            const int64_t *key_positions, const uint8_t *mask,
                            const float *upstream, float *dq, float *dk,
                            float *dv);
/* ---- A2 RoPE [N,H,T,Dh] (a2_attention_provider.c:792-935) */
void orc_rope(const int64_t shape[4], const float *x, const int64_t *positions,
              const float *inv_freq, int backward, float *y);

/* ---- N2 primitives (n2_primitives_provider.c:313-622) */
void orc_linear_forward(size_t rows, size_t din, size_t dout, const float *x,
                        const float *w, const float *bias, float *y);
void orc_linear_backward(size_t rows, size_t din, size_t dout, const float *x,
                         const float *w, const float *dy, float *dx, float *dw,
                         float *dbias);
void orc_layer_norm_forward(size_t rows, size_t d, const float *x,
                            const float *gamma, const float *beta,
                            float epsilon, float *y);
void orc_layer_norm_backward(size_t rows, size_t d, const float *x,
                             const float *gamma, float epsilon,
                             const float *dy, float *dx, float *dgamma,
                             float *dbeta);
void orc_gelu_forward(size_t count, const float *x, float *y);
void orc_gelu_backward(size_t count, const float *x, const float *dy,
                       float *dx);
void orc_embedding_forward(size_t rows, size_t vocabulary, size_t d,
                           const int64_t *ids, const float *w, float *y);
void orc_embedding_backward(size_t rows, size_t vocabulary, size_t d,
                            const int64_t *ids, const float *dy, float *dw);

/* ---- L2 indexed cross-entropy (indexed_cross_entropy.c:109-280) */
void orc_ce_forward(size_t rows, size_t vocabulary, const float *logits,
                    const int64_t *targets, float *loss);
void orc_ce_backward(size_t rows, size_t vocabulary, const float *logits,
                     const int64_t *targets, const float *upstream,
                     float *grad);
/* L3S masked mean with an all-ones mask: sequential numerator / weight. */
float orc_mean_loss(size_t rows, const float *loss);

/* ---- O2 AdamW (o2_optimizer.c:381-435, 1548-1618, 1626-1781) */
typedef struct orc_adamw_options {
  uint32_t learning_rate_bits;
  uint32_t beta1_bits;
  uint32_t beta2_bits;
  uint32_t epsilon_bits;
  uint32_t weight_decay_bits;
} orc_adamw_options;
uint32_t orc_pow_bits(uint32_t base_bits, uint64_t exponent);
/* Returns 0 on success, 1 when any staged value would be nonfinite (the
 * caller's tensors are then unchanged, as with the reference's staging). */
int orc_adamw_step(size_t count, float *parameter, const float *gradient,
                   float *exp_avg, float *exp_avg_sq,
                   const orc_adamw_options *options, uint64_t update,
                   uint32_t weight_bits, uint32_t schedule_factor_bits,
                   uint32_t clip_factor_bits);
/* Scaled sum-of-squares norm of gradient/weight over tensors in order. */
uint32_t orc_global_norm(size_t tensor_count, const float *const *gradients,
                         const size_t *counts, uint32_t weight_bits);
/* Linear warmup/decay schedule factor with exact rational rounding. */
uint32_t orc_schedule_factor(uint32_t kind, uint64_t warmup, uint64_t total,
                             uint32_t minimum_ratio_bits, uint64_t update);

/* ---- decoder-only LM composed from the primitives above */
typedef struct orc_lm_config {
  int64_t layers, d_model, heads, ffn, vocabulary, seq_len, batch;
  float ln_epsilon;
  double rope_base;
} orc_lm_config;
size_t orc_lm_tensor_count(const orc_lm_config *c);
/* Fills sizes[i] (elements) of every parameter tensor; returns the total. */
size_t orc_lm_tensor_sizes(const orc_lm_config *c, size_t *sizes);
void orc_lm_init(const orc_lm_config *c, uint64_t seed, float *params);
void orc_rope_inv_freq(int64_t head_dim, double base, float *inv_freq);
/* One forward + backward over ids/targets [batch, seq_len]; gradients are
 * the CE upstream 1/N times the reference's numerators (N = batch*seq_len
 * of this call unless token_scale > 0 overrides N). Returns the mean loss. */
float orc_lm_forward_backward(const orc_lm_config *c, const float *params,
                              const int64_t *ids, const int64_t *targets,
                              double token_scale, float *grads);
float orc_lm_forward_backward_masked(const orc_lm_config *c, const float *params,
                                     const int64_t *ids, const int64_t *targets,
                                     const uint8_t *loss_mask, float upstream_scale,
                                     float *grads);
float orc_masked_mean_loss(size_t rows, const float *loss, const uint8_t *mask);
/* One AdamW update over all tensors in parameter order. */
int orc_lm_adamw(const orc_lm_config *c, float *params, const float *grads,
                 float *exp_avg, float *exp_avg_sq,
                 const orc_adamw_options *options, uint64_t update);

#ifdef __cplusplus
}
#endif
#endif
