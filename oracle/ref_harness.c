/*
 * Harness translation unit for oracle/_ref -- TEST INFRASTRUCTURE ONLY.
 *
 * Built by oracle/Makefile.ref from the reference sources where they lie
 * (the include below resolves through -I<reference>/native); nothing of the
 * reference is copied into this repository.  Including the N2 provider gives
 * this unit access to its file-static numerical runners, which the provider's
 * own capability rows would otherwise refuse at realistic shapes
 * (n2_primitives_provider.c:887-895).  Each wrapper forwards to the runner
 * unchanged.
 */
#include "n2_primitives_provider.c"

int ref_n2_linear_forward(size_t n, size_t t, size_t din, size_t dout,
                          const float *x, const float *w, const float *bias,
                          float *y) {
  const shape4 s = {n, t, din, dout};
  return linear_forward_run(&s, x, w, bias, y);
}

int ref_n2_linear_backward(size_t n, size_t t, size_t din, size_t dout,
                           const float *x, const float *w, const float *dy,
                           int include_dbias, float *dx, float *dw,
                           float *dbias) {
  const shape4 s = {n, t, din, dout};
  return linear_backward_run(&s, x, w, dy, include_dbias, dx, dw, dbias);
}

int ref_n2_layer_norm_forward(size_t n, size_t t, size_t d, const float *x,
                              const float *gamma, const float *beta,
                              float epsilon, float *y) {
  const shape3 s = {n, t, d};
  return layer_norm_forward_run(&s, x, gamma, beta, epsilon, y);
}

int ref_n2_layer_norm_backward(size_t n, size_t t, size_t d, const float *x,
                               const float *gamma, float epsilon,
                               const float *dy, float *dx, float *dgamma,
                               float *dbeta) {
  const shape3 s = {n, t, d};
  return layer_norm_backward_run(&s, x, gamma, epsilon, dy, dx, dgamma, dbeta);
}

int ref_n2_gelu(size_t n, size_t t, size_t d, const float *x,
                const float *upstream, float *out) {
  const shape3 s = {n, t, d};
  return activation_run(&s, x, upstream, 1, out);
}

int ref_n2_embedding_forward(size_t n, size_t t, size_t v, size_t d,
                             const int64_t *ids, const float *w, float *y) {
  const shape4 s = {n, t, v, d};
  return embedding_forward_run(&s, ids, w, y);
}

int ref_n2_embedding_backward(size_t n, size_t t, size_t v, size_t d,
                              const int64_t *ids, const float *dy, float *dw) {
  const shape4 s = {n, t, v, d};
  return embedding_backward_run(&s, ids, dy, dw);
}
