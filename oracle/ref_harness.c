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

/*
 * O2 through its own public API (o2_optimizer_internal.h:137-160) over one I2
 * parameter, the way the reference's tests/o2 drive it: create the
 * parameter from host bits, accumulate a weighted gradient through an I2
 * gradient plan, step, zero the gradient.  O2 has no public destroy outside
 * its private retire path, so the harness builds one optimizer per process.
 */
#include "o2_optimizer_internal.h"

static et_f32_parameter *ref_o2_parameter;
static et_o2_optimizer *ref_o2_optimizer;
static int ref_o2_identity;
static size_t ref_o2_count;

int ref_o2_create(const uint32_t *initial_bits, size_t count, uint32_t lr, uint32_t beta1,
                  uint32_t beta2, uint32_t epsilon, uint32_t weight_decay) {
  uint64_t shape[1] = {(uint64_t)count};
  et_f32_tensor *initial = NULL;
  et_f32_tensor_error te;
  et_o2_error_v1 oe;
  et_o2_optimizer_builder *builder = NULL;
  if (ref_o2_optimizer != NULL) return 3;
  memset(&te, 0, sizeof(te));
  memset(&oe, 0, sizeof(oe));
  if (et_f32_tensor_create_v1(1u, shape, &initial, &te) != 0 ||
      et_f32_tensor_copy_bits_from_v1(initial, initial_bits, count, &te) != 0 ||
      et_f32_parameter_create_v1(initial, &ref_o2_parameter, &te) != 0 ||
      et_f32_parameter_bind_identity_v1(ref_o2_parameter, &ref_o2_identity, &te) != 0)
    return 1;
  (void)et_f32_tensor_destroy_v1(&initial, &te);
  if (et_o2_optimizer_builder_create_v1(1u, ET_O2_CLIP_NONE, 0u, ET_O2_SCHEDULE_CONSTANT, 0u, 0u,
                                        UINT32_C(0x3f800000), &builder, &oe) != 0 ||
      et_o2_optimizer_builder_set_v1(builder, 0u, ref_o2_parameter, &ref_o2_identity, lr, beta1,
                                     beta2, epsilon, weight_decay, &oe) != 0 ||
      et_o2_optimizer_builder_finish_v1(&builder, &ref_o2_optimizer, &oe) != 0)
    return 2;
  ref_o2_count = count;
  return 0;
}

/* The gradient contribution (weighted numerator) through an I2 plan. */
int ref_o2_accumulate(const uint32_t *gradient_bits, uint32_t weight_bits) {
  uint64_t shape[1] = {(uint64_t)ref_o2_count};
  et_f32_tensor *source = NULL;
  et_f32_gradient_plan *plan = NULL;
  et_f32_gradient_contribution_v1 contribution;
  et_f32_tensor_error te;
  memset(&te, 0, sizeof(te));
  if (et_f32_tensor_create_v1(1u, shape, &source, &te) != 0 ||
      et_f32_tensor_copy_bits_from_v1(source, gradient_bits, ref_o2_count, &te) != 0)
    return 1;
  contribution.struct_size = sizeof(contribution);
  contribution.destination = ref_o2_parameter;
  contribution.weighted_numerator = source;
  contribution.expected_ordinal = 0u;
  int rc = 0;
  if (et_f32_gradient_plan_prepare_v1(1u, &contribution, weight_bits, &plan, &te) != 0 ||
      et_f32_gradient_plan_commit_v1(plan, &te) != 0)
    rc = 2;
  if (plan != NULL) (void)et_f32_gradient_plan_release_v1(&plan, &te);
  (void)et_f32_tensor_destroy_v1(&source, &te);
  return rc;
}

int ref_o2_step(void) {
  et_o2_error_v1 oe;
  memset(&oe, 0, sizeof(oe));
  return et_o2_optimizer_step_v1(ref_o2_optimizer, &oe);
}

int ref_o2_zero_grad(void) {
  et_o2_error_v1 oe;
  memset(&oe, 0, sizeof(oe));
  return et_o2_optimizer_zero_grad_v1(ref_o2_optimizer, &oe);
}

/* The parameter's current value bits (count elements). */
int ref_o2_value(uint32_t *bits) {
  et_f32_tensor *snapshot = NULL;
  et_f32_tensor_error te;
  memset(&te, 0, sizeof(te));
  if (et_f32_parameter_value_snapshot_v1(ref_o2_parameter, &snapshot, &te) != 0) return 1;
  int rc = et_f32_tensor_copy_bits_to_v1(snapshot, bits, ref_o2_count, &te) != 0;
  (void)et_f32_tensor_destroy_v1(&snapshot, &te);
  return rc;
}
