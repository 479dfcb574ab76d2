/*
 * The O2 optimizer's Eshkol binding surface over libet_b200's device AdamW.
 *
 * native/o2_wave2_extension.esk:4-29 binds the reference's optimizer through
 * these et_o2_private_*_v1 externs (native/o2_wave2_package_bridge.c:72-200),
 * with I2 parameters (native/f32_parameter_internal.h) as the `parameter`
 * handles.  The same names and signatures here run the update on the GPU; the
 * `parameter` handles are et_b200_parameter objects: a device value and
 * gradient (f32, `count` elements) plus the accumulation metadata I2 keeps
 * (gradient present, contribution count, normalisation weight).  A host that
 * links this library instead of the reference's O2 bridge binds the extension
 * unchanged.  i64 results are O2 status codes (o2_optimizer_internal.h:19-30:
 * 0 ok, 1 invalid argument, 2 shape mismatch, 7 invalid state, 9 internal);
 * handle results are NULL on failure; et_o2_private_last_error_category_v1
 * returns the last failure's category on the calling thread (0 after a
 * success).
 */
#ifndef ESHKOL_B200_O2_BRIDGE_H
#define ESHKOL_B200_O2_BRIDGE_H

#include <stddef.h>
#include <stdint.h>

#include "eshkol_b200/kernel_abi_v1.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device parameters (the I2 parameter's role,
 * native/f32_parameter_internal.h:55-67) */
typedef struct et_b200_parameter et_b200_parameter;
/* value / gradient: device f32 [count] the caller owns for the parameter's
 * lifetime. */
int32_t et_b200_parameter_create_v1(float *value, float *gradient, size_t count,
                                    et_b200_parameter **parameter,
                                    et_kernel_error *error);
/* Marks the gradient present: the gradient buffer holds the sum of the
 * weighted numerators of `contributions` contributions with normalisation
 * weight `normalization_weight_bits` (f32 bits), the state an I2 gradient plan
 * commit leaves (native/f32_tensor.c:3089-3339); with data-parallel training,
 * the all-reduced sum. */
int32_t et_b200_parameter_set_gradient_v1(et_b200_parameter *parameter,
                                          uint64_t contributions,
                                          uint32_t normalization_weight_bits,
                                          et_kernel_error *error);
int32_t et_b200_parameter_gradient_present_v1(const et_b200_parameter *parameter);
void et_b200_parameter_destroy_v1(et_b200_parameter **parameter);

/* ---- the extension's externs (o2_wave2_extension.esk:4-29) */
/* replaces et_o2_private_last_error_category_v1 */
int64_t et_o2_private_last_error_category_v1(void);
/* replaces et_o2_private_builder_create_v1 (o2_wave2_package_bridge.c:72) */
void *et_o2_private_builder_create_v1(int64_t count, int64_t clip_kind,
                                      int64_t clip_bits, int64_t schedule_kind,
                                      int64_t warmup, int64_t total,
                                      int64_t minimum_ratio_bits);
/* replaces et_o2_private_builder_set_v1 (o2_wave2_package_bridge.c:92);
 * `parameter` is an et_b200_parameter, p1_handle the caller's identity token */
int64_t et_o2_private_builder_set_v1(void *builder, int64_t index,
                                     void *parameter, void *p1_handle,
                                     int64_t learning_rate_bits,
                                     int64_t beta1_bits, int64_t beta2_bits,
                                     int64_t epsilon_bits,
                                     int64_t weight_decay_bits);
/* replaces et_o2_private_builder_finish_v1 (consumes the builder) */
void *et_o2_private_builder_finish_v1(void *builder);
/* replaces et_o2_private_builder_abort_v1 */
int64_t et_o2_private_builder_abort_v1(void *builder);
/* replaces et_o2_private_optimizer_step_v1: every gradient present with one
 * contribution count and weight, then the all-or-nothing device update */
int64_t et_o2_private_optimizer_step_v1(void *optimizer);
/* replaces et_o2_private_optimizer_zero_grad_v1: zeroes every gradient buffer
 * and marks it absent */
int64_t et_o2_private_optimizer_zero_grad_v1(void *optimizer);
/* replaces et_o2_private_optimizer_require_absent_gradients_v1 */
int64_t et_o2_private_optimizer_require_absent_gradients_v1(void *optimizer);
/* replaces et_o2_private_optimizer_completed_updates_v1 (-1 on failure) */
int64_t et_o2_private_optimizer_completed_updates_v1(void *optimizer);
/* replaces et_o2_private_optimizer_schedule_factor_bits_v1: the factor of
 * the next update (-1 on failure) */
int64_t et_o2_private_optimizer_schedule_factor_bits_v1(void *optimizer);
/* replaces et_o2_private_optimizer_state_snapshot_v1 (o2_optimizer.c:2052):
 * configuration, completed updates, options and moment bits in host memory;
 * gradients must be absent */
void *et_o2_private_optimizer_state_snapshot_v1(void *optimizer);
/* replaces et_o2_private_optimizer_load_state_v1 (o2_optimizer.c:2173): the
 * state must match the optimizer's configuration, parameter counts and
 * options; all or nothing */
int64_t et_o2_private_optimizer_load_state_v1(void *optimizer, void *state);
/* replaces et_o2_private_optimizer_state_release_v1 */
int64_t et_o2_private_optimizer_state_release_v1(void *state);

/* ---- additions without a reference counterpart */
/* The last failure's message on the calling thread ("" after a success). */
const char *et_b200_o2_bridge_last_error_message_v1(void);
/* Frees a bridge optimizer and its device moments (the reference's optimizer
 * lives for the process); the parameters remain the caller's. */
void et_b200_o2_bridge_destroy_v1(void **optimizer);
/* A snapshot state written to `path` atomically, the way the reference's C1
 * writer et_checkpoint_io_atomic_write_v1 (native/checkpoint_io.c:599)
 * publishes a file: written in full to a temporary file in the same
 * directory, flushed to storage, renamed over `path`, directory flushed.
 * Format: "ETB2O2S\1", then little-endian u32 clip kind, clip bits, schedule
 * kind, minimum ratio bits, u64 warmup, total, completed updates, entry
 * count; per entry u64 element count, five u32 option bits, the exp_avg then
 * exp_avg_sq bits; finally a u64 FNV-1a hash of every preceding byte. */
int64_t et_b200_o2_state_write_v1(void *state, const char *path);
/* Reads a file written by et_b200_o2_state_write_v1 into a new state (NULL
 * on a missing, truncated or corrupted file); release it with
 * et_o2_private_optimizer_state_release_v1. */
void *et_b200_o2_state_read_v1(const char *path);

#ifdef __cplusplus
}
#endif
#endif
