/*
 * libet_b200 -- B200 (sm_100a) implementation of eshkol-transformer's f32
 * training-step hot path behind its K1 kernel ABI.
 *
 * Every entry point is plain C: pointers, sizes and the K1 v1 structs.  Each
 * declaration names the reference interface it replaces (path:line within the
 * eshkol-transformer project).  Device pointers are CUDA global memory on the
 * current device; "host" pointers are ordinary (preferably pinned) memory.
 * Functions returning int32_t return 0 on success or a K1 error category
 * (ET_KERNEL_ERROR_*) and fill the optional et_kernel_error record.
 */
#ifndef ESHKOL_B200_ET_B200_H
#define ESHKOL_B200_ET_B200_H

#include "eshkol_b200/kernel_abi_v1.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ET_B200_ABI_MAJOR 1u
#define ET_B200_ABI_MINOR 0u

/* ------------------------------------------------------------ library */

int32_t et_b200_abi_major_v1(void);
int32_t et_b200_abi_minor_v1(void);
/* Kernels this library has launched since load (all devices, all threads).
 * A caller samples it around a region to count the region's launches. */
uint64_t et_b200_launch_count_v1(void);
/* 0 when the current CUDA device is an sm_100 part this build runs on. */
int32_t et_b200_device_check_v1(et_kernel_error *error);

/* ------------------------------------------------------------ K1 providers
 *
 * Drop-in replacements for the reference's carrier-neutral providers.  They
 * accept dense zero-offset views on device "cuda" (device pointers, results
 * complete when invoke returns; the call first waits for all work already
 * enqueued on the device, so inputs produced on any stream are complete) and
 * on device "cpu" (host pointers, staged through the GPU).  Capabilities are
 * verified for every shape the kernels
 * support rather than the reference's exact tiny rows.  validate_call keeps
 * the reference's checks (finite inputs, canonical positions and masks, ids
 * in range) and its error categories; invoke_call never fails.
 */
/* replaces include/eshkol_transformer/a2_attention_abi.h:32
 * (kernel.causal-attention forward/backward, kernel.rope forward/backward) */
const et_kernel_provider_v1 *et_a2_kernel_provider_v1(void);
/* replaces include/eshkol_transformer/n2_primitives_abi.h:18
 * (kernel.matmul linear.*, kernel.norm, kernel.activation gelu/relu,
 *  kernel.residual, kernel.embedding-forward/backward) */
const et_kernel_provider_v1 *et_n2_kernel_provider_v1(void);
/* replaces include/eshkol_transformer/n3k_primitives_abi.h:12
 * (n3k.linear forward/backward-no-bias) */
const et_kernel_provider_v1 *et_n3k_kernel_provider_v1(void);
/* replaces include/eshkol_transformer/indexed_cross_entropy.h:22-29 */
int32_t et_l2_indexed_cross_entropy_abi_major_v1(void);
int32_t et_l2_indexed_cross_entropy_abi_minor_v1(void);
const et_kernel_provider_v1 *et_l2_indexed_cross_entropy_provider_v1(void);
/* Every capability above in one provider (sorted by name; each call goes to
 * the provider owning its capability), for K1 runtimes, which take exactly
 * one provider from their resolver (native/kernel_abi.c:764-840).  No
 * reference counterpart: the reference composes no providers. */
const et_kernel_provider_v1 *et_b200_kernel_provider_v1(void);
/* K2 capability facade support (native/k2_capabilities.c).  K2 discovers
 * through a fixed private resolver that answers only the K1 provider symbol
 * with its private context sentinel, and exact-audits the provider it gets,
 * identity by callback pointers (k2_capabilities.c:493-561).  These are that
 * resolver and that audit for the B200 provider: a K2 built over libet_b200
 * calls et_kernel_runtime_discover(et_b200_k2_resolver_v1,
 * (void *)et_b200_k2_resolver_context_v1(), ...) and admits the provider
 * when the audit returns ET_B200_K2_PROVIDER_EXACT (the values mirror
 * enum et_k2_provider_audit, k2_capabilities.c:565-570). */
enum {
  ET_B200_K2_PROVIDER_ABSENT = 0,
  ET_B200_K2_PROVIDER_VERSION_MISMATCH = 1,
  ET_B200_K2_PROVIDER_METADATA_MISMATCH = 2,
  ET_B200_K2_PROVIDER_EXACT = 3
};
const void *et_b200_k2_resolver_context_v1(void);
const et_kernel_provider_v1 *et_b200_k2_resolver_v1(void *context,
                                                    const char *symbol_name);
int32_t et_b200_k2_audit_provider_v1(const et_kernel_provider_v1 *provider);
/* Contraction mode (ET_B200_PRECISION_*) the kernel.matmul and n3k.linear
 * providers use; process-wide, default ET_B200_PRECISION_TF32X3.  No
 * reference counterpart: the reference's only mode is serial FP32. */
int32_t et_b200_k1_precision_v1(uint32_t precision);

/* ------------------------------------------------------------ attention on device
 * Causal attention with RoPE on device tensors, for callers that run many
 * steps without a K1 round trip per call (the A2 provider's arithmetic,
 * native/a2_attention_provider.c:669-790, with rope.forward on Q and K and
 * rope.backward on dQ and dK, :792-935).  No reference counterpart for the
 * split of the statistics: the forward returns per query row the maximum of
 * the scaled scores and the sum of their exponentials, which the backward
 * takes instead of recomputing the forward as a K1 backward call does.
 * Tensors are dense row-major f32 [batch, heads, len, head_dim] on the
 * current device; the calls enqueue on `stream` (a cudaStream_t, NULL = the
 * legacy default stream) and return without synchronising.  Inputs are not
 * validated on the device (finite values, canonical positions): the caller
 * supplies what the A2 provider's validate_call would accept. */
typedef struct et_b200_attention_v1 {
  size_t struct_size;
  int64_t batch, q_heads, kv_heads, q_len, k_len, head_dim;
  const int64_t *q_positions; /* device [batch, q_len], strictly increasing */
  const int64_t *k_positions; /* device [batch, k_len], strictly increasing */
  const uint8_t *keep;        /* device [batch, q_len, k_len] or NULL (all) */
  const float *rope_cos;      /* device [len, head_dim/2] (or [batch*len, ..]
                                 with rope_batched) for Q and K; NULL = no RoPE */
  const float *rope_sin;
  int32_t rope_batched;
  int32_t contraction; /* ET_B200_ATTENTION_* (0 = the default) */
} et_b200_attention_v1;
/* Contraction modes.  f32-grade (three products of operand pairs, about 22
 * significant bits per operand element):
 * ET_B200_ATTENTION_DEFAULT: binary16 pairs with per-tensor power-of-two
 *   scales at head_dim 128 and at head_dim 64 from q_len k_len = 768^2 up,
 *   3xTF32 pairs otherwise;
 * ET_B200_ATTENTION_BWD_PAIRS16: binary16 pairs in the backward at head_dim
 *   64 as well.
 * TF32-grade (one product of the hi parts, 11 significant bits per operand
 * element, the reference sweep's "TF32" mode):
 * ET_B200_ATTENTION_TF32: TF32 operands (round to nearest), binary16 ones
 *   with per-tensor scales (the same 11 bits) in the head_dim-128 backward. */
enum {
  ET_B200_ATTENTION_DEFAULT = 0,
  ET_B200_ATTENTION_BWD_PAIRS16 = 1,
  ET_B200_ATTENTION_TF32 = 2
};
/* Bytes of the workspace both calls take (256-byte aligned). */
size_t et_b200_attention_workspace_bytes_v1(const et_b200_attention_v1 *shape);
/* Host-side RoPE tables [len, head_dim/2] the way the reference builds its
 * rotation: inv_freq = (float)(1 / base^(2i/head_dim)), angle = (float)t *
 * inv_freq, cosf / sinf (a2_attention_provider.c:792-935 with the base-10000
 * frequencies the callers pass). */
void et_b200_rope_tables_v1(int64_t len, int64_t head_dim, double base,
                            float *cos_out, float *sin_out);
int32_t et_b200_attention_forward_v1(const et_b200_attention_v1 *shape,
                                     const float *q, const float *k,
                                     const float *v, float *o, float *row_max,
                                     float *row_sum, void *workspace,
                                     size_t workspace_bytes, void *stream,
                                     et_kernel_error *error);
/* workspace_from_forward: the workspace still holds what the forward of the
 * same Q/K/V wrote into it (the prepared operands are then reused). */
int32_t et_b200_attention_backward_v1(
    const et_b200_attention_v1 *shape, const float *q, const float *k,
    const float *v, const float *o, const float *dout, const float *row_max,
    const float *row_sum, float *dq, float *dk, float *dv, void *workspace,
    size_t workspace_bytes, int32_t workspace_from_forward, void *stream,
    et_kernel_error *error);

/* ------------------------------------------------------------ synthetic data
 * Seeded inputs shared with the tests: value i of (seed, stream) is a pure
 * function of (seed, stream, i).  Host-only; no device is needed. */
void et_b200_fill_normal_v1(uint64_t seed, uint64_t stream, size_t count,
                            double mean, double stddev, float *out);
void et_b200_fill_tokens_v1(uint64_t seed, uint64_t stream, size_t count,
                            uint64_t vocabulary, int64_t *out);

/* ------------------------------------------------------------ O2 AdamW
 * Device counterpart of the O2 optimizer (native/o2_optimizer_internal.h:
 * 137-160 builder/step API; element maths o2_optimizer.c:1738-1756).  The
 * optimizer owns zero-initialised device moments; parameters and gradients are
 * caller-owned device tensors.  Each step divides gradients by the
 * normalisation weight, applies the global-L2 clip factor and the schedule
 * factor, and updates all tensors in one fused multi-tensor pass whose
 * per-element arithmetic is bit-identical to the reference. */
enum { ET_B200_O2_CLIP_NONE = 0, ET_B200_O2_CLIP_GLOBAL_L2 = 1 };
enum { ET_B200_O2_SCHEDULE_CONSTANT = 0, ET_B200_O2_SCHEDULE_LINEAR = 1 };

typedef struct et_b200_o2_parameter_v1 {
  size_t struct_size;
  float *value;    /* device, count f32 */
  float *gradient; /* device, count f32 (weighted numerators) */
  size_t count;
  uint32_t learning_rate_bits;
  uint32_t beta1_bits;
  uint32_t beta2_bits;
  uint32_t epsilon_bits;
  uint32_t weight_decay_bits;
  uint32_t reserved;
} et_b200_o2_parameter_v1;

typedef struct et_b200_o2_optimizer et_b200_o2_optimizer;

/* replaces et_o2_optimizer_builder_create_v1/_set_v1/_finish_v1
 * (native/o2_optimizer_internal.h:137-150) */
int32_t et_b200_o2_optimizer_create_v1(
    size_t parameter_count, const et_b200_o2_parameter_v1 *parameters,
    uint32_t clip_kind, uint32_t clip_max_bits, uint32_t schedule_kind,
    uint64_t warmup_updates, uint64_t total_updates,
    uint32_t minimum_ratio_bits, et_b200_o2_optimizer **optimizer,
    et_kernel_error *error);
/* replaces et_o2_optimizer_step_v1 (native/o2_optimizer.c:1784-1944).
 * normalization_weight_bits is the f32 bit pattern of the accumulated
 * contribution weight.  norm_bits (optional) receives the global norm.  All
 * or nothing like the reference's staged commit: a nonfinite gradient,
 * parameter or moment, or an update that would be nonfinite, leaves every
 * tensor and the update counter unchanged and returns INVALID_ARGUMENT.  The
 * global norm is an f64 sum of squares rounded once to f32; the reference's
 * is a scaled f32 recurrence in parameter order (o2_optimizer.c:1548-1618),
 * so the two norms (and with clipping active, the clipped updates) can differ
 * in the last bits. */
int32_t et_b200_o2_optimizer_step_v1(et_b200_o2_optimizer *optimizer,
                                     uint32_t normalization_weight_bits,
                                     uint32_t *norm_bits,
                                     et_kernel_error *error);
int32_t et_b200_o2_optimizer_completed_updates_v1(
    const et_b200_o2_optimizer *optimizer, uint64_t *updates);
/* Device pointers of parameter `index`'s moments (for checkpoint/inspection). */
int32_t et_b200_o2_optimizer_moments_v1(et_b200_o2_optimizer *optimizer,
                                        size_t index, float **exp_avg,
                                        float **exp_avg_sq);
void et_b200_o2_optimizer_destroy_v1(et_b200_o2_optimizer **optimizer);
/* AdamW step for callers that cannot allocate device memory: hosts that give
 * all of HBM to their own allocator at start-up, and loops that keep the
 * device footprint fixed because cudaMalloc/cudaFree can synchronise the
 * device mid-step.  No counterpart in the reference (its O2 optimizer is a
 * CPU object).  The caller owns the parameter, gradient and both moments
 * (device f32, `count` elements, moments zero before update 1); the call
 * divides the gradient by the normalisation weight, computes the global L2
 * norm, clips to clip_max_bits when that is nonzero, and applies the O2
 * update `update` (1-based, constant schedule) with the same per-element
 * rounding as et_b200_o2_optimizer_step_v1.  Its only scratch is a 64 KiB
 * file-scope device array that every GPU loading the library holds until
 * exit; count above ET_B200_ADAMW_NOALLOC_MAX_ELEMENTS is rejected.  Calls
 * share that array and its contents persist between calls: the call clears
 * what must start at zero itself, and calls that overlap on the GPU (on
 * different streams or host threads) race on it.  The first call on each
 * device looks up the array's device address (cudaGetSymbolAddress) and
 * should come before any stream capture.  Enqueued on `stream` (a
 * cudaStream_t, NULL = legacy default stream) and synchronised before
 * returning; norm_bits (optional) receives the norm.  The update is all or
 * nothing: a nonfinite gradient, a norm beyond f32's range, a nonfinite
 * parameter or moment, or an update that would produce a nonfinite value
 * leaves every tensor unchanged and returns INVALID_ARGUMENT (messages as
 * the reference's optimizer-step!). */
#define ET_B200_ADAMW_NOALLOC_MAX_ELEMENTS ((uint64_t)8192u * 65536u)
int32_t et_b200_adamw_step_noalloc_v1(
    float *value, const float *gradient, float *exp_avg, float *exp_avg_sq,
    uint64_t count, uint32_t learning_rate_bits, uint32_t beta1_bits,
    uint32_t beta2_bits, uint32_t epsilon_bits, uint32_t weight_decay_bits,
    uint64_t update, uint32_t normalization_weight_bits,
    uint32_t clip_max_bits, void *stream, uint32_t *norm_bits,
    et_kernel_error *error);
/* The schedule factor of update `update` as f32 bits: 1 for the constant
 * schedule; the exactly rounded linear warmup/decay ratio otherwise
 * (replaces et_o2_schedule_factor, native/o2_optimizer.c:1345-1374). */
uint32_t et_b200_o2_schedule_factor_v1(uint32_t kind, uint64_t warmup,
                                       uint64_t total,
                                       uint32_t minimum_ratio_bits,
                                       uint64_t update);

/* ------------------------------------------------------------ LM training
 * A decoder-only LM training step composed from the same primitives in the
 * reference's schedule order (native/m3_schedule.esk:3-52): token embedding,
 * L pre-LN blocks (fused QKV linear, RoPE on Q/K, causal attention, output
 * linear, residual, LN, FFN up, exact-erf GELU, FFN down, residual), final
 * LN, head tied to the embedding, indexed cross-entropy with the 1/N token
 * weight fused into its backward, AdamW.  This is the training loop's fast
 * path: it runs the kernels directly instead of one K1 dispatch per role.
 */
enum {
  ET_B200_PRECISION_TF32X3 = 0, /* 3xTF32 tcgen05 contractions (f32-grade) */
  ET_B200_PRECISION_TF32 = 1,   /* single TF32 tcgen05 contractions        */
  ET_B200_PRECISION_F32 = 2,    /* FP32 FFMA contractions (no tensor core)  */
  ET_B200_PRECISION_F16X3 = 3   /* split-f16 tcgen05 contractions: binary16
                                   hi/lo pairs with per-tensor power-of-two
                                   scales, 3 products (f32-grade)           */
};

typedef struct et_b200_lm_config_v1 {
  size_t struct_size;
  int64_t layers;
  int64_t d_model;
  int64_t heads;
  int64_t ffn;
  int64_t vocabulary;
  int64_t seq_len;
  int64_t batch;            /* sequences per step on this rank */
  int64_t global_tokens;    /* CE weight N across all ranks; 0 = batch*seq */
  uint32_t ln_epsilon_bits; /* 0x3727c5ac = 1e-5 */
  uint32_t precision;       /* ET_B200_PRECISION_* */
  double rope_base;         /* 10000 */
  uint32_t learning_rate_bits, beta1_bits, beta2_bits, epsilon_bits,
      weight_decay_bits;
  uint32_t reserved;
} et_b200_lm_config_v1;

typedef struct et_b200_lm et_b200_lm;

int32_t et_b200_lm_create_v1(const et_b200_lm_config_v1 *config,
                             et_b200_lm **lm, et_kernel_error *error);
void et_b200_lm_destroy_v1(et_b200_lm **lm);
/* Parameter tensors, in order, and their element counts. */
size_t et_b200_lm_tensor_count_v1(const et_b200_lm *lm);
size_t et_b200_lm_parameter_count_v1(const et_b200_lm *lm);
int32_t et_b200_lm_tensor_sizes_v1(const et_b200_lm *lm, size_t *sizes);
/* Seeded initialisation: weights N(0, 0.02), LN gammas 1, biases 0. */
int32_t et_b200_lm_init_v1(et_b200_lm *lm, uint64_t seed,
                           et_kernel_error *error);
/* which: 0 parameters, 1 gradients, 2 exp_avg, 3 exp_avg_sq (host copies). */
int32_t et_b200_lm_read_v1(et_b200_lm *lm, int32_t which, float *host,
                           size_t count, et_kernel_error *error);
int32_t et_b200_lm_write_v1(et_b200_lm *lm, int32_t which, const float *host,
                            size_t count, et_kernel_error *error);
/* One training step from HOST token ids/targets [batch, seq_len]: copies
 * them in, runs forward, backward (with the data-parallel gradient allreduce
 * when enabled), the AdamW update, and copies the mean loss out.  The update
 * is all or nothing, as O2's staged commit is (o2_optimizer.c:1813-1926): a
 * token id or target outside the vocabulary (on any rank), a nonfinite
 * gradient, parameter or moment, or an update that would be nonfinite leaves
 * parameters, moments and the update counter unchanged and returns
 * INVALID_ARGUMENT. */
int32_t et_b200_lm_step_v1(et_b200_lm *lm, const int64_t *host_ids,
                           const int64_t *host_targets, float *host_loss,
                           et_kernel_error *error);
/* The same step on DEVICE-resident ids/targets; the mean loss stays on the
 * device (device_loss may be NULL).  Enqueued on the model's stream; returns
 * without synchronising.  A step the host call above would reject is
 * skipped on the device with nothing updated; such steps are counted by
 * et_b200_lm_update_counts_v1 (the update number of later steps is taken
 * from the device's count of applied updates, so skipped steps do not shift
 * the bias corrections). */
int32_t et_b200_lm_step_device_v1(et_b200_lm *lm, const int64_t *device_ids,
                                  const int64_t *device_targets,
                                  float *device_loss, et_kernel_error *error);
/* Forward + backward only (no optimizer update): gradients left in place. */
int32_t et_b200_lm_forward_backward_v1(et_b200_lm *lm,
                                       const int64_t *host_ids,
                                       const int64_t *host_targets,
                                       float *host_loss,
                                       et_kernel_error *error);
/* Loss mask of the following steps (the L3S masked objective,
 * native/l3s_masked_objective_provider.c:125-175, with the reference's O2
 * division by the accumulated weight, o2_optimizer.c:1738): `mask` is
 * u8 [batch * seq_len] (row-major [batch, seq_len], the D2 loss-mask plane),
 * each byte 0 or 1, in host memory (on_device 0: checked and copied before
 * the call returns) or device memory (on_device 1: copied on the model's
 * stream; a byte other than 0 / 1 voids the next step, which then reports
 * INVALID_ARGUMENT with nothing updated).  NULL restores the unmasked
 * objective.  With a mask the loss is sum(mask ce) / sum(mask) over this
 * rank's tokens, each token's CE gradient is seeded with mask 2^-k
 * (k = ceil(log2 global tokens), an exact scaling) so the gradients hold the
 * mask-weighted numerators 2^-k, and AdamW divides them by the global weight
 * sum(mask) 2^-k (summed over the data-parallel ranks with the last gradient
 * bucket).  A step whose global weight is 0 updates nothing and reports
 * INVALID_ARGUMENT.  No reference counterpart for the entry point itself: the
 * reference feeds the mask through its Eshkol objective bridge. */
int32_t et_b200_lm_set_loss_mask_v1(et_b200_lm *lm, const uint8_t *mask,
                                    int32_t on_device, et_kernel_error *error);
/* The cudaStream_t the model enqueues on. */
void *et_b200_lm_stream_v1(et_b200_lm *lm);

/* ------------------------------------------------------------ D2 batch planes
 * The i64 input / target planes and the bool loss-mask plane of a fixed
 * [rows, seq_len] batch from one flat token stream, by the row rule of the
 * reference's D2 shard loader in packed mode (docs/D2_SHARD_LOADER.md, "Rows,
 * shift, mask, and ordering"): the stream holds 0 rows when length < 2, else
 * 1 + floor((length - 2) / seq_len); row r starts at r seq_len; a position
 * whose target exists in the stream takes input token[s + t], target
 * token[s + t + 1] and mask 1; every other position holds 0, 0, 0.  Host
 * memory; rows first_row .. first_row + rows - 1 of the stream (rows past its
 * end are all padding); INVALID_ARGUMENT when first_row is past the last row
 * (a batch needs a true mask bit).  Shuffling and shard boundaries (unpacked
 * mode) stay with the caller's loader. */
int64_t et_b200_d2_row_count_v1(uint64_t tokens, int64_t seq_len);
int32_t et_b200_d2_rows_v1(const int64_t *tokens, uint64_t length, int64_t seq_len,
                           int64_t first_row, int64_t rows, int64_t *ids,
                           int64_t *targets, uint8_t *mask, et_kernel_error *error);
/* Data parallelism: NCCL communicator over `world` ranks.  unique_id is the
 * 128-byte ncclUniqueId rank 0 obtained from et_b200_nccl_unique_id_v1 and
 * shared with every rank.  Gradients are then summed across ranks in buckets
 * on a side stream as backward produces them. */
int32_t et_b200_nccl_unique_id_v1(uint8_t unique_id[128],
                                  et_kernel_error *error);
int32_t et_b200_lm_enable_data_parallel_v1(et_b200_lm *lm,
                                           const uint8_t unique_id[128],
                                           int32_t rank, int32_t world,
                                           et_kernel_error *error);
/* Per-kernel-class timing with CUDA events on the model's stream.  Classes,
 * in order: 0 GEMM, 1 attention forward, 2 attention backward, 3 cross-
 * entropy, 4 AdamW (the writing pass), 5 LayerNorm, 6 other elementwise,
 * 7 embedding, 8 TF32 split, 9 allreduce wait, 10 AdamW check pass.  read
 * fills count >= 44 doubles: per class
 * {launch groups, milliseconds, algorithmic FLOP, algorithmic bytes}
 * accumulated since profiling was enabled; collect folds the events of
 * device-side steps into those totals (host steps do it themselves). */
int32_t et_b200_lm_profile_v1(et_b200_lm *lm, int32_t enable);
int32_t et_b200_lm_profile_collect_v1(et_b200_lm *lm);
int32_t et_b200_lm_profile_read_v1(et_b200_lm *lm, double *out, size_t count);
/* Split-f16 models (ET_B200_PRECISION_F16X3): how many steps of the
 * host-synchronised calls had an operand reach binary16's overflow and were
 * redone with 3xTF32 contractions since the model was created (0 for other
 * modes).  No reference counterpart: the reference has one contraction mode. */
int32_t et_b200_lm_f16_redone_steps_v1(const et_b200_lm *lm);
/* Applied AdamW updates (the reference's completed_updates,
 * o2_optimizer.c:1929) and device-enqueued steps whose update was skipped
 * since the model was created; synchronises the model's stream.  No
 * reference counterpart for `skipped`: reference steps are host calls that
 * return their error. */
int32_t et_b200_lm_update_counts_v1(et_b200_lm *lm, uint64_t *completed,
                                    uint64_t *skipped, et_kernel_error *error);

/* ------------------------------------------------------------ A2 KV cache
 *
 * The reference's transactional K/V cache with its storage in device memory
 * (replaces include/eshkol_transformer/a2_kv_cache.h:42-147, semantics of
 * native/a2_kv_cache.c:394-880).  Same names, arguments, lease rules and error
 * categories/codes.  Differences a caller sees: K/V storage [layers, batch,
 * kv_heads, capacity, head_dimension], the lengths [batch] and the key-keep
 * mask [batch, capacity] handed out by views and read borrows are device
 * ("cuda") tensor views on the GPU that was current at create; stage_layer
 * sources may be "cpu" or "cuda" views; append_counts stays a "cpu" view.
 * Every call has finished its device work when it returns.  The views feed
 * the A2 provider's attention directly (cached decoding: Tq new tokens over
 * Tk = capacity keys, the key-keep mask broadcast over the queries).
 */
typedef struct et_a2_kv_cache et_a2_kv_cache;
typedef struct et_a2_kv_cache_transaction et_a2_kv_cache_transaction;
typedef struct et_a2_kv_cache_transaction_view et_a2_kv_cache_transaction_view;
typedef struct et_a2_kv_cache_read_borrow et_a2_kv_cache_read_borrow;
/* replaces a2_kv_cache.h:42-53 */
int32_t et_a2_kv_cache_abi_major_v1(void);
int32_t et_a2_kv_cache_abi_minor_v1(void);
int32_t et_a2_kv_cache_abi_require_v1(uint32_t major, uint32_t minimum_minor,
                                      et_kernel_error *error);
/* replaces a2_kv_cache.h:61-68 (storage zero-initialised in device memory) */
int32_t et_a2_kv_cache_create_v1(uint64_t layers, uint64_t batch,
                                 uint64_t kv_heads, uint64_t capacity,
                                 uint64_t head_dimension,
                                 et_a2_kv_cache **cache,
                                 et_kernel_error *error);
int32_t et_a2_kv_cache_destroy_v1(et_a2_kv_cache **cache,
                                  et_kernel_error *error);
/* replaces a2_kv_cache.h:70-85 */
int32_t et_a2_kv_cache_transaction_begin_v1(
    et_a2_kv_cache *cache, uint64_t append_width,
    const et_kernel_tensor_view_v1 *append_counts,
    et_a2_kv_cache_transaction **transaction, et_kernel_error *error);
/* replaces a2_kv_cache.h:87-96 ("cpu" or "cuda" sources).  "cuda" sources
 * are read after a device synchronisation, so work that produced them on any
 * stream of that device (and was enqueued before this call) has finished;
 * work enqueued later, from another host thread, is not waited for. */
int32_t et_a2_kv_cache_transaction_stage_layer_v1(
    et_a2_kv_cache_transaction *transaction, uint64_t layer,
    const et_kernel_tensor_view_v1 *keys,
    const et_kernel_tensor_view_v1 *values, et_kernel_error *error);
/* replaces a2_kv_cache.h:98-120 (device views) */
int32_t et_a2_kv_cache_transaction_view_begin_v1(
    et_a2_kv_cache_transaction *transaction, uint64_t layer,
    et_a2_kv_cache_transaction_view **view, et_kernel_error *error);
int32_t et_a2_kv_cache_transaction_view_tensors_v1(
    const et_a2_kv_cache_transaction_view *view,
    const et_kernel_tensor_view_v1 **keys,
    const et_kernel_tensor_view_v1 **values,
    const et_kernel_tensor_view_v1 **effective_lengths,
    const et_kernel_tensor_view_v1 **key_keep_mask,
    et_kernel_error *error);
int32_t et_a2_kv_cache_transaction_view_end_v1(
    et_a2_kv_cache_transaction_view **view, et_kernel_error *error);
/* replaces a2_kv_cache.h:122-126 (abort scrubs staged slots to +0) */
int32_t et_a2_kv_cache_transaction_commit_v1(
    et_a2_kv_cache_transaction **transaction, et_kernel_error *error);
int32_t et_a2_kv_cache_transaction_abort_v1(
    et_a2_kv_cache_transaction **transaction, et_kernel_error *error);
/* replaces a2_kv_cache.h:128-147 (device views) */
int32_t et_a2_kv_cache_read_borrow_begin_v1(
    et_a2_kv_cache *cache, et_a2_kv_cache_read_borrow **borrow,
    et_kernel_error *error);
int32_t et_a2_kv_cache_read_borrow_layer_v1(
    et_a2_kv_cache_read_borrow *borrow, uint64_t layer,
    const et_kernel_tensor_view_v1 **keys,
    const et_kernel_tensor_view_v1 **values,
    const et_kernel_tensor_view_v1 **lengths,
    const et_kernel_tensor_view_v1 **key_keep_mask,
    et_kernel_error *error);
int32_t et_a2_kv_cache_read_borrow_end_v1(
    et_a2_kv_cache_read_borrow **borrow, et_kernel_error *error);

#ifdef __cplusplus
}
#endif

#include "eshkol_b200/o2_bridge.h"
#endif
