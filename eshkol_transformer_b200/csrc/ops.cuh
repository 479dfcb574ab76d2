// Internal launch API shared by the libet_b200 translation units.  Every
// function enqueues on `stream`, counts its launches and never synchronises.
#pragma once

#include "common.cuh"

namespace etb {

// ---------------------------------------------------------------- L2 CE
// Fused indexed cross-entropy: per row r of logits [rows, V], the loss
// log(sum exp(x - m)) + (m - x[t]) and, when dlogits != nullptr, the gradient
// u_r (softmax(x) - onehot(t)) with u_r = upstream[r] (or upstream_scale when
// upstream is null).  dlogits may alias logits.  status[0] is set to 1 when a
// target is outside [0, V).
// With dlogits_lo, dlogits receives the TF32 hi part and dlogits_lo the
// residual (the 3xTF32 operand pair) instead of the f32 gradient; with
// sc.f16 the binary16 pair of the gradient 2^(*sc.exp) (dlogits must not
// alias logits then); sc.amax receives max |gradient|.
void ce_fused(const float* logits, float* dlogits, const int64_t* targets,
              const float* upstream, float upstream_scale, float* loss,
              size_t rows, size_t V, int* status, cudaStream_t stream,
              float* dlogits_lo = nullptr, OperandScale sc = OperandScale{});
// Mean of loss[rows] as one f32 (fixed-order tree in f64); with `mask`
// (u8 [rows], 0 / 1) the masked mean sum(mask loss) / sum(mask), +0 when no
// row is selected.
void mean_loss(const float* loss, size_t rows, float* out, cudaStream_t stream,
               const uint8_t* mask = nullptr);
// The L3S numerator seed of a loss mask (native/l3s_masked_objective_provider.c:
// 125-175): upstream[r] = mask[r] ? scale : 0, and *weight = sum of the mask
// (the objective's weight, as f32); a byte other than 0 or 1 sets bit 2 of
// status[0] (the reference rejects it).
void loss_mask_seed(const uint8_t* mask, size_t rows, float scale, float* upstream, float* weight,
                    int* status, cudaStream_t stream);

// ---------------------------------------------------------------- O2 AdamW
struct AdamwTensor {
  float* value;
  const float* grad;
  float* exp_avg;
  float* exp_avg_sq;
  uint64_t count;
  // per-tensor scalars computed on the host with the reference's rounding
  float beta1, beta2, one_minus_beta1, one_minus_beta2, bias1, bias2, lr,
      decay, epsilon;
  // optional: the updated value's TF32 hi / residual lo pair (the weight
  // operands of the 3xTF32 GEMMs), written in the same pass; with value_sc.f16
  // the binary16 pair of value 2^(*value_sc.exp) instead (uint16 arrays)
  float* value_hi;
  float* value_lo;
  OperandScale value_sc;
  // 1 when this tensor's scalars admit adamw_check's finiteness envelope
  // (adamw_envelope_ok); 0 computes every element's update in the check
  int envelope;
};
// The scalars of T (lr, epsilon, decay, with bias corrections >= 2^-24 as
// every 1 - beta^t of a beta < 1 is) admit the envelope under which an
// element's update is finite without computing it.
bool adamw_envelope_ok(const AdamwTensor& T);
// An AdamW update is all or nothing, as the reference's staged commit is
// (o2_optimizer.c:1813-1926): adamw_check computes every element's update
// without writing and sets status bits; adamw_apply then writes the table
// only if no bit is set.  Both are fused passes over every tensor of the
// table (device array `tensors`, `prefix[i]` = first global element of tensor
// i, total = prefix[count]); weight/clip divide and scale gradients as
// o2_optimizer.c:1738 does.
enum : int {
  kAdamwInputNonfinite = 1,     // a parameter, gradient or moment is nonfinite
  kAdamwProducedNonfinite = 2,  // an intermediate or result is nonfinite
};
struct AdamwControl {
  const float* skip;     // optional: nothing is checked or written when *skip != 0
  int* status;           // [1] |= kAdamw* bits (check); [2] += 1 per skipped apply
  uint64_t* completed;   // optional: applied updates, +1 by each apply that writes
  // optional: the gradients' normalisation weight read on the device
  // (*weight_dev * weight_mul replaces the `weight` argument)
  const float* weight_dev;
  float weight_mul;
};
// `vec`: every tensor's arrays are 16-byte aligned and its count a multiple
// of 4 (128-bit loads and stores).
void adamw_check(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                 uint64_t total, float weight, float clip, AdamwControl ctl, bool vec,
                 cudaStream_t stream);
void adamw_apply(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                 uint64_t total, float weight, float clip, AdamwControl ctl, bool vec,
                 cudaStream_t stream);
// tensors[0].bias1 / bias2 of update *completed + 1, computed on the device
// with the host's rounding sequence (o2_optimizer.c:419-435), so that steps
// enqueued without a host synchronisation, some of which may be skipped,
// still use the right update number.
void adamw_prepare(AdamwTensor* tensors, const uint64_t* completed, cudaStream_t stream);
// *flag += amount when status[0] is set (a token id or target of the step is
// out of range).
void fold_index_flag(const int* status, float* flag, float amount, cudaStream_t stream);
// Sum of squares of grad/weight over the table, in f64, plus status[0] = 1 on
// any nonfinite gradient.  out_sumsq receives one double.
void grad_sumsq(const AdamwTensor* tensors, const uint64_t* prefix,
                int tensor_count, uint64_t total, float weight,
                double* partials, int partial_count, double* out_sumsq,
                int* status, cudaStream_t stream);

// ---------------------------------------------------------------- N2 family
// With y_lo, y receives the TF32 hi part of the output and y_lo the residual;
// with sc.f16 the binary16 pair (y as hi, y_lo as lo, both uint16 arrays) of
// y 2^(*sc.exp); sc.amax (either format) receives max |y|.
void layer_norm_forward(const float* x, const float* gamma, const float* beta,
                        float epsilon, float* y, float* mean, float* rstd,
                        size_t rows, size_t d, cudaStream_t stream, float* y_lo = nullptr,
                        OperandScale sc = OperandScale{});
// dx = (accumulate ? dx : 0) + LN'(dy); dgamma/dbeta over all rows via a
// fixed-order two-stage column reduction in `workspace` (>= ln_workspace()).
size_t ln_workspace_floats(size_t rows, size_t d);
// With dx_hi/dx_lo, the final dx is also written as a 3xTF32 operand pair (or
// with sc.f16 as the binary16 pair of dx 2^(*sc.exp); d % 128 == 0, d <= 1024
// only); with dsum, the column sums of the final dx (the next bias gradient).
void layer_norm_backward(const float* x, const float* gamma, const float* mean,
                         const float* rstd, const float* dy, float* dx,
                         int accumulate, float* dgamma, float* dbeta,
                         float* workspace, size_t rows, size_t d,
                         cudaStream_t stream, float* dx_hi = nullptr, float* dx_lo = nullptr,
                         float* dsum = nullptr, OperandScale sc = OperandScale{});
// With a lo output, the result is written as TF32 hi (y / dx) plus residual.
void gelu_forward(const float* x, float* y, size_t count, cudaStream_t stream,
                  float* y_lo = nullptr);
void gelu_backward(const float* x, const float* dy, float* dx, size_t count,
                   cudaStream_t stream, float* dx_lo = nullptr);
// GELU backward over a [rows, n] matrix that also sums the columns of dx
// (the bias gradient of the layer that produced x) into dsum; `workspace`
// holds gelu_colsum_workspace_floats(rows, n) floats.
size_t gelu_colsum_workspace_floats(size_t rows, size_t n);
void gelu_backward_colsum(const float* x, const float* dy, float* dx, float* dx_lo, float* dsum,
                          float* workspace, size_t rows, size_t n, cudaStream_t stream);
void relu_forward(const float* x, float* y, size_t count, cudaStream_t stream);
void relu_backward(const float* x, const float* dy, float* dx, size_t count,
                   cudaStream_t stream);
void add_tensors(const float* a, const float* b, float* out, size_t count,
                 cudaStream_t stream);
void copy_tensor(const float* a, float* out, size_t count, cudaStream_t stream);
// Row gather y[r] = W[ids[r]]; status[0] = 1 on an id outside [0, V).
void embedding_forward(const int64_t* ids, const float* w, float* y,
                       size_t rows, size_t V, size_t d, int* status,
                       cudaStream_t stream);
// dW[v] = (base ? base[v] : 0) + (sum over rows r with ids[r] == v, in
// ascending r, starting from +0).  Bit-identical to the reference's order.
// `scratch` holds >= embedding_scratch_bytes(rows, V) bytes.
size_t embedding_scratch_bytes(size_t rows, size_t V);
void embedding_backward(const int64_t* ids, const float* dy, const float* base,
                        float* dw, size_t rows, size_t V, size_t d,
                        void* scratch, cudaStream_t stream);
// out[n] = sum over rows of dy[r, n] (fixed-order two-stage).
size_t colsum_workspace_floats(size_t rows, size_t n);
// out_q[j] = sum over p of partial[p * stride + q * width + j] for the
// quantities q = 0, 1, 2 whose outputs o0, o1, o2 are given (o1, o2 may be
// null); a fixed summation order (deterministic).
void reduce_partials(const float* partial, int count, int64_t width, int64_t stride, float* o0,
                     float* o1, float* o2, cudaStream_t stream);
// dy_lo (optional) is added to dy element by element first (hi + lo is exact).
void column_sum(const float* dy, float* out, size_t rows, size_t n,
                float* workspace, cudaStream_t stream, const float* dy_lo = nullptr);
// 3xTF32 operand split: hi = x rounded to the nearest TF32 value (exactly
// representable, low 13 mantissa bits zero) and lo = x - hi (exact, at most
// 2^-11 |x|).  hi may alias x.
void split_tf32(const float* x, float* hi, float* lo, size_t count, cudaStream_t stream);
// Standalone RoPE over [N,H,T,Dh] with a host-built cos/sin table
// [N*T, Dh/2] each (bit-identical rotation).
void rope_apply(const float* x, float* y, const float* cos_table,
                const float* sin_table, size_t N, size_t H, size_t T,
                size_t Dh, int backward, cudaStream_t stream);
// ---- split-f16 operand pairs (OperandScale in common.cuh)
// *amax = max(*amax, max |x|) as f32 bits (not reset here).
void abs_max(const float* x, size_t count, unsigned* amax, cudaStream_t stream);
// Per slot i: exp[i] = target - k for amax[i] = f 2^k, f in [0.5, 1) (amax
// 2^exp in [2^(target-1), 2^target)); a zero or nonfinite amax keeps
// exp[i]; amax cleared when reset.
void scale_from_amax(unsigned* amax, int* exp, int count, int target, int reset,
                     cudaStream_t stream);
// hi / lo binary16 arrays of (x + xlo) 2^(*exp) (xlo optional); the max |x +
// xlo| goes to amax when it is not null.
void split_f16(const float* x, const float* xlo, size_t count, uint16_t* hi, uint16_t* lo,
               const int* exp, unsigned* amax, cudaStream_t stream);
// flag[0] += 1.0 when some slot's amax 2^exp is not below 65504 (a binary16
// overflow) or NaN; then clears amax[reset_slot] (if >= 0).
void operand_range_check(unsigned* amax, const int* exp, int count, int reset_slot, float* flag,
                         cudaStream_t stream);
// status flags: sets *flag = 1 if any of count values is nonfinite.
void check_finite(const float* x, size_t count, int* flag, cudaStream_t stream);

// ---------------------------------------------------------------- A2
// Strided attention operands: element (b, h, t, j) of a tensor lives at
// base + b*sb + h*sh + t*st + j.
struct AttnTensor {
  const float* ptr;
  int64_t sb, sh, st;
};
struct AttnOut {
  float* ptr;
  int64_t sb, sh, st;
  // optional: when set (same strides as ptr), ptr receives the TF32 hi part
  // and lo the residual (a 3xTF32 operand pair); tensor-core kernels only
  float* lo;
  // optional (tensor-core backward): per 128-row tile of each sequence, the
  // column sums of that tile's rows go to colsum[(b * ceil(T/128) + tile) *
  // colsum_ld + h * Dh + j]; summed over the B * ceil(T/128) rows they are the
  // column sums of the whole gradient (a bias gradient)
  float* colsum;
  int64_t colsum_ld;
  // optional (tensor-core kernels): sc.f16 makes ptr / lo the binary16 pair
  // of the output 2^(*sc.exp) (uint16 arrays, same element strides; 8-byte
  // aligned rows); sc.amax receives max |output| in either format
  OperandScale sc;
};
struct AttnParams {
  int B, Hq, Hkv, Tq, Tk, Dh;
  float scale;
  AttnTensor q, k, v;
  // positions i64 [B,Tq] / [B,Tk]; keep mask u8 [B,Tq,Tk] (null = all kept)
  const int64_t* qpos;
  const int64_t* kpos;
  const uint8_t* mask;
  // optional RoPE applied to q/k on load (tables [B*T, Dh/2]; null = none)
  const float* q_cos;
  const float* q_sin;
  const float* k_cos;
  const float* k_sin;
  // 1 when a table has B*T rows (row b*T + t), 0 when it has T rows shared
  // by every sequence (row t).
  int q_rope_batched, k_rope_batched;
  // optional device workspace of attention_workspace_floats(p) floats, 16-byte
  // aligned; the tensor-core kernels need it (null = SIMT kernels).  With
  // ws_grad set, the backward's dO / statistics part lives there instead
  // (attention_grad_workspace_floats) and ws needs only the Q/K/V part
  // (attention_qkv_workspace_floats).  ws_ready: ws already holds this
  // call's prepared Q/K/V (written by its forward), so the backward skips
  // that pass.
  float* ws;
  float* ws_grad;
  int ws_ready;
  // qkv_ready: ws already holds the prepared Q/K/V (the fused QKV GEMM
  // epilogue wrote them), so the forward skips that pass as well.
  int qkv_ready;
  // grad_ready: the backward's dO hi/lo (workspace) and delta were written by
  // the GEMM that produced dO (AttnGradPrep), so the backward skips its prepass.
  int grad_ready;
  // bwd_pairs16: the backward carries its operands as binary16 pairs
  // (attention_bwd_f16.cu) wherever that kernel exists (head_dim 64, 128);
  // otherwise only head_dim 128 uses it and 32 / 64 take the 3xTF32 kernels.
  int bwd_pairs16;
  // single: one product of the hi parts per contraction (TF32-grade: 11
  // significant bits per operand element) instead of the three of the
  // f32-grade pairs
  int single;
  // pairs16 (head_dim 64 / 128): the producers write the binary16 operand
  // pairs themselves, each operand x as x 2^pair_exps[i] (i = 0 Q, 1 K, 2 V,
  // 3 dO): the QKV GEMM epilogue writes the Q / K / V pairs at the start of
  // ws (qkv_ready), the dO GEMM epilogue the dO pair, delta and lse2 in
  // ws_grad (grad_ready; the backward needs it).  The forward and the
  // backward of one call both set it.
  int pairs16;
  const int* pair_exps;
  // optional: pair_amax[0..3] receives max |x| of Q, K, V (the QKV epilogue,
  // after RoPE) and dO (the dO epilogue) in either operand format; with
  // pairs16 the backward takes dS's exponent from this call's V and dO
  // maxima there (they bound |dS|), so they must be recorded before it runs
  unsigned* pair_amax;
};
// Where the GEMM producing dO = dY Wo (rows [B*T, H*Dh], token-major) writes
// the attention backward's inputs: dO split into TF32 hi / lo head-major
// [B, H, T, Dh] and delta[(b*H + h)*T + t] = sum_j dO_j (o_j + o_lo_j) over
// the head's Dh columns (o, o_lo: the forward output, same layout as dO), and
// the row's base-2 log-sum-exp lse2 from the forward's statistics.
struct AttnGradPrep {
  int T, H, Dh;
  const float* o;
  const float* o_lo;
  // non-null: o / o_lo are the binary16 pair of o 2^(*o_exp) (uint16 arrays)
  const int* o_exp;
  const float *row_max, *row_sum;
  float *doh, *dol, *delta, *lse2;
  // non-null (AttnParams.pairs16): dO goes to g16h / g16l as the binary16
  // pair of dO 2^(*g_exp) instead of doh / dol
  uint16_t *g16h, *g16l;
  const int* g_exp;
  // optional: receives max |dO| (either format)
  unsigned* g_amax;
};
// The AttnGradPrep of p's backward workspace when the tensor-core backward
// will run with o given as the merged [B*T, Hq*Dh] rows (false otherwise).
bool attention_grad_prep(const AttnParams& p, AttnTensor o, const float* o_lo,
                         const float* row_max, const float* row_sum, float* delta,
                         AttnGradPrep* out);
// The same from a dO matrix already in memory (row stride ld).
void attention_prepare_grad_from(const float* dout, int64_t ld, int rows, const AttnGradPrep& g,
                                 cudaStream_t stream);
// Where a fused QKV projection writes the attention operands: the RoPE'd Q
// and K and plain V of a [B*T, (Hq + 2 Hkv) Dh] row-major qkv matrix (the
// columns Q | K | V, head-major within each), split into TF32 hi / residual
// lo, each [B, H, T, Dh] (the layout attention_prepare_qkv writes).
struct QkvPrep {
  int T, Hq, Hkv, Dh;
  const float *q_cos, *q_sin, *k_cos, *k_sin;  // null: no RoPE
  int q_rope_batched, k_rope_batched;
  float *qh, *ql, *kh, *kl, *vh, *vl;
  // non-null q16h (AttnParams.pairs16): the operands go to the binary16 pairs
  // q16h / q16l, k16h / k16l, v16h / v16l (same element layout) as x
  // 2^exps[i] (i = 0 Q, 1 K, 2 V) instead of the TF32 pairs
  uint16_t *q16h, *q16l, *k16h, *k16l, *v16h, *v16l;
  const int* exps;
  // optional: amax[i] receives max |x| of section i (either format)
  unsigned* amax;
};
// The QkvPrep of p's workspace (p.ws set, p.q / p.k / p.v columns of one qkv
// matrix); false when the tensor-core attention cannot use it (Dh not
// 32 / 64 / 128, or 32 with pairs16, or no workspace).
bool attention_qkv_prep(const AttnParams& p, QkvPrep* out);
// The same operands from a qkv matrix already in memory (row stride ld).
void attention_prepare_from_qkv(const float* qkv, int64_t ld, int rows, const QkvPrep& q,
                                cudaStream_t stream);
size_t attention_workspace_floats(const AttnParams& p);
size_t attention_qkv_workspace_floats(const AttnParams& p);
size_t attention_grad_workspace_floats(const AttnParams& p);
// Forward: o and per-row statistics m (row max of scaled scores) and l (sum
// of exp(s - m)); rows with no admitted key produce o = 0, m = 0, l = 0.
// Returns true when the tensor-core path ran (and so prepared p.ws).
bool attention_forward(const AttnParams& p, AttnOut o, float* row_max,
                       float* row_sum, cudaStream_t stream);
// The tcgen05 forward (attention_tc.cu); false when the shape or layout is
// outside it (Dh not 32/64/128, strides TMA cannot describe), nothing launched.
bool attention_forward_tc(const AttnParams& p, AttnOut o, float* row_max,
                          float* row_sum, cudaStream_t stream);
// Backward: dq/dk/dv (RoPE backward applied to dq/dk when tables are set).
// delta[B*Hq*Tq] is scratch for rowsum(dO * O); when o_lo is given (same
// strides as o) the forward output is o + o_lo (a 3xTF32 hi/lo pair).
// Returns true when the tensor-core path ran (the only one writing lo outputs).
bool attention_backward(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                        const float* row_max, const float* row_sum,
                        float* delta, AttnOut dq, AttnOut dk, AttnOut dv,
                        cudaStream_t stream);
// The tcgen05 backward (attention_bwd_tc.cu); false when the shape is outside
// it (Dh not 32/64, no workspace), nothing launched.
bool attention_backward_tc(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                           const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                           AttnOut dk, AttnOut dv, cudaStream_t stream);
// Whether attention carries binary16 operand pairs for p: always at
// head_dim 128, at head_dim 64 with bwd_pairs16 or from Tq Tk = 768^2 up
// (forward and backward decide alike, so a backward reuses its forward's
// pairs).
bool attention_uses_pairs16(const AttnParams& p);
// Binary16 pairs of RoPE'd Q, K and V and their maxima into the workspace.
void attention_prepare_pairs16(const AttnParams& p, cudaStream_t stream);
// The binary16-pair tensor-core forward (head_dim 64 and 128).
bool attention_forward_f16(const AttnParams& p, AttnOut o, float* row_max, float* row_sum,
                           cudaStream_t stream);
// The binary16-pair tensor-core backward (head_dim 64 and 128, dO from
// `dout`: not with grad_ready); false when it cannot run this call.
bool attention_backward_f16(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                            const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                            AttnOut dk, AttnOut dv, cudaStream_t stream);

// ---------------------------------------------------------------- GEMM
// Floats of GemmArgs::chunk_ws for any GEMM on the current device.
size_t gemm_chunk_ws_floats();
// C[m, n] = sum_k A(m, k) B(n, k) (+ bias[n]) (+ C when accumulate).
// A(m,k) = a_kmajor ? A[m*lda + k] : A[k*lda + m]
// B(n,k) = b_kmajor ? B[n*ldb + k] : B[k*ldb + n]
// For the TF32 modes a_lo/b_lo hold x - tf32(x) of the same layout (3xTF32
// uses A*B + A*B_lo + A_lo*B); they are ignored in the other modes.
struct GemmArgs {
  int M, N, K;
  const float* A;
  const float* A_lo;
  int64_t lda;
  bool a_kmajor;
  const float* B;
  const float* B_lo;
  int64_t ldb;
  bool b_kmajor;
  float* C;
  int64_t ldc;
  const float* bias;
  bool accumulate;
  // optional scratch for split-K: when the output has too few tiles to fill
  // the GPU and K is long, the K range is split across CTAs into partial
  // [M, N] sums here, then reduced in a fixed order (gemm_splitk_floats).
  float* workspace;
  size_t workspace_floats;
  // optional scratch of gemm_chunk_ws_floats() floats: the f32-grade pair
  // GEMM then sums K in chunks (the tensor pipe's accumulation truncates, so
  // one accumulator over a long K drifts) and adds them in f32 here.  Calls
  // that may run at the same time need separate scratch.
  float* chunk_ws;
  size_t chunk_ws_floats;
  // Epilogue applied to y = sum_k A B (all outputs share ldc; `accumulate`
  // applies to GEMM_EPI_PLAIN only):
  //   PLAIN     C = y (+ bias) (+ C)
  //   RESIDUAL  C = y + bias + aux                    (aux: residual stream)
  //   GELU_FWD  C = u = y + bias; out2 = GELU(u), or its TF32 hi with out3 = lo
  //   GELU_BWD  d = y * GELU'(aux) (aux = the GELU input); C = d, or its TF32
  //             hi with out2 = lo; dsum[n] = column sums of d (the bias
  //             gradient), through `epi_ws` (gemm_epilogue_ws_floats)
  //   QKV       C = y + bias, and the attention operands of C (QkvPrep `qkv`)
  //   ATTN_DO   C = y, and the attention backward's dO hi/lo and delta
  //             (AttnGradPrep `dprep`)
  int epilogue;
  const float* aux;
  float* out2;
  float* out3;
  float* dsum;
  float* epi_ws;
  const QkvPrep* qkv;
  const AttnGradPrep* dprep;
  // split-f16 operands: A/B (and A_lo/B_lo) hold binary16 arrays scaled by
  // 2^(*exp_a) / 2^(*exp_b); pair kernel only
  bool f16;
  const int* exp_a;
  const int* exp_b;
  // format, scale and max-|x| slot of the GELU_FWD (out2/out3) or GELU_BWD
  // (C/out2) operand-pair output
  OperandScale out_sc;
  // QKV / ATTN_DO on the pair kernel's staged epilogue: leave C unwritten
  // (when the attention operands it writes are C's only consumers)
  bool skip_c;
  // GELU_FWD: C receives GELU'(u) instead of u; GELU_BWD: aux is GELU'(u)
  // (pair kernel's staged epilogue only)
  bool gelu_slope_c;
};
enum {
  GEMM_EPI_PLAIN = 0,
  GEMM_EPI_RESIDUAL = 1,
  GEMM_EPI_GELU_FWD = 2,
  GEMM_EPI_GELU_BWD = 3,
  GEMM_EPI_QKV = 4,
  GEMM_EPI_ATTN_DO = 5
};
// Scratch floats split-K may use for an M x N output.
size_t gemm_splitk_floats(int M, int N);
// Scratch floats the GELU_BWD epilogue needs for an M x N output.
size_t gemm_epilogue_ws_floats(int M, int N);
void gemm(const GemmArgs& g, int precision, cudaStream_t stream);
// True when the tensor-core path accepts this problem (alignment / shape);
// otherwise gemm() uses the FFMA path.
bool gemm_tc_supported(const GemmArgs& g);
void gemm_simt(const GemmArgs& g, cudaStream_t stream);
void gemm_tc(const GemmArgs& g, bool three_pass, cudaStream_t stream);

}  // namespace etb
