// Causal attention with RoPE on device tensors: et_b200_attention_*_v1.
//
// The A2 provider's arithmetic (native/a2_attention_provider.c:669-790,
// rope :792-935) without a K1 round trip: the caller passes device Q/K/V
// [batch, heads, len, head_dim], positions and an optional keep mask, and the
// calls enqueue on its stream without synchronising.  The forward returns the
// per-row statistics (row max of the scaled scores, sum of exponentials), so
// the backward does not recompute the forward the way a K1 backward call must
// (the K1 backward receives only Q/K/V/dO).  RoPE (when tables are given) is
// applied to Q and K on load and its backward rotation to dQ and dK, as the
// reference's rope.forward / rope.backward around the attention op.
#include <math.h>

#include "ops.cuh"

using namespace etb;

namespace {

int32_t check_shape(const et_b200_attention_v1* s, et_kernel_error* e, const char* op) {
  if (s == nullptr || s->struct_size < sizeof(et_b200_attention_v1))
    return set_error(e, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_INVALID_STRUCT_SIZE, op,
                     "attention descriptor is missing or truncated");
  if (s->batch < 1 || s->q_heads < 1 || s->kv_heads < 1 || s->q_heads % s->kv_heads != 0 ||
      s->q_len < 1 || s->k_len < 1 || s->head_dim < 2 || s->head_dim % 2 != 0 ||
      s->head_dim > 256 || s->batch * s->q_heads * s->q_len > INT32_MAX ||
      s->batch * s->kv_heads * s->k_len > INT32_MAX)
    return set_error(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                     "attention shape is outside [batch, heads, len, head_dim] limits");
  if (s->q_positions == nullptr || s->k_positions == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "query and key positions are required");
  if (s->contraction != ET_B200_ATTENTION_DEFAULT && s->contraction != ET_B200_ATTENTION_BWD_PAIRS16 &&
      s->contraction != ET_B200_ATTENTION_TF32)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op,
                     "unknown attention contraction mode");
  if ((s->rope_cos == nullptr) != (s->rope_sin == nullptr))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "RoPE needs both the cosine and the sine table");
  return 0;
}

AttnParams params_of(const et_b200_attention_v1* s, const float* q, const float* k,
                     const float* v) {
  AttnParams p{};
  p.B = (int)s->batch; p.Hq = (int)s->q_heads; p.Hkv = (int)s->kv_heads;
  p.Tq = (int)s->q_len; p.Tk = (int)s->k_len; p.Dh = (int)s->head_dim;
  volatile float root = sqrtf((float)s->head_dim);  // a2_attention_provider.c:221
  p.scale = 1.0f / root;
  const int64_t Dh = s->head_dim;
  p.q = AttnTensor{q, s->q_heads * s->q_len * Dh, s->q_len * Dh, Dh};
  p.k = AttnTensor{k, s->kv_heads * s->k_len * Dh, s->k_len * Dh, Dh};
  p.v = AttnTensor{v, s->kv_heads * s->k_len * Dh, s->k_len * Dh, Dh};
  p.qpos = s->q_positions;
  p.kpos = s->k_positions;
  p.mask = s->keep;
  p.q_cos = s->rope_cos; p.q_sin = s->rope_sin;
  p.k_cos = s->rope_cos; p.k_sin = s->rope_sin;
  p.q_rope_batched = s->rope_batched ? 1 : 0;
  p.k_rope_batched = s->rope_batched ? 1 : 0;
  p.bwd_pairs16 = s->contraction == ET_B200_ATTENTION_BWD_PAIRS16 ? 1 : 0;
  p.single = s->contraction == ET_B200_ATTENTION_TF32 ? 1 : 0;
  return p;
}

// Workspace: the attention kernels' part, then delta (one float per query
// row, the backward's rowsum(dO o)).
size_t delta_offset(const AttnParams& p) { return (attention_workspace_floats(p) + 63) & ~(size_t)63; }
size_t workspace_floats(const AttnParams& p) {
  return delta_offset(p) + (((size_t)p.B * p.Hq * p.Tq + 63) & ~(size_t)63);
}

int32_t workspace_ok(const AttnParams& p, void* ws, size_t bytes, et_kernel_error* e,
                     const char* op) {
  if (bytes < workspace_floats(p) * sizeof(float) ||
      (ws == nullptr && bytes != 0) || (reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_BUFFER_TOO_SMALL, op,
                     "workspace is smaller than et_b200_attention_workspace_bytes_v1 or not "
                     "256-byte aligned");
  return 0;
}

int32_t launched(et_kernel_error* e, const char* op) {
  const cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return cuda_error(e, st, op);
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

}  // namespace

extern "C" {

size_t et_b200_attention_workspace_bytes_v1(const et_b200_attention_v1* s) {
  if (check_shape(s, nullptr, "attention-workspace")) return 0;
  const AttnParams p = params_of(s, nullptr, nullptr, nullptr);
  return workspace_floats(p) * sizeof(float);
}

void et_b200_rope_tables_v1(int64_t len, int64_t head_dim, double base, float* cos_out,
                            float* sin_out) {
  // the trainer's and the reference's construction: inv_freq in double
  // rounded to f32, angle = (float)t * inv_freq in f32, libm cosf / sinf
  const int64_t half = head_dim / 2;
  for (int64_t i = 0; i < half; i++) {
    const float inv = (float)(1.0 / pow(base, (double)(2 * i) / (double)head_dim));
    for (int64_t t = 0; t < len; t++) {
      volatile float angle = (float)t * inv;
      cos_out[t * half + i] = cosf(angle);
      sin_out[t * half + i] = sinf(angle);
    }
  }
}

int32_t et_b200_attention_forward_v1(const et_b200_attention_v1* s, const float* q,
                                     const float* k, const float* v, float* o, float* row_max,
                                     float* row_sum, void* workspace, size_t workspace_bytes,
                                     void* stream, et_kernel_error* e) {
  const char* op = "attention-forward";
  if (int32_t r = check_shape(s, e, op)) return r;
  if (!q || !k || !v || !o || !row_max || !row_sum)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "q, k, v, o and both row statistics are required");
  AttnParams p = params_of(s, q, k, v);
  if (int32_t r = workspace_ok(p, workspace, workspace_bytes, e, op)) return r;
  p.ws = static_cast<float*>(workspace);
  const int64_t Dh = s->head_dim;
  attention_forward(p, AttnOut{o, s->q_heads * s->q_len * Dh, s->q_len * Dh, Dh}, row_max,
                    row_sum, static_cast<cudaStream_t>(stream));
  return launched(e, op);
}

int32_t et_b200_attention_backward_v1(const et_b200_attention_v1* s, const float* q,
                                      const float* k, const float* v, const float* o,
                                      const float* dout, const float* row_max,
                                      const float* row_sum, float* dq, float* dk, float* dv,
                                      void* workspace, size_t workspace_bytes,
                                      int32_t workspace_from_forward, void* stream,
                                      et_kernel_error* e) {
  const char* op = "attention-backward";
  if (int32_t r = check_shape(s, e, op)) return r;
  if (!q || !k || !v || !o || !dout || !row_max || !row_sum || !dq || !dk || !dv)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "every tensor of the backward is required");
  AttnParams p = params_of(s, q, k, v);
  if (int32_t r = workspace_ok(p, workspace, workspace_bytes, e, op)) return r;
  p.ws = static_cast<float*>(workspace);
  // the forward prepared Q/K/V into the workspace only on the tensor-core path
  QkvPrep prep;
  p.ws_ready = workspace_from_forward && attention_qkv_prep(p, &prep) ? 1 : 0;
  const int64_t Dh = s->head_dim;
  const int64_t qsb = s->q_heads * s->q_len * Dh, qsh = s->q_len * Dh;
  const int64_t ksb = s->kv_heads * s->k_len * Dh, ksh = s->k_len * Dh;
  float* delta = static_cast<float*>(workspace) + delta_offset(p);
  attention_backward(p, AttnTensor{o, qsb, qsh, Dh}, nullptr, AttnTensor{dout, qsb, qsh, Dh},
                     row_max, row_sum, delta, AttnOut{dq, qsb, qsh, Dh},
                     AttnOut{dk, ksb, ksh, Dh}, AttnOut{dv, ksb, ksh, Dh},
                     static_cast<cudaStream_t>(stream));
  return launched(e, op);
}

}  // extern "C"
