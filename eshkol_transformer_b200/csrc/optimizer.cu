// O2 AdamW over caller-owned device tensors (native/o2_optimizer.c).
//
// Step order follows et_o2_optimizer_step_v1 (o2_optimizer.c:1784-1944):
// validate the normalisation weight, compute the schedule factor, the global
// gradient norm of g / W (always), the clip factor, then update every tensor.
// The norm pass also checks every gradient is finite before anything is
// written.  The update itself is one fused multi-tensor kernel whose
// per-element operations round exactly where the reference rounds
// (o2_optimizer.c:1738-1756), so parameters and moments are bit-identical.
// The global norm is summed in f64 in a fixed order; the reference's scaled
// running sum differs from it by rounding only.
#include <math.h>

#include <vector>

#include "ops.cuh"

using namespace etb;

namespace {

float f_of(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
uint32_t bits_of(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
bool pos_finite(uint32_t b) { const float f = f_of(b); return isfinite(f) && f > 0.0f; }
bool nonneg_finite(uint32_t b) { const float f = f_of(b); return isfinite(f) && f >= 0.0f; }

float pow_steps(float base, uint64_t e) {
  volatile float result = 1.0f;
  volatile float b = base;
  while (e != 0u) {
    if (e & 1u) result = result * b;
    e >>= 1u;
    if (e != 0u) b = b * b;
  }
  return result;
}

// Exact rational -> binary32 rounding (half to even) for the linear schedule
// ((D - e) 2^p + e r) / (D 2^p), o2_optimizer.c:589-611, over 32-bit limbs.
struct Big {
  uint32_t w[10] = {};
  void set(uint64_t v) { *this = Big(); w[0] = (uint32_t)v; w[1] = (uint32_t)(v >> 32); }
  int cmp(const Big& o) const {
    for (int i = 9; i >= 0; i--) if (w[i] != o.w[i]) return w[i] < o.w[i] ? -1 : 1;
    return 0;
  }
  bool zero() const { for (uint32_t x : w) if (x) return false; return true; }
  void shl(unsigned s) {
    Big r;
    const unsigned limb = s / 32, bit = s % 32;
    for (int i = 9; i >= (int)limb; i--) {
      const uint64_t v = (uint64_t)w[i - limb] << bit;
      r.w[i] |= (uint32_t)v;
      if (i + 1 < 10) r.w[i + 1] |= (uint32_t)(v >> 32);
    }
    *this = r;
  }
  void add(const Big& o) {
    uint64_t c = 0;
    for (int i = 0; i < 10; i++) { c += (uint64_t)w[i] + o.w[i]; w[i] = (uint32_t)c; c >>= 32; }
  }
  void sub(const Big& o) {
    int64_t c = 0;
    for (int i = 0; i < 10; i++) { int64_t v = (int64_t)w[i] - o.w[i] + c; w[i] = (uint32_t)v; c = v < 0 ? -1 : 0; }
  }
  void mul(uint32_t m) {
    uint64_t c = 0;
    for (int i = 0; i < 10; i++) { c += (uint64_t)w[i] * m; w[i] = (uint32_t)c; c >>= 32; }
  }
};

uint32_t round_f32(Big num, const Big& den) {
  if (num.zero()) return 0u;
  int e = 0;
  Big t = num;
  while (t.cmp(den) < 0) { t.shl(1); e--; }
  int keep = e < -126 ? 24 - (-126 - e) : 24;
  if (keep < 0) keep = 0;
  Big scaled = num;
  scaled.shl((unsigned)(keep - 1 - e));
  uint32_t q = 0;
  Big rem;
  for (int bit = 319; bit >= 0; bit--) {
    rem.shl(1);
    rem.w[0] |= (scaled.w[bit / 32] >> (bit % 32)) & 1u;
    q <<= 1;
    if (rem.cmp(den) >= 0) { rem.sub(den); q |= 1u; }
  }
  Big twice = rem;
  twice.shl(1);
  const int c = twice.cmp(den);
  if (c > 0 || (c == 0 && (q & 1u))) q++;
  if (e < -126) return q;
  if (q == (1u << 24)) { q >>= 1; e++; }
  return ((uint32_t)(e + 127) << 23) | (q - (1u << 23));
}

uint32_t schedule_factor(uint32_t kind, uint64_t warmup, uint64_t total, uint32_t min_bits,
                         uint64_t update) {
  if (kind == ET_B200_O2_SCHEDULE_CONSTANT) return 0x3f800000u;
  if (update > total) return min_bits;
  Big num, den;
  if (warmup > 0 && update <= warmup) {
    num.set(update);
    den.set(warmup);
    return round_f32(num, den);
  }
  const uint64_t elapsed = update - warmup, duration = total - warmup;
  const uint32_t exponent = (min_bits >> 23) & 0xffu, fraction = min_bits & 0x7fffffu;
  const unsigned p = exponent == 0u ? 149u : 150u - exponent;
  const uint32_t r = exponent == 0u ? fraction : (0x800000u | fraction);
  Big term;
  term.set(elapsed);
  term.mul(r);
  num.set(duration - elapsed);
  num.shl(p);
  num.add(term);
  den.set(duration);
  den.shl(p);
  return round_f32(num, den);
}

constexpr int kNormPartials = 592;

}  // namespace

struct et_b200_o2_optimizer {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<et_b200_o2_parameter_v1> params;
  std::vector<float*> m1, m2;
  uint32_t clip_kind = 0, clip_max_bits = 0, schedule_kind = 0, min_ratio_bits = 0;
  uint64_t warmup = 0, total = 0, updates = 0, elems = 0;
  AdamwTensor* d_table = nullptr;
  uint64_t* d_prefix = nullptr;
  double* d_partials = nullptr;
  double* d_sumsq = nullptr;
  int* d_status = nullptr;
  bool vec = false;  // every tensor 16-byte aligned with a count divisible by 4
  std::vector<AdamwTensor> table;
  std::vector<uint64_t> prefix;
};

extern "C" {

void et_b200_o2_optimizer_destroy_v1(et_b200_o2_optimizer** slot) {
  if (!slot || !*slot) return;
  et_b200_o2_optimizer* o = *slot;
  cudaSetDevice(o->device);
  if (o->stream) cudaStreamSynchronize(o->stream);
  for (float* p : o->m1) cudaFree(p);
  for (float* p : o->m2) cudaFree(p);
  cudaFree(o->d_table);
  cudaFree(o->d_prefix);
  cudaFree(o->d_partials);
  cudaFree(o->d_sumsq);
  cudaFree(o->d_status);
  if (o->stream) cudaStreamDestroy(o->stream);
  delete o;
  *slot = nullptr;
}

int32_t et_b200_o2_optimizer_create_v1(size_t count, const et_b200_o2_parameter_v1* params,
                                       uint32_t clip_kind, uint32_t clip_max_bits,
                                       uint32_t schedule_kind, uint64_t warmup_updates,
                                       uint64_t total_updates, uint32_t minimum_ratio_bits,
                                       et_b200_o2_optimizer** out, et_kernel_error* e) {
  const char* op = "optimizer-create";
  if (out == nullptr || (count > 0 && params == nullptr))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op, "parameters and output are required");
  *out = nullptr;
  if (count == 0 || count > 1365)  // ET_O2_MAX_PARAMETERS (o2_optimizer_internal.h:17)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_SHAPE, op, "parameter count must lie in [1, 1365]");
  const bool clip_ok = clip_kind == ET_B200_O2_CLIP_NONE ? clip_max_bits == 0u
                       : clip_kind == ET_B200_O2_CLIP_GLOBAL_L2 ? pos_finite(clip_max_bits) : false;
  bool sched_ok = schedule_kind == ET_B200_O2_SCHEDULE_CONSTANT
                      ? (warmup_updates == 0 && total_updates == 0 && minimum_ratio_bits == 0)
                      : schedule_kind == ET_B200_O2_SCHEDULE_LINEAR;
  if (schedule_kind == ET_B200_O2_SCHEDULE_LINEAR)
    sched_ok = total_updates > 0 && warmup_updates < total_updates &&
               nonneg_finite(minimum_ratio_bits) && f_of(minimum_ratio_bits) <= 1.0f;
  if (!clip_ok || !sched_ok)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op, "clip or schedule configuration is invalid");
  for (size_t i = 0; i < count; i++) {
    const et_b200_o2_parameter_v1& p = params[i];
    if (p.struct_size < sizeof(et_b200_o2_parameter_v1) || p.value == nullptr ||
        p.gradient == nullptr || p.count == 0)
      return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op, "parameter entry is incomplete");
    if (!nonneg_finite(p.learning_rate_bits) || !nonneg_finite(p.beta1_bits) ||
        f_of(p.beta1_bits) >= 1.0f || !nonneg_finite(p.beta2_bits) || f_of(p.beta2_bits) >= 1.0f ||
        !pos_finite(p.epsilon_bits) || !nonneg_finite(p.weight_decay_bits))
      return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op, "AdamW option is outside its domain");
  }
  et_b200_o2_optimizer* o = new et_b200_o2_optimizer();
  cudaGetDevice(&o->device);
  cudaStreamCreateWithFlags(&o->stream, cudaStreamNonBlocking);
  o->params.assign(params, params + count);
  o->clip_kind = clip_kind; o->clip_max_bits = clip_max_bits;
  o->schedule_kind = schedule_kind; o->warmup = warmup_updates; o->total = total_updates;
  o->min_ratio_bits = minimum_ratio_bits;
  bool ok = true;
  o->prefix.push_back(0);
  for (size_t i = 0; i < count; i++) {
    float *a = nullptr, *b = nullptr;
    ok = ok && cudaMalloc(&a, params[i].count * 4) == cudaSuccess;
    ok = ok && cudaMalloc(&b, params[i].count * 4) == cudaSuccess;
    o->m1.push_back(a);
    o->m2.push_back(b);
    if (ok) {
      cudaMemset(a, 0, params[i].count * 4);
      cudaMemset(b, 0, params[i].count * 4);
    }
    o->elems += params[i].count;
    o->prefix.push_back(o->elems);
  }
  ok = ok && cudaMalloc(&o->d_table, count * sizeof(AdamwTensor)) == cudaSuccess;
  ok = ok && cudaMalloc(&o->d_prefix, (count + 1) * sizeof(uint64_t)) == cudaSuccess;
  ok = ok && cudaMalloc(&o->d_partials, kNormPartials * sizeof(double)) == cudaSuccess;
  ok = ok && cudaMalloc(&o->d_sumsq, sizeof(double)) == cudaSuccess;
  ok = ok && cudaMalloc(&o->d_status, 3 * sizeof(int)) == cudaSuccess;
  if (!ok) {
    et_b200_o2_optimizer_destroy_v1(&o);
    return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_ALLOCATION_FAILED, op, "cannot allocate optimizer state");
  }
  cudaMemcpy(o->d_prefix, o->prefix.data(), o->prefix.size() * sizeof(uint64_t), cudaMemcpyHostToDevice);
  cudaMemset(o->d_status, 0, 3 * sizeof(int));
  o->table.resize(count);
  o->vec = true;
  for (size_t i = 0; i < count; i++)
    o->vec = o->vec && params[i].count % 4 == 0 && ((uintptr_t)params[i].value & 15) == 0 &&
             ((uintptr_t)params[i].gradient & 15) == 0;
  cudaDeviceSynchronize();
  *out = o;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_o2_optimizer_step_v1(et_b200_o2_optimizer* o, uint32_t weight_bits,
                                     uint32_t* norm_bits, et_kernel_error* e) {
  const char* op = "optimizer-step!";
  if (o == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op, "optimizer is null");
  if (!pos_finite(weight_bits))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op, "gradient accumulation metadata is inconsistent");
  cudaSetDevice(o->device);
  const uint64_t update = o->updates + 1;
  const uint32_t sched = schedule_factor(o->schedule_kind, o->warmup, o->total, o->min_ratio_bits, update);
  const float weight = f_of(weight_bits);
  for (size_t i = 0; i < o->params.size(); i++) {
    const et_b200_o2_parameter_v1& p = o->params[i];
    AdamwTensor& t = o->table[i];
    t.value = p.value; t.grad = p.gradient; t.exp_avg = o->m1[i]; t.exp_avg_sq = o->m2[i];
    t.count = p.count;
    volatile float one = 1.0f, b1 = f_of(p.beta1_bits), b2 = f_of(p.beta2_bits);
    t.beta1 = b1; t.beta2 = b2;
    t.one_minus_beta1 = one - b1;
    t.one_minus_beta2 = one - b2;
    t.bias1 = one - pow_steps(b1, update);
    t.bias2 = one - pow_steps(b2, update);
    volatile float lr = f_of(p.learning_rate_bits) * f_of(sched);
    volatile float lrwd = lr * f_of(p.weight_decay_bits);
    t.lr = lr;
    t.decay = one - lrwd;
    t.epsilon = f_of(p.epsilon_bits);
    t.envelope = adamw_envelope_ok(t) ? 1 : 0;
    if (!(t.bias1 > 0.0f) || !(t.bias2 > 0.0f) || !isfinite((float)lr))
      return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                       "bias correction or effective learning rate is invalid");
  }
  cudaMemcpyAsync(o->d_table, o->table.data(), o->table.size() * sizeof(AdamwTensor),
                  cudaMemcpyHostToDevice, o->stream);
  cudaMemsetAsync(o->d_status, 0, 3 * sizeof(int), o->stream);
  grad_sumsq(o->d_table, o->d_prefix, (int)o->table.size(), o->elems, weight, o->d_partials,
             kNormPartials, o->d_sumsq, o->d_status, o->stream);
  double sumsq = 0.0;
  int status[2] = {0, 0};
  cudaMemcpyAsync(&sumsq, o->d_sumsq, sizeof(double), cudaMemcpyDeviceToHost, o->stream);
  cudaMemcpyAsync(status, o->d_status, sizeof(status), cudaMemcpyDeviceToHost, o->stream);
  cudaError_t st = cudaStreamSynchronize(o->stream);
  if (st != cudaSuccess) return cuda_error(e, st, op);
  if (status[0])
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op, "gradient contains a nonfinite value");
  const float norm = (float)sqrt(sumsq);
  if (!isfinite(norm))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op, "gradient norm is unrepresentable");
  if (norm_bits) *norm_bits = bits_of(norm);
  float clip = 1.0f;
  if (o->clip_kind == ET_B200_O2_CLIP_GLOBAL_L2 && norm > f_of(o->clip_max_bits)) {
    volatile float mx = f_of(o->clip_max_bits);
    clip = mx / norm;
  }
  // all or nothing: the check pass computes every update without writing;
  // the apply pass writes only when the check set no status bit
  const AdamwControl ctl{nullptr, o->d_status, nullptr};
  adamw_check(o->d_table, o->d_prefix, (int)o->table.size(), o->elems, weight, clip, ctl, o->vec,
              o->stream);
  adamw_apply(o->d_table, o->d_prefix, (int)o->table.size(), o->elems, weight, clip, ctl, o->vec,
              o->stream);
  int after[3] = {0, 0, 0};
  cudaMemcpyAsync(after, o->d_status, sizeof(after), cudaMemcpyDeviceToHost, o->stream);
  st = cudaStreamSynchronize(o->stream);
  if (st == cudaSuccess) st = cudaGetLastError();
  if (st != cudaSuccess) return cuda_error(e, st, op);
  if (after[1] & kAdamwInputNonfinite)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "parameter, gradient, or moment is nonfinite");
  if (after[1] & kAdamwProducedNonfinite)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "AdamW produced a nonfinite value");
  o->updates = update;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_o2_optimizer_completed_updates_v1(const et_b200_o2_optimizer* o, uint64_t* updates) {
  if (!o || !updates) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  *updates = o->updates;
  return 0;
}

int32_t et_b200_o2_optimizer_moments_v1(et_b200_o2_optimizer* o, size_t index, float** exp_avg,
                                        float** exp_avg_sq) {
  if (!o || index >= o->params.size()) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  if (exp_avg) *exp_avg = o->m1[index];
  if (exp_avg_sq) *exp_avg_sq = o->m2[index];
  return 0;
}

// Host-side schedule factor (exposed for tests of the exact rational rounding).
uint32_t et_b200_o2_schedule_factor_v1(uint32_t kind, uint64_t warmup, uint64_t total,
                                       uint32_t minimum_ratio_bits, uint64_t update) {
  return schedule_factor(kind, warmup, total, minimum_ratio_bits, update);
}

}  // extern "C"
