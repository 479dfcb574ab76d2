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
#include <fcntl.h>
#include <math.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "eshkol_b200/o2_bridge.h"
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

// ===================================================================== O2 bridge
//
// The reference's Eshkol extension binds its optimizer through the
// et_o2_private_*_v1 externs of native/o2_wave2_extension.esk:4-29
// (implemented by native/o2_wave2_package_bridge.c:72-200 over the CPU O2
// optimizer and I2 parameters).  The same names and signatures here drive
// the device optimizer above, with et_b200_parameter objects (a device value
// and gradient plus the I2 accumulation metadata, native/f32_parameter_
// internal.h:55-67) in place of I2 parameters, so the extension binds
// unchanged.  Return values follow the bridge: O2 status codes
// (o2_optimizer_internal.h:19-30) for i64 results, NULL for a failed handle,
// and the last failure's category through et_o2_private_last_error_category_v1.

namespace {

enum : int64_t {
  kO2Ok = 0, kO2InvalidArgument = 1, kO2ShapeMismatch = 2, kO2InvalidState = 7,
  kO2Internal = 9
};

thread_local int64_t g_bridge_category = 0;
thread_local char g_bridge_message[192] = "";

int64_t bridge_fail(int64_t category, const char* message) {
  g_bridge_category = category;
  snprintf(g_bridge_message, sizeof(g_bridge_message), "%s", message);
  return category;
}
int64_t bridge_ok() {
  g_bridge_category = 0;
  g_bridge_message[0] = '\0';
  return kO2Ok;
}
// A device optimizer's K1-category failure as the O2 status the reference
// returns for the same condition.
int64_t bridge_from(int32_t k1, const et_kernel_error& e) {
  if (k1 == 0) return bridge_ok();
  const int64_t cat = k1 == ET_KERNEL_ERROR_INVALID_ARGUMENT ? kO2InvalidState
                      : k1 == ET_KERNEL_ERROR_SHAPE_MISMATCH ? kO2ShapeMismatch
                                                             : kO2Internal;
  return bridge_fail(cat, e.message);
}

struct BridgeEntry {
  et_b200_parameter* parameter = nullptr;
  const void* p1_handle = nullptr;
  uint32_t lr = 0, beta1 = 0, beta2 = 0, eps = 0, wd = 0;
  bool set = false;
};

}  // namespace

struct et_b200_parameter {
  float* value = nullptr;
  float* gradient = nullptr;
  size_t count = 0;
  bool present = false;       // a gradient has been accumulated
  uint64_t contributions = 0;
  uint32_t weight_bits = 0;   // normalisation weight (f32 bits)
  int device = 0;
};

struct et_b200_o2_builder {
  uint32_t clip_kind = 0, clip_bits = 0, schedule_kind = 0, min_ratio_bits = 0;
  uint64_t warmup = 0, total = 0;
  std::vector<BridgeEntry> entries;
};

struct et_b200_o2_bridge {
  et_b200_o2_optimizer* opt = nullptr;
  std::vector<BridgeEntry> entries;
};

struct et_b200_o2_state {
  uint32_t clip_kind = 0, clip_bits = 0, schedule_kind = 0, min_ratio_bits = 0;
  uint64_t warmup = 0, total = 0, completed = 0;
  std::vector<uint64_t> counts;
  std::vector<uint32_t> options;        // 5 per entry: lr, beta1, beta2, epsilon, weight decay
  std::vector<std::vector<uint32_t>> m, v;  // moment bits per entry
};

extern "C" {

int32_t et_b200_parameter_create_v1(float* value, float* gradient, size_t count,
                                    et_b200_parameter** out, et_kernel_error* e) {
  const char* op = "parameter-create";
  if (out == nullptr || value == nullptr || gradient == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "value, gradient and output are required");
  if (count == 0)
    return set_error(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                     "a parameter needs at least one element");
  et_b200_parameter* p = new et_b200_parameter();
  p->value = value;
  p->gradient = gradient;
  p->count = count;
  cudaGetDevice(&p->device);
  *out = p;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_parameter_set_gradient_v1(et_b200_parameter* p, uint64_t contributions,
                                          uint32_t weight_bits, et_kernel_error* e) {
  const char* op = "parameter-gradient";
  if (p == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "parameter is null");
  if (contributions == 0 || contributions > (uint64_t)INT64_MAX || !pos_finite(weight_bits))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op,
                     "gradient accumulation metadata is inconsistent");
  p->present = true;
  p->contributions = contributions;
  p->weight_bits = weight_bits;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_parameter_gradient_present_v1(const et_b200_parameter* p) {
  return p != nullptr && p->present ? 1 : 0;
}

void et_b200_parameter_destroy_v1(et_b200_parameter** p) {
  if (p == nullptr || *p == nullptr) return;
  delete *p;
  *p = nullptr;
}

int64_t et_o2_private_last_error_category_v1(void) { return g_bridge_category; }

const char* et_b200_o2_bridge_last_error_message_v1(void) { return g_bridge_message; }

void* et_o2_private_builder_create_v1(int64_t count, int64_t clip_kind, int64_t clip_bits,
                                      int64_t schedule_kind, int64_t warmup, int64_t total,
                                      int64_t minimum_ratio_bits) {
  if (count < 1 || count > 1365 || clip_kind < 0 || clip_bits < 0 || schedule_kind < 0 ||
      warmup < 0 || total < 0 || minimum_ratio_bits < 0 || clip_kind > UINT32_MAX ||
      clip_bits > UINT32_MAX || schedule_kind > UINT32_MAX || minimum_ratio_bits > UINT32_MAX) {
    bridge_fail(kO2InvalidArgument, "optimizer builder arguments are outside their domain");
    return nullptr;
  }
  const uint32_t ck = (uint32_t)clip_kind, cb = (uint32_t)clip_bits,
                 sk = (uint32_t)schedule_kind, mr = (uint32_t)minimum_ratio_bits;
  const bool clip_ok = ck == ET_B200_O2_CLIP_NONE ? cb == 0u
                       : ck == ET_B200_O2_CLIP_GLOBAL_L2 ? pos_finite(cb) : false;
  bool sched_ok = sk == ET_B200_O2_SCHEDULE_CONSTANT;
  if (sk == ET_B200_O2_SCHEDULE_LINEAR)
    sched_ok = total > 0 && warmup < total && nonneg_finite(mr) && f_of(mr) <= 1.0f;
  if (!clip_ok || !sched_ok) {
    bridge_fail(kO2InvalidArgument, "clip or schedule configuration is invalid");
    return nullptr;
  }
  et_b200_o2_builder* b = new et_b200_o2_builder();
  b->clip_kind = ck; b->clip_bits = cb; b->schedule_kind = sk; b->min_ratio_bits = mr;
  b->warmup = (uint64_t)warmup; b->total = (uint64_t)total;
  b->entries.resize((size_t)count);
  bridge_ok();
  return b;
}

int64_t et_o2_private_builder_set_v1(void* builder, int64_t index, void* parameter,
                                     void* p1_handle, int64_t learning_rate_bits,
                                     int64_t beta1_bits, int64_t beta2_bits,
                                     int64_t epsilon_bits, int64_t weight_decay_bits) {
  et_b200_o2_builder* b = static_cast<et_b200_o2_builder*>(builder);
  if (b == nullptr || parameter == nullptr || p1_handle == nullptr)
    return bridge_fail(kO2InvalidArgument, "builder, parameter and identity are required");
  if (index < 0 || (size_t)index >= b->entries.size())
    return bridge_fail(kO2InvalidArgument, "parameter index is outside the builder");
  const int64_t bits[5] = {learning_rate_bits, beta1_bits, beta2_bits, epsilon_bits,
                           weight_decay_bits};
  for (int64_t x : bits)
    if (x < 0 || x > UINT32_MAX) return bridge_fail(kO2InvalidArgument, "option bits are invalid");
  const uint32_t lr = (uint32_t)learning_rate_bits, b1 = (uint32_t)beta1_bits,
                 b2 = (uint32_t)beta2_bits, eps = (uint32_t)epsilon_bits,
                 wd = (uint32_t)weight_decay_bits;
  if (!nonneg_finite(lr) || !nonneg_finite(b1) || f_of(b1) >= 1.0f || !nonneg_finite(b2) ||
      f_of(b2) >= 1.0f || !pos_finite(eps) || !nonneg_finite(wd))
    return bridge_fail(kO2InvalidArgument, "AdamW option is outside its domain");
  for (size_t i = 0; i < b->entries.size(); i++)
    if (i != (size_t)index && b->entries[i].set && b->entries[i].parameter == parameter)
      return bridge_fail(kO2InvalidArgument, "parameter is bound twice");
  BridgeEntry& en = b->entries[(size_t)index];
  en.parameter = static_cast<et_b200_parameter*>(parameter);
  en.p1_handle = p1_handle;
  en.lr = lr; en.beta1 = b1; en.beta2 = b2; en.eps = eps; en.wd = wd;
  en.set = true;
  return bridge_ok();
}

void* et_o2_private_builder_finish_v1(void* builder) {
  et_b200_o2_builder* b = static_cast<et_b200_o2_builder*>(builder);
  if (b == nullptr) {
    bridge_fail(kO2InvalidArgument, "builder is null");
    return nullptr;
  }
  std::vector<et_b200_o2_parameter_v1> ps;
  for (const BridgeEntry& en : b->entries) {
    if (!en.set) {
      bridge_fail(kO2InvalidState, "every parameter slot must be bound before finish");
      return nullptr;
    }
    et_b200_o2_parameter_v1 p{};
    p.struct_size = sizeof(p);
    p.value = en.parameter->value;
    p.gradient = en.parameter->gradient;
    p.count = en.parameter->count;
    p.learning_rate_bits = en.lr; p.beta1_bits = en.beta1; p.beta2_bits = en.beta2;
    p.epsilon_bits = en.eps; p.weight_decay_bits = en.wd;
    ps.push_back(p);
  }
  et_kernel_error e{};
  et_b200_o2_optimizer* opt = nullptr;
  const int32_t rc = et_b200_o2_optimizer_create_v1(
      ps.size(), ps.data(), b->clip_kind, b->clip_bits, b->schedule_kind, b->warmup, b->total,
      b->min_ratio_bits, &opt, &e);
  if (rc != 0) {
    bridge_from(rc, e);
    return nullptr;
  }
  et_b200_o2_bridge* br = new et_b200_o2_bridge();
  br->opt = opt;
  br->entries = b->entries;
  delete b;  // the builder is consumed
  bridge_ok();
  return br;
}

int64_t et_o2_private_builder_abort_v1(void* builder) {
  if (builder == nullptr) return bridge_fail(kO2InvalidArgument, "builder is null");
  delete static_cast<et_b200_o2_builder*>(builder);
  return bridge_ok();
}

int64_t et_o2_private_optimizer_step_v1(void* optimizer) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  if (br == nullptr) return bridge_fail(kO2InvalidArgument, "optimizer is null");
  // o2_optimizer.c:1813-1856: every gradient present, one contribution count
  // and one normalisation weight across parameters
  uint64_t count = 0;
  uint32_t weight = 0;
  for (size_t i = 0; i < br->entries.size(); i++) {
    const et_b200_parameter* p = br->entries[i].parameter;
    if (!p->present)
      return bridge_fail(kO2InvalidState, "every bound parameter requires a present gradient");
    if (i > 0 && (p->contributions != count || p->weight_bits != weight))
      return bridge_fail(kO2InvalidState, "gradient accumulation metadata is inconsistent");
    count = p->contributions;
    weight = p->weight_bits;
  }
  et_kernel_error e{};
  return bridge_from(et_b200_o2_optimizer_step_v1(br->opt, weight, nullptr, &e), e);
}

int64_t et_o2_private_optimizer_zero_grad_v1(void* optimizer) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  if (br == nullptr) return bridge_fail(kO2InvalidArgument, "optimizer is null");
  cudaSetDevice(br->opt->device);
  for (BridgeEntry& en : br->entries) {
    const cudaError_t st =
        cudaMemsetAsync(en.parameter->gradient, 0, en.parameter->count * 4, br->opt->stream);
    if (st != cudaSuccess) return bridge_fail(kO2Internal, cudaGetErrorString(st));
  }
  const cudaError_t st = cudaStreamSynchronize(br->opt->stream);
  if (st != cudaSuccess) return bridge_fail(kO2Internal, cudaGetErrorString(st));
  for (BridgeEntry& en : br->entries) {
    en.parameter->present = false;
    en.parameter->contributions = 0;
    en.parameter->weight_bits = 0;
  }
  return bridge_ok();
}

int64_t et_o2_private_optimizer_require_absent_gradients_v1(void* optimizer) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  if (br == nullptr) return bridge_fail(kO2InvalidArgument, "optimizer is null");
  for (const BridgeEntry& en : br->entries)
    if (en.parameter->present)
      return bridge_fail(kO2InvalidState, "optimizer parameters still hold gradients");
  return bridge_ok();
}

int64_t et_o2_private_optimizer_completed_updates_v1(void* optimizer) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  if (br == nullptr) {
    bridge_fail(kO2InvalidArgument, "optimizer is null");
    return -1;
  }
  bridge_ok();
  return (int64_t)br->opt->updates;
}

int64_t et_o2_private_optimizer_schedule_factor_bits_v1(void* optimizer) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  if (br == nullptr) {
    bridge_fail(kO2InvalidArgument, "optimizer is null");
    return -1;
  }
  const et_b200_o2_optimizer* o = br->opt;
  bridge_ok();
  return (int64_t)schedule_factor(o->schedule_kind, o->warmup, o->total, o->min_ratio_bits,
                                  o->updates + 1);
}

// Snapshot: configuration, completed updates, per-parameter options and the
// moments' bits (copied to host memory).  Like the reference's
// et_o2_optimizer_state_snapshot_v1 (o2_optimizer.c:2052), it requires every
// gradient absent.
void* et_o2_private_optimizer_state_snapshot_v1(void* optimizer) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  if (br == nullptr) {
    bridge_fail(kO2InvalidArgument, "optimizer is null");
    return nullptr;
  }
  if (et_o2_private_optimizer_require_absent_gradients_v1(optimizer) != 0) return nullptr;
  const et_b200_o2_optimizer* o = br->opt;
  et_b200_o2_state* st = new et_b200_o2_state();
  st->clip_kind = o->clip_kind; st->clip_bits = o->clip_max_bits;
  st->schedule_kind = o->schedule_kind; st->min_ratio_bits = o->min_ratio_bits;
  st->warmup = o->warmup; st->total = o->total; st->completed = o->updates;
  cudaSetDevice(o->device);
  for (size_t i = 0; i < o->params.size(); i++) {
    const et_b200_o2_parameter_v1& p = o->params[i];
    st->counts.push_back(p.count);
    for (uint32_t x : {p.learning_rate_bits, p.beta1_bits, p.beta2_bits, p.epsilon_bits,
                       p.weight_decay_bits})
      st->options.push_back(x);
    st->m.emplace_back(p.count);
    st->v.emplace_back(p.count);
    cudaError_t err = cudaMemcpy(st->m.back().data(), o->m1[i], p.count * 4, cudaMemcpyDeviceToHost);
    if (err == cudaSuccess)
      err = cudaMemcpy(st->v.back().data(), o->m2[i], p.count * 4, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) {
      delete st;
      bridge_fail(kO2Internal, cudaGetErrorString(err));
      return nullptr;
    }
  }
  bridge_ok();
  return st;
}

// Load (o2_optimizer.c:2173): the state must describe this optimizer's
// configuration and parameters (counts, options); gradients absent.  All or
// nothing: nothing changes unless every check passes and every copy lands.
int64_t et_o2_private_optimizer_load_state_v1(void* optimizer, void* state) {
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(optimizer);
  const et_b200_o2_state* st = static_cast<const et_b200_o2_state*>(state);
  if (br == nullptr || st == nullptr)
    return bridge_fail(kO2InvalidArgument, "optimizer and state are required");
  if (int64_t r = et_o2_private_optimizer_require_absent_gradients_v1(optimizer)) return r;
  et_b200_o2_optimizer* o = br->opt;
  if (st->counts.size() != o->params.size())
    return bridge_fail(kO2ShapeMismatch, "optimizer state parameter count differs");
  if (st->clip_kind != o->clip_kind || st->clip_bits != o->clip_max_bits ||
      st->schedule_kind != o->schedule_kind || st->min_ratio_bits != o->min_ratio_bits ||
      st->warmup != o->warmup || st->total != o->total)
    return bridge_fail(kO2InvalidState, "optimizer state configuration differs");
  for (size_t i = 0; i < o->params.size(); i++) {
    const et_b200_o2_parameter_v1& p = o->params[i];
    const uint32_t* opt5 = st->options.data() + 5 * i;
    if (st->counts[i] != p.count)
      return bridge_fail(kO2ShapeMismatch, "optimizer state parameter shape differs");
    if (opt5[0] != p.learning_rate_bits || opt5[1] != p.beta1_bits || opt5[2] != p.beta2_bits ||
        opt5[3] != p.epsilon_bits || opt5[4] != p.weight_decay_bits)
      return bridge_fail(kO2InvalidState, "optimizer state options differ");
    for (size_t k = 0; k < p.count; k++)
      if (!isfinite(f_of(st->m[i][k])) || !nonneg_finite(st->v[i][k]))
        return bridge_fail(kO2InvalidState, "optimizer state moment is invalid");
  }
  cudaSetDevice(o->device);
  for (size_t i = 0; i < o->params.size(); i++) {
    cudaError_t err = cudaMemcpy(o->m1[i], st->m[i].data(), st->counts[i] * 4, cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
      err = cudaMemcpy(o->m2[i], st->v[i].data(), st->counts[i] * 4, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return bridge_fail(kO2Internal, cudaGetErrorString(err));
  }
  o->updates = st->completed;
  return bridge_ok();
}

int64_t et_o2_private_optimizer_state_release_v1(void* state) {
  if (state == nullptr) return bridge_fail(kO2InvalidArgument, "state is null");
  delete static_cast<et_b200_o2_state*>(state);
  return bridge_ok();
}

}  // extern "C"

namespace {
void put_bytes(std::vector<uint8_t>& out, const void* p, size_t n) {
  const uint8_t* b = static_cast<const uint8_t*>(p);
  out.insert(out.end(), b, b + n);
}
template <typename T> void put(std::vector<uint8_t>& out, T v) { put_bytes(out, &v, sizeof v); }
uint64_t fnv1a(const uint8_t* p, size_t n) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 0x100000001b3ull;
  return h;
}
const char kStateMagic[8] = {'E', 'T', 'B', '2', 'O', '2', 'S', 1};
bool write_all(int fd, const uint8_t* p, size_t n) {
  while (n > 0) {
    const ssize_t w = write(fd, p, n);
    if (w <= 0) return false;
    p += w;
    n -= (size_t)w;
  }
  return true;
}
}  // namespace

extern "C" {

int64_t et_b200_o2_state_write_v1(void* state, const char* path) {
  const et_b200_o2_state* st = static_cast<const et_b200_o2_state*>(state);
  if (st == nullptr || path == nullptr || path[0] == '\0')
    return bridge_fail(kO2InvalidArgument, "state and path are required");
  std::vector<uint8_t> out;
  put_bytes(out, kStateMagic, sizeof kStateMagic);
  put(out, st->clip_kind); put(out, st->clip_bits); put(out, st->schedule_kind);
  put(out, st->min_ratio_bits); put(out, st->warmup); put(out, st->total);
  put(out, st->completed); put(out, (uint64_t)st->counts.size());
  for (size_t i = 0; i < st->counts.size(); i++) {
    put(out, st->counts[i]);
    put_bytes(out, st->options.data() + 5 * i, 5 * sizeof(uint32_t));
    put_bytes(out, st->m[i].data(), st->counts[i] * 4);
    put_bytes(out, st->v[i].data(), st->counts[i] * 4);
  }
  put(out, fnv1a(out.data(), out.size()));
  // temporary file beside the target, flushed, renamed over it, directory flushed
  const std::string target(path);
  const std::string tmp = target + ".tmp." + std::to_string((long)getpid());
  const int fd = open(tmp.c_str(), O_WRONLY | O_CREAT | O_EXCL | O_CLOEXEC, 0644);
  if (fd < 0) return bridge_fail(kO2Internal, "cannot create the temporary state file");
  const bool ok = write_all(fd, out.data(), out.size()) && fsync(fd) == 0;
  close(fd);
  if (!ok || rename(tmp.c_str(), target.c_str()) != 0) {
    unlink(tmp.c_str());
    return bridge_fail(kO2Internal, "cannot write the state file");
  }
  const size_t slash = target.find_last_of('/');
  const std::string dir = slash == std::string::npos ? "." : (slash == 0 ? "/" : target.substr(0, slash));
  const int dfd = open(dir.c_str(), O_RDONLY | O_DIRECTORY | O_CLOEXEC);
  if (dfd >= 0) {
    fsync(dfd);
    close(dfd);
  }
  return bridge_ok();
}

void* et_b200_o2_state_read_v1(const char* path) {
  if (path == nullptr) {
    bridge_fail(kO2InvalidArgument, "path is required");
    return nullptr;
  }
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    bridge_fail(kO2InvalidArgument, "cannot open the state file");
    return nullptr;
  }
  std::vector<uint8_t> in;
  uint8_t buf[1 << 16];
  for (;;) {
    const ssize_t r = read(fd, buf, sizeof buf);
    if (r < 0) { close(fd); bridge_fail(kO2Internal, "cannot read the state file"); return nullptr; }
    if (r == 0) break;
    in.insert(in.end(), buf, buf + r);
  }
  close(fd);
  size_t at = 0;
  auto take = [&](void* dst, size_t n) {
    if (in.size() - at < n || at > in.size()) return false;
    memcpy(dst, in.data() + at, n);
    at += n;
    return true;
  };
  char magic[8];
  uint64_t n = 0, hash = 0;
  et_b200_o2_state* st = new et_b200_o2_state();
  bool ok = in.size() >= 16 && take(magic, 8) && memcmp(magic, kStateMagic, 8) == 0;
  if (ok) {
    memcpy(&hash, in.data() + in.size() - 8, 8);
    ok = fnv1a(in.data(), in.size() - 8) == hash;
  }
  ok = ok && take(&st->clip_kind, 4) && take(&st->clip_bits, 4) && take(&st->schedule_kind, 4) &&
       take(&st->min_ratio_bits, 4) && take(&st->warmup, 8) && take(&st->total, 8) &&
       take(&st->completed, 8) && take(&n, 8) && n <= 1365;
  for (uint64_t i = 0; ok && i < n; i++) {
    uint64_t c = 0;
    uint32_t o5[5];
    ok = take(&c, 8) && take(o5, sizeof o5) && c > 0 && c <= (in.size() - at) / 8;
    if (!ok) break;
    st->counts.push_back(c);
    st->options.insert(st->options.end(), o5, o5 + 5);
    st->m.emplace_back(c);
    st->v.emplace_back(c);
    ok = take(st->m.back().data(), c * 4) && take(st->v.back().data(), c * 4);
  }
  ok = ok && at + 8 == in.size();
  if (!ok) {
    delete st;
    bridge_fail(kO2InvalidState, "state file is truncated or corrupted");
    return nullptr;
  }
  bridge_ok();
  return st;
}

// Destroys a bridge optimizer (and its device moments); the parameters stay
// the caller's.  The reference's optimizer has no public destroy.
void et_b200_o2_bridge_destroy_v1(void** optimizer) {
  if (optimizer == nullptr || *optimizer == nullptr) return;
  et_b200_o2_bridge* br = static_cast<et_b200_o2_bridge*>(*optimizer);
  et_b200_o2_optimizer_destroy_v1(&br->opt);
  delete br;
  *optimizer = nullptr;
}

}  // extern "C"
