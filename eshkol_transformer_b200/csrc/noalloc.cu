// AdamW step that allocates nothing: et_b200_adamw_step_noalloc_v1.
//
// Some callers cannot let a library allocate device memory: hosts that hand
// all of HBM to their own allocator at start-up (a cudaMalloc from inside a
// library would fail, or land outside the host's accounting), and training
// loops that keep the device footprint fixed after start-up because cudaMalloc
// and cudaFree can synchronise the device in the middle of a step.  The O2
// optimizer object (et_b200_o2_optimizer_*) allocates its moments and its norm
// scratch when it is created; this entry point instead takes every tensor
// from the caller and keeps its only scratch -- the partial sums of the
// global gradient norm and three status words -- in the file-scope static
// device array below, sized for a stated maximum tensor length.  Like the
// reference's staged commit, the update is all or nothing: a check pass
// computes every element's update without writing, and the writing pass
// runs only when neither the gradient pass nor the check found a nonfinite
// value.
//
// Per element it applies the same separately rounded O2 arithmetic
// (native/o2_optimizer.c:1738-1756) as the multi-tensor kernel, so with the
// same gradient norm the updated parameters and moments are bit-identical to
// et_b200_o2_optimizer_step_v1's.
#include <math.h>

#include "ops.cuh"

using namespace etb;

namespace {

constexpr uint64_t kElementsPerPartial = 65536;
constexpr int kMaxPartials = 8192;
constexpr int kSumThreads = 256;

struct NoallocScratch {
  double partials[kMaxPartials];  // one f64 sum of squares per 65,536 elements
  double sumsq;
  float clip;
  uint32_t norm_bits;
  // [0] a gradient is nonfinite, [1] kAdamw* bits of the check pass, [2] the
  // norm of finite gradients is not representable in f32
  int status[3];
};

// The scratch every call shares (64 KiB + a few words per GPU, resident for
// the life of the process on every device that loads the library).  Host code
// must not use this name as an address: the device address comes from
// cudaGetSymbolAddress (scratch_address below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(NoallocScratch)];

__global__ void noalloc_clear(NoallocScratch* s) {
  s->status[0] = 0;
  s->status[1] = 0;
  s->status[2] = 0;
}

// Block b owns elements [b * 65536, (b + 1) * 65536): a fixed partition, so
// the norm is the same from call to call.
__global__ void __launch_bounds__(kSumThreads)
noalloc_sumsq(const float* __restrict__ grad, uint64_t count, float weight, NoallocScratch* s) {
  __shared__ double red[32];
  const uint64_t begin = (uint64_t)blockIdx.x * kElementsPerPartial;
  const uint64_t end = min(count, begin + kElementsPerPartial);
  double acc = 0.0;
  bool bad = false;
  for (uint64_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const float g = __fdiv_rn(grad[i], weight);
    bad |= !isfinite(g);
    acc += (double)g * (double)g;
  }
  const double total = block_reduce(acc, red, AddOp());
  if (threadIdx.x == 0) s->partials[blockIdx.x] = total;
  if (bad) atomicExch(&s->status[0], 1);
}

// Global norm, clip factor (clip_max / norm when the norm exceeds it).
__global__ void noalloc_finalize(NoallocScratch* s, int partials, float clip_max) {
  __shared__ double red[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < partials; i += blockDim.x) acc += s->partials[i];
  const double sumsq = block_reduce(acc, red, AddOp());
  if (threadIdx.x == 0) {
    s->sumsq = sumsq;
    const float norm = (float)sqrt(sumsq);
    s->norm_bits = __float_as_uint(norm);
    s->clip = (clip_max > 0.0f && norm > clip_max) ? __fdiv_rn(clip_max, norm) : 1.0f;
    if (!isfinite(norm) && s->status[0] == 0) s->status[2] = 1;
  }
}

struct Scalars {
  float beta1, beta2, one_minus_beta1, one_minus_beta2, bias1, bias2, lr, decay, epsilon, weight;
};

// One element of native/o2_optimizer.c:1738-1756 (each operation separately
// rounded, as the multi-tensor kernel does); with CHECK, *bad collects the
// kAdamw* bits for nonfinite inputs, intermediates and results.
template <bool CHECK>
__device__ __forceinline__ void noalloc_element(const Scalars& c, float clip, float p0, float g0,
                                                float m0, float v0, float& p, float& m, float& v,
                                                int& bad) {
  const float g = rn_mul(rn_div(g0, c.weight), clip);
  m = rn_add(rn_mul(c.beta1, m0), rn_mul(c.one_minus_beta1, g));
  v = rn_add(rn_mul(c.beta2, v0), rn_mul(c.one_minus_beta2, rn_mul(g, g)));
  const float mh = rn_div(m, c.bias1);
  const float vh = rn_div(v, c.bias2);
  const float den = rn_add(rn_sqrt(vh), c.epsilon);
  p = rn_sub(rn_mul(p0, c.decay), rn_div(rn_mul(c.lr, mh), den));
  if (CHECK) {
    if (!(isfinite(p0) && isfinite(g0) && isfinite(m0) && isfinite(v0)))
      bad |= kAdamwInputNonfinite;
    else if (!(isfinite(g) && isfinite(m) && isfinite(v) && isfinite(mh) && isfinite(vh) &&
               vh >= 0.0f && isfinite(den) && den > 0.0f && isfinite(p)))
      bad |= kAdamwProducedNonfinite;
  }
}

// APPLY = false: compute every update and record problems, write nothing.
// APPLY = true: write, unless the gradient pass or the check pass recorded a
// problem (then no block writes: the update is all or nothing).
template <bool APPLY>
__global__ void __launch_bounds__(256)
noalloc_adamw(float* __restrict__ value, const float* __restrict__ grad, float* __restrict__ m1,
              float* __restrict__ m2, uint64_t count, Scalars c, NoallocScratch* s) {
  if (s->status[0] || s->status[2] || (APPLY && s->status[1])) return;
  const float clip = s->clip;
  int bad = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float p, m, v;
    noalloc_element<!APPLY>(c, clip, value[i], grad[i], m1[i], m2[i], p, m, v, bad);
    if (APPLY) {
      value[i] = p;
      m1[i] = m;
      m2[i] = v;
    }
  }
  if (!APPLY && bad) atomicOr(&s->status[1], bad);
}

float f_of(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}

float pow_steps(float base, uint64_t e) {  // o2_optimizer.c:419-435
  volatile float result = 1.0f;
  volatile float b = base;
  while (e != 0u) {
    if (e & 1u) result = result * b;
    e >>= 1u;
    if (e != 0u) b = b * b;
  }
  return result;
}

// Device address of the scratch array, looked up once per device (with that
// device current) and kept in a fixed table, so later calls allocate nothing,
// not even on the host.
constexpr int kMaxDevices = 64;
NoallocScratch* g_addresses[kMaxDevices] = {};

int32_t scratch_address(NoallocScratch** out, et_kernel_error* e) {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return cuda_error(e, st, "adamw-step-noalloc");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED,
                     "adamw-step-noalloc", "device index beyond the scratch table");
  if (g_addresses[dev] == nullptr) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (st != cudaSuccess) return cuda_error(e, st, "adamw-step-noalloc");
    g_addresses[dev] = static_cast<NoallocScratch*>(p);
  }
  *out = g_addresses[dev];
  return 0;
}

}  // namespace

extern "C" int32_t et_b200_adamw_step_noalloc_v1(
    float* value, const float* gradient, float* exp_avg, float* exp_avg_sq, uint64_t count,
    uint32_t learning_rate_bits, uint32_t beta1_bits, uint32_t beta2_bits, uint32_t epsilon_bits,
    uint32_t weight_decay_bits, uint64_t update, uint32_t normalization_weight_bits,
    uint32_t clip_max_bits, void* stream, uint32_t* norm_bits, et_kernel_error* error) {
  const char* op = "adamw-step-noalloc";
  if (value == nullptr || gradient == nullptr || exp_avg == nullptr || exp_avg_sq == nullptr)
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "parameter, gradient and both moments are required");
  if (count == 0 || count > ET_B200_ADAMW_NOALLOC_MAX_ELEMENTS)
    return set_error(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_BUFFER_TOO_SMALL, op,
                     "count must lie in [1, 536870912]: the static norm scratch holds 8192 "
                     "partial sums of 65536 elements each");
  const float lr = f_of(learning_rate_bits), b1 = f_of(beta1_bits), b2 = f_of(beta2_bits);
  const float eps = f_of(epsilon_bits), wd = f_of(weight_decay_bits);
  const float weight = f_of(normalization_weight_bits), clip_max = f_of(clip_max_bits);
  if (!(isfinite(lr) && lr >= 0.0f) || !(isfinite(b1) && b1 >= 0.0f && b1 < 1.0f) ||
      !(isfinite(b2) && b2 >= 0.0f && b2 < 1.0f) || !(isfinite(eps) && eps > 0.0f) ||
      !(isfinite(wd) && wd >= 0.0f) || !(isfinite(weight) && weight > 0.0f) ||
      !(isfinite(clip_max) && clip_max >= 0.0f) || update == 0)
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op,
                     "AdamW option, normalisation weight, clip bound or update is invalid");
  NoallocScratch* s = nullptr;
  int32_t rc = scratch_address(&s, error);
  if (rc != 0) return rc;
  Scalars c;
  volatile float one = 1.0f, vb1 = b1, vb2 = b2;
  c.beta1 = vb1;
  c.beta2 = vb2;
  c.one_minus_beta1 = one - vb1;
  c.one_minus_beta2 = one - vb2;
  c.bias1 = one - pow_steps(b1, update);
  c.bias2 = one - pow_steps(b2, update);
  volatile float vlr = lr, lrwd = vlr * wd;
  c.lr = vlr;
  c.decay = one - lrwd;
  c.epsilon = eps;
  c.weight = weight;
  if (!(c.bias1 > 0.0f) || !(c.bias2 > 0.0f))
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "bias correction is invalid");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int partials = (int)((count + kElementsPerPartial - 1) / kElementsPerPartial);
  noalloc_clear<<<1, 1, 0, st>>>(s);
  noalloc_sumsq<<<partials, kSumThreads, 0, st>>>(gradient, count, weight, s);
  noalloc_finalize<<<1, 1024, 0, st>>>(s, partials, clip_max_bits ? clip_max : 0.0f);
  const uint64_t want = (count + 255) / 256;
  const unsigned blocks = (unsigned)(want < (uint64_t)sm_count() * 8 ? want : sm_count() * 8);
  noalloc_adamw<false><<<blocks, 256, 0, st>>>(value, gradient, exp_avg, exp_avg_sq, count, c, s);
  noalloc_adamw<true><<<blocks, 256, 0, st>>>(value, gradient, exp_avg, exp_avg_sq, count, c, s);
  count_launch(5);
  cudaError_t err = cudaGetLastError();  // a launch that failed to start
  if (err != cudaSuccess) return cuda_error(error, err, op);
  struct {
    uint32_t norm;
    int status[3];
  } out = {0, {0, 0, 0}};
  err = cudaMemcpyAsync(&out.norm, &s->norm_bits, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(out.status, s->status, sizeof(out.status), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err != cudaSuccess) return cuda_error(error, err, op);
  if (norm_bits) *norm_bits = out.norm;
  if (out.status[0])
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "gradient contains a nonfinite value; nothing was updated");
  if (out.status[2])
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "gradient norm is unrepresentable; nothing was updated");
  if (out.status[1] & kAdamwInputNonfinite)
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "parameter, gradient, or moment is nonfinite; nothing was updated");
  if (out.status[1] & kAdamwProducedNonfinite)
    return set_error(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "AdamW produced a nonfinite value; nothing was updated");
  if (error) memset(error, 0, sizeof(*error));
  return 0;
}
