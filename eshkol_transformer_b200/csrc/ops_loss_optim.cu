// L2 indexed cross-entropy (fused softmax + target gather + upstream scale)
// and the O2 AdamW multi-tensor update.
//
// Cross-entropy follows native/indexed_cross_entropy.c:109-280: per row the
// maximum m, s = sum exp(x - m), loss = log(s) + (m - x[target]) and the
// gradient u (exp(x - m) / s - [j == target]), here exp(x - m) (1 / s).  One
// CTA owns one row: the first sweep forms per-thread online (max, sum) pairs
// from 128-bit loads (one maximum update per 4 values), a block reduction
// combines them, and the second sweep re-reads the row (mostly from L2) and
// writes the gradient.
//
// The exponentials are the hardware-approximated __expf (relative error a
// few 1e-7 at the arguments that carry weight, up to about 1e-5 at
// exp(-80)): the row's sweeps are instruction-bound with the accurate expf,
// and the loss and gradient stay within the L2 tolerances (2e-6 absolute +
// 2e-5 relative against float64).
//
// AdamW follows native/o2_optimizer.c:1738-1756 with every operation rounded
// separately (no contraction), which makes each updated parameter and moment
// bit-identical to the reference's SSE scalar sequence.
#include <algorithm>

#include "ops.cuh"

namespace etb {

namespace {

// 256 threads per row, eight rows in flight per SM: measured faster than 128
// (3.98 ms), 512 (4.4-4.9 ms) and 1,024 (5.2 ms) per medium-LM step, and than
// variants that unroll the sweeps or keep part of the row in shared memory.
constexpr int kCeThreads = 256;

__device__ __forceinline__ void online_push(float x, float& m, float& s) {
  if (x > m) {
    s = s * __expf(m - x) + 1.0f;
    m = x;
  } else {
    s += __expf(x - m);
  }
}

__global__ void __launch_bounds__(kCeThreads)
ce_fused_kernel(const float* __restrict__ logits, float* dlogits,
                const int64_t* __restrict__ targets,
                const float* __restrict__ upstream, float upstream_scale,
                float* __restrict__ loss, int64_t V, int* status, float* __restrict__ dlo,
                OperandScale sc) {
  __shared__ float red_m[32];
  __shared__ float red_s[32];
  const int64_t row = blockIdx.x;
  const float* x = logits + row * V;
  const int64_t target = targets[row];
  const bool target_ok = target >= 0 && target < V;
  if (!target_ok && threadIdx.x == 0) atomicOr(status, 1);
  // The target logit is read before the block reductions: once they finish,
  // other threads overwrite the row with gradients when dlogits == logits.
  const float x_target = (threadIdx.x == 0 && target_ok) ? x[target] : 0.0f;

  float m = -INFINITY, s = 0.0f;
  const bool vec = ((V & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int64_t n4 = V >> 2;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
      // one running-maximum update per 4 values, then their 4 exponentials
      const float4 v = __ldg(x4 + i);
      const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      if (mx > m) {
        s = s * __expf(m - mx);
        m = mx;
      }
      s += (__expf(v.x - m) + __expf(v.y - m)) + (__expf(v.z - m) + __expf(v.w - m));
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) online_push(__ldg(x + i), m, s);
  }
  // combine (m, s) pairs: first the maximum, then rescaled sums
  const float row_max = block_reduce(m, red_m, MaxOp());
  const float mine = (s == 0.0f) ? 0.0f : s * __expf(m - row_max);
  const float row_sum = block_reduce(mine, red_s, AddOp());

  if (threadIdx.x == 0 && loss != nullptr) loss[row] = logf(row_sum) + (row_max - x_target);
  if (dlogits == nullptr) return;
  const float u = upstream != nullptr ? upstream[row] : upstream_scale;
  const float inv_sum = rn_div(1.0f, row_sum);  // softmax = exp(x - max) * (1 / sum)
  float* g = dlogits + row * V;
  // split-f16: dlogits / dlo hold binary16 hi / lo of the gradient 2^e
  const float s16 = sc.f16 ? exp2_int(*sc.exp) : 1.0f;
  uint16_t* gh = reinterpret_cast<uint16_t*>(dlogits) + row * V;
  uint16_t* gl = reinterpret_cast<uint16_t*>(dlo) + row * V;
  float amax = 0.0f;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* g4 = reinterpret_cast<float4*>(g);
    const int64_t n4 = V >> 2;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = x4[i];  // plain load: dlogits may alias logits
      float4 r;
      const int64_t j = i << 2;
      r.x = u * (rn_mul(__expf(v.x - row_max), inv_sum) - (j + 0 == target ? 1.0f : 0.0f));
      r.y = u * (rn_mul(__expf(v.y - row_max), inv_sum) - (j + 1 == target ? 1.0f : 0.0f));
      r.z = u * (rn_mul(__expf(v.z - row_max), inv_sum) - (j + 2 == target ? 1.0f : 0.0f));
      r.w = u * (rn_mul(__expf(v.w - row_max), inv_sum) - (j + 3 == target ? 1.0f : 0.0f));
      amax = abs_max4(amax, r);
      if (sc.f16) {
        f16_store4(gh, gl, j, r, s16);
        continue;
      }
      if (dlo != nullptr) {
        float4 l;
        tf32_split(r.x, r.x, l.x);
        tf32_split(r.y, r.y, l.y);
        tf32_split(r.z, r.z, l.z);
        tf32_split(r.w, r.w, l.w);
        reinterpret_cast<float4*>(dlo + row * V)[i] = l;
      }
      g4[i] = r;
    }
  } else {
    for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
      const float v = x[j];
      float r = u * (rn_mul(__expf(v - row_max), inv_sum) - (j == target ? 1.0f : 0.0f));
      amax = fmaxf(amax, fabsf(r));
      if (sc.f16) {
        f16_split(r * s16, gh[j], gl[j]);
        continue;
      }
      if (dlo != nullptr) tf32_split(r, r, dlo[row * V + j]);
      g[j] = r;
    }
  }
  if (sc.amax != nullptr) amax_record_warp(sc.amax, amax);
}

__global__ void mean_loss_kernel(const float* __restrict__ loss, int64_t rows,
                                 float* out, const uint8_t* __restrict__ mask) {
  __shared__ double red[32];
  double acc = 0.0, count = 0.0;
  for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) {
    if (mask == nullptr) {
      acc += (double)loss[i];
    } else if (mask[i] != 0) {
      acc += (double)loss[i];
      count += 1.0;
    }
  }
  const double total = block_reduce(acc, red, AddOp());
  const double n = mask == nullptr ? (double)rows : block_reduce(count, red, AddOp());
  if (threadIdx.x == 0) *out = n > 0.0 ? (float)(total / n) : 0.0f;
}

// One block: the numerator seed upstream[r] = mask[r] ? scale : 0 and the
// mask's sum (exact: an integer count below 2^24 per call).
__global__ void loss_mask_seed_kernel(const uint8_t* __restrict__ mask, int64_t rows, float scale,
                                      float* __restrict__ upstream, float* weight, int* status) {
  __shared__ double red[32];
  double count = 0.0;
  bool bad = false;
  for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) {
    const uint8_t m = mask[i];
    bad |= m > 1;
    upstream[i] = m != 0 ? scale : 0.0f;
    count += m != 0 ? 1.0 : 0.0;
  }
  const double total = block_reduce(count, red, AddOp());
  if (threadIdx.x == 0) *weight = (float)total;
  if (bad) atomicOr(status, 2);
}

// ---- AdamW ----------------------------------------------------------------
//
// Two passes per update.  adamw_check reads parameter, gradient and both
// moments (16 B per element) and computes each element's update exactly as
// adamw_apply will, writing nothing: any nonfinite input, intermediate or
// result sets a status bit (the reference checks the same quantities,
// o2_optimizer.c:1730-1768).  adamw_apply reads the same 16 B, writes value
// and both moments (12 B) and the weights' next operand pair, unless a
// status bit or the step's skip flag is set; then no block writes anything.
// With `vec` each thread moves four consecutive elements per 128-bit access
// and has the next group's loads in flight while it updates the current one.

constexpr int kAdamThreads = 256;
constexpr int kAdamScalarPerThread = 8;
constexpr int64_t kAdamChunk = (int64_t)kAdamThreads * kAdamScalarPerThread;

__device__ __forceinline__ int find_tensor(const uint64_t* prefix, int count, uint64_t e) {
  int lo = 0, hi = count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= e) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One element of native/o2_optimizer.c:1738-1756, each operation separately
// rounded.  With CHECK, *bad collects the kAdamw* bits.
// UNIT: weight and clip are 1, so g0 / weight * clip is g0 exactly.
template <bool CHECK, bool UNIT = false>
__device__ __forceinline__ void adamw_element(const AdamwTensor& T, float weight, float clip,
                                              float p0, float g0, float m0, float v0, float& p,
                                              float& m, float& v, int& bad) {
  const float g = UNIT ? g0 : rn_mul(rn_div(g0, weight), clip);
  m = rn_add(rn_mul(T.beta1, m0), rn_mul(T.one_minus_beta1, g));
  v = rn_add(rn_mul(T.beta2, v0), rn_mul(T.one_minus_beta2, rn_mul(g, g)));
  const float mh = rn_div(m, T.bias1);
  const float vh = rn_div(v, T.bias2);
  const float den = rn_add(rn_sqrt(vh), T.epsilon);
  p = rn_sub(rn_mul(p0, T.decay), rn_div(rn_mul(T.lr, mh), den));
  if (CHECK) {
    if (!(isfinite(p0) && isfinite(g0) && isfinite(m0) && isfinite(v0)))
      bad |= kAdamwInputNonfinite;
    else if (!(isfinite(g) && isfinite(m) && isfinite(v) && isfinite(mh) && isfinite(vh) &&
               vh >= 0.0f && isfinite(den) && den > 0.0f && isfinite(p)))
      bad |= kAdamwProducedNonfinite;
  }
}

// The check pass's finiteness envelope.  With the tensor's scalars admitted
// (adamw_envelope_ok: lr <= 2^60, 0 < epsilon <= 2^60, lr / epsilon <= 2^64,
// |decay| <= 2^10) and an element inside
//   p0, g0, m0, v0 finite, |g| <= 2^30, |m0| <= 2^30, 0 <= v0 <= 2^60,
//   |p0| <= 2^100   (g = g0 / weight * clip),
// every value of the update is finite: |m| <= 2^31 and 0 <= v <= 2^61
// (convex combinations, g^2 <= 2^60); both bias corrections are at least
// 1 - beta >= 2^-24 (beta^t <= beta < 1 in f32), so |m_hat| <= 2^55 and
// 0 <= v_hat <= 2^85; epsilon <= den <= 2^43 + 2^60; |lr m_hat / den| <=
// (lr / epsilon) 2^55 <= 2^119; |p decay| <= 2^110.  Such an element needs no
// arithmetic in the check; the others get the exact computation.
__device__ __forceinline__ bool adamw_in_envelope(float p0, float g, float m0, float v0) {
  return isfinite(p0) && isfinite(g) && isfinite(m0) && isfinite(v0) && fabsf(g) <= 0x1p30f &&
         fabsf(m0) <= 0x1p30f && v0 >= 0.0f && v0 <= 0x1p60f && fabsf(p0) <= 0x1p100f;
}

// True when this launch must not write (APPLY) or need not check: the step
// is void (skip flag, summed across ranks) or the check found a problem.
template <bool APPLY>
__device__ __forceinline__ bool adamw_void(const AdamwControl& ctl) {
  const bool skip = (ctl.skip != nullptr && *ctl.skip != 0.0f) || (APPLY && ctl.status[1] != 0);
  if (skip && APPLY && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(ctl.status + 2, 1);
  return skip;
}

template <bool APPLY>
__device__ __forceinline__ void adamw_finish(const AdamwTensor* tensors, const AdamwControl& ctl,
                                             float amax, int bad) {
  if (APPLY) {
    // (a single max slot per launch: the first tensor's)
    if (tensors[0].value_sc.amax != nullptr) amax_record_warp(tensors[0].value_sc.amax, amax);
    if (blockIdx.x == 0 && threadIdx.x == 0 && ctl.completed != nullptr) *ctl.completed += 1;
  } else if (bad) {
    atomicOr(ctl.status + 1, bad);
  }
}

// Vector path: groups of 4 elements never straddle two tensors (every count
// is a multiple of 4, so every prefix is too).  A grid-stride loop over the
// groups, each thread loading its next group while it updates the current
// one; the first group's loads are issued before the control words are read.
template <bool APPLY, bool UNIT>
__global__ void __launch_bounds__(kAdamThreads)
adamw_vec_kernel(const AdamwTensor* __restrict__ tensors, const uint64_t* __restrict__ prefix,
                 int tensor_count, uint64_t total, float weight, float clip, AdamwControl ctl) {
  const uint64_t groups = total >> 2;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t gi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int t = find_tensor(prefix, tensor_count, min(gi, groups - 1) * 4);
  float4 p0, g0, m0, v0;
  auto load = [&](uint64_t g, int& tt, float4& p, float4& gr, float4& m, float4& v) {
    const uint64_t e = g * 4;
    while (tt + 1 < tensor_count && prefix[tt + 1] <= e) tt++;
    const AdamwTensor& T = tensors[tt];
    const uint64_t i = e - prefix[tt];
    p = *reinterpret_cast<const float4*>(T.value + i);
    gr = __ldg(reinterpret_cast<const float4*>(T.grad + i));
    m = *reinterpret_cast<const float4*>(T.exp_avg + i);
    v = *reinterpret_cast<const float4*>(T.exp_avg_sq + i);
  };
  if (gi < groups) load(gi, t, p0, g0, m0, v0);
  if (adamw_void<APPLY>(ctl)) return;
  if (ctl.weight_dev != nullptr) weight = *ctl.weight_dev * ctl.weight_mul;
  if (UNIT) weight = clip = 1.0f;
  float amax = 0.0f;
  int bad = 0;
  while (gi < groups) {
    const uint64_t next = gi + stride;
    int tn = t;
    float4 p1, g1, m1, v1;
    if (next < groups) load(next, tn, p1, g1, m1, v1);
    const AdamwTensor& T = tensors[t];
    float4 p, m, v;
    if (!APPLY) {
      const bool inside =
          T.envelope &&
          adamw_in_envelope(p0.x, UNIT ? g0.x : rn_mul(rn_div(g0.x, weight), clip), m0.x, v0.x) &&
          adamw_in_envelope(p0.y, UNIT ? g0.y : rn_mul(rn_div(g0.y, weight), clip), m0.y, v0.y) &&
          adamw_in_envelope(p0.z, UNIT ? g0.z : rn_mul(rn_div(g0.z, weight), clip), m0.z, v0.z) &&
          adamw_in_envelope(p0.w, UNIT ? g0.w : rn_mul(rn_div(g0.w, weight), clip), m0.w, v0.w);
      if (!inside) {
        adamw_element<true, UNIT>(T, weight, clip, p0.x, g0.x, m0.x, v0.x, p.x, m.x, v.x, bad);
        adamw_element<true, UNIT>(T, weight, clip, p0.y, g0.y, m0.y, v0.y, p.y, m.y, v.y, bad);
        adamw_element<true, UNIT>(T, weight, clip, p0.z, g0.z, m0.z, v0.z, p.z, m.z, v.z, bad);
        adamw_element<true, UNIT>(T, weight, clip, p0.w, g0.w, m0.w, v0.w, p.w, m.w, v.w, bad);
      }
    } else {
      adamw_element<false, UNIT>(T, weight, clip, p0.x, g0.x, m0.x, v0.x, p.x, m.x, v.x, bad);
      adamw_element<false, UNIT>(T, weight, clip, p0.y, g0.y, m0.y, v0.y, p.y, m.y, v.y, bad);
      adamw_element<false, UNIT>(T, weight, clip, p0.z, g0.z, m0.z, v0.z, p.z, m.z, v.z, bad);
      adamw_element<false, UNIT>(T, weight, clip, p0.w, g0.w, m0.w, v0.w, p.w, m.w, v.w, bad);
    }
    if (APPLY) {
      const uint64_t i = gi * 4 - prefix[t];
      *reinterpret_cast<float4*>(T.value + i) = p;
      *reinterpret_cast<float4*>(T.exp_avg + i) = m;
      *reinterpret_cast<float4*>(T.exp_avg_sq + i) = v;
      if (T.value_sc.f16) {
        amax = abs_max4(amax, p);
        f16_store4(reinterpret_cast<uint16_t*>(T.value_hi),
                   reinterpret_cast<uint16_t*>(T.value_lo), (int64_t)i, p,
                   exp2_int(*T.value_sc.exp));
      } else if (T.value_hi != nullptr) {
        float4 h, l;
        tf32_split(p.x, h.x, l.x);
        tf32_split(p.y, h.y, l.y);
        tf32_split(p.z, h.z, l.z);
        tf32_split(p.w, h.w, l.w);
        *reinterpret_cast<float4*>(T.value_hi + i) = h;
        *reinterpret_cast<float4*>(T.value_lo + i) = l;
      }
    }
    gi = next;
    t = tn;
    p0 = p1; g0 = g1; m0 = m1; v0 = v1;
  }
  adamw_finish<APPLY>(tensors, ctl, amax, bad);
}

// Scalar path for tensors of any count and alignment.
template <bool APPLY>
__global__ void __launch_bounds__(kAdamThreads)
adamw_scalar_kernel(const AdamwTensor* __restrict__ tensors, const uint64_t* __restrict__ prefix,
                    int tensor_count, uint64_t total, float weight, float clip, AdamwControl ctl) {
  if (adamw_void<APPLY>(ctl)) return;
  if (ctl.weight_dev != nullptr) weight = *ctl.weight_dev * ctl.weight_mul;
  const uint64_t begin = (uint64_t)blockIdx.x * kAdamChunk;
  const uint64_t end = min(total, begin + (uint64_t)kAdamChunk);
  int t = find_tensor(prefix, tensor_count, begin);
  float amax = 0.0f;
  int bad = 0;
  for (uint64_t e = begin + threadIdx.x; e < end; e += blockDim.x) {
    while (t + 1 < tensor_count && prefix[t + 1] <= e) t++;
    const AdamwTensor& T = tensors[t];
    const uint64_t i = e - prefix[t];
    float p, m, v;
    adamw_element<!APPLY>(T, weight, clip, T.value[i], T.grad[i], T.exp_avg[i], T.exp_avg_sq[i],
                          p, m, v, bad);
    if (!APPLY) continue;
    T.value[i] = p;
    T.exp_avg[i] = m;
    T.exp_avg_sq[i] = v;
    if (T.value_sc.f16) {
      amax = fmaxf(amax, fabsf(p));
      f16_split(p * exp2_int(*T.value_sc.exp), reinterpret_cast<uint16_t*>(T.value_hi)[i],
                reinterpret_cast<uint16_t*>(T.value_lo)[i]);
    } else if (T.value_hi != nullptr) {
      tf32_split(p, T.value_hi[i], T.value_lo[i]);
    }
  }
  adamw_finish<APPLY>(tensors, ctl, amax, bad);
}

// base^e with one f32 rounding per multiply, the host's sequence
// (o2_optimizer.c:419-435).
__device__ float pow_steps_device(float base, uint64_t e) {
  float result = 1.0f, b = base;
  while (e != 0u) {
    if (e & 1u) result = __fmul_rn(result, b);
    e >>= 1u;
    if (e != 0u) b = __fmul_rn(b, b);
  }
  return result;
}

__global__ void fold_index_flag_kernel(const int* status, float* flag, float amount) {
  if (status[0] != 0) *flag += amount;
}

__global__ void adamw_prepare_kernel(AdamwTensor* tensors, const uint64_t* completed) {
  const uint64_t t = *completed + 1;
  tensors[0].bias1 = __fsub_rn(1.0f, pow_steps_device(tensors[0].beta1, t));
  tensors[0].bias2 = __fsub_rn(1.0f, pow_steps_device(tensors[0].beta2, t));
}

__global__ void __launch_bounds__(kAdamThreads)
grad_sumsq_kernel(const AdamwTensor* __restrict__ tensors, const uint64_t* __restrict__ prefix,
                  int tensor_count, uint64_t total, float weight, double* partials, int* status) {
  __shared__ double red[32];
  double acc = 0.0;
  bool bad = false;
  const uint64_t stride = (uint64_t)gridDim.x * kAdamChunk;
  for (uint64_t begin = (uint64_t)blockIdx.x * kAdamChunk; begin < total; begin += stride) {
    const uint64_t end = min(total, begin + (uint64_t)kAdamChunk);
    int t = find_tensor(prefix, tensor_count, begin);
    uint64_t seg = begin;
    while (seg < end) {
      while (t + 1 < tensor_count && prefix[t + 1] <= seg) t++;
      const AdamwTensor T = tensors[t];
      const uint64_t seg_end = min(end, prefix[t] + T.count);
      for (uint64_t e = seg + threadIdx.x; e < seg_end; e += blockDim.x) {
        const float g = rn_div(T.grad[e - prefix[t]], weight);
        bad |= !isfinite(g);
        acc += (double)g * (double)g;
      }
      seg = seg_end;
    }
  }
  const double total_block = block_reduce(acc, red, AddOp());
  if (threadIdx.x == 0) partials[blockIdx.x] = total_block;
  if (bad) atomicOr(status, 1);
}

__global__ void sum_partials_kernel(const double* partials, int count, double* out) {
  __shared__ double red[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < count; i += blockDim.x) acc += partials[i];
  const double t = block_reduce(acc, red, AddOp());
  if (threadIdx.x == 0) *out = t;
}

}  // namespace

void ce_fused(const float* logits, float* dlogits, const int64_t* targets,
              const float* upstream, float upstream_scale, float* loss,
              size_t rows, size_t V, int* status, cudaStream_t stream, float* dlogits_lo,
              OperandScale sc) {
  if (rows == 0) return;
  if (dlogits == nullptr) sc = OperandScale{};
  ce_fused_kernel<<<(unsigned)rows, kCeThreads, 0, stream>>>(
      logits, dlogits, targets, upstream, upstream_scale, loss, (int64_t)V, status,
      dlogits ? dlogits_lo : nullptr, sc);
  count_launch();
}

void mean_loss(const float* loss, size_t rows, float* out, cudaStream_t stream,
               const uint8_t* mask) {
  mean_loss_kernel<<<1, 1024, 0, stream>>>(loss, (int64_t)rows, out, mask);
  count_launch();
}

void loss_mask_seed(const uint8_t* mask, size_t rows, float scale, float* upstream, float* weight,
                    int* status, cudaStream_t stream) {
  loss_mask_seed_kernel<<<1, 1024, 0, stream>>>(mask, (int64_t)rows, scale, upstream, weight,
                                               status);
  count_launch();
}

namespace {
template <bool APPLY>
void adamw_pass(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                uint64_t total, float weight, float clip, AdamwControl ctl, bool vec,
                cudaStream_t stream) {
  if (total == 0) return;
  if (vec) {
    const unsigned blocks =
        (unsigned)std::min<uint64_t>(ceil_div(total / 4, kAdamThreads), (uint64_t)sm_count() * 8);
    if (weight == 1.0f && clip == 1.0f && ctl.weight_dev == nullptr)
      adamw_vec_kernel<APPLY, true><<<blocks, kAdamThreads, 0, stream>>>(
          tensors, prefix, tensor_count, total, weight, clip, ctl);
    else
      adamw_vec_kernel<APPLY, false><<<blocks, kAdamThreads, 0, stream>>>(
          tensors, prefix, tensor_count, total, weight, clip, ctl);
  } else {
    adamw_scalar_kernel<APPLY><<<ceil_div(total, kAdamChunk), kAdamThreads, 0, stream>>>(
        tensors, prefix, tensor_count, total, weight, clip, ctl);
  }
  count_launch();
}
}  // namespace

bool adamw_envelope_ok(const AdamwTensor& T) {
  const double lr = T.lr, eps = T.epsilon, decay = T.decay;
  return lr >= 0.0 && lr <= 0x1p60 && eps > 0.0 && eps <= 0x1p60 && lr / eps <= 0x1p64 &&
         std::fabs(decay) <= 0x1p10;
}

void adamw_check(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                 uint64_t total, float weight, float clip, AdamwControl ctl, bool vec,
                 cudaStream_t stream) {
  adamw_pass<false>(tensors, prefix, tensor_count, total, weight, clip, ctl, vec, stream);
}

void adamw_apply(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                 uint64_t total, float weight, float clip, AdamwControl ctl, bool vec,
                 cudaStream_t stream) {
  adamw_pass<true>(tensors, prefix, tensor_count, total, weight, clip, ctl, vec, stream);
}

void fold_index_flag(const int* status, float* flag, float amount, cudaStream_t stream) {
  fold_index_flag_kernel<<<1, 1, 0, stream>>>(status, flag, amount);
  count_launch();
}

void adamw_prepare(AdamwTensor* tensors, const uint64_t* completed, cudaStream_t stream) {
  adamw_prepare_kernel<<<1, 1, 0, stream>>>(tensors, completed);
  count_launch();
}

void grad_sumsq(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                uint64_t total, float weight, double* partials, int partial_count,
                double* out_sumsq, int* status, cudaStream_t stream) {
  grad_sumsq_kernel<<<partial_count, kAdamThreads, 0, stream>>>(tensors, prefix, tensor_count,
                                                               total, weight, partials, status);
  sum_partials_kernel<<<1, 1024, 0, stream>>>(partials, partial_count, out_sumsq);
  count_launch(2);
}

}  // namespace etb
