// L2 indexed cross-entropy (fused softmax + target gather + upstream scale)
// and the O2 AdamW multi-tensor update.
//
// Cross-entropy follows native/indexed_cross_entropy.c:109-280: per row the
// maximum m, s = sum exp(x - m), loss = log(s) + (m - x[target]) and the
// gradient u (exp(x - m) / s - [j == target]), here exp(x - m) (1 / s).  One
// CTA owns one row: the first sweep forms per-thread online (max, sum) pairs
// from 128-bit loads (one maximum update per 4 values), a block reduction
// combines them, and the second sweep re-reads the row (an L2 hit: the rows in
// flight occupy far less than the 126 MB L2) and writes the gradient, so HBM
// sees one read and one write per logit.
//
// AdamW follows native/o2_optimizer.c:1738-1756 with every operation rounded
// separately (no contraction), which makes each updated parameter and moment
// bit-identical to the reference's SSE scalar sequence.
#include "ops.cuh"

namespace etb {

namespace {

constexpr int kCeThreads = 512;

__device__ __forceinline__ void online_push(float x, float& m, float& s) {
  if (x > m) {
    s = s * expf(m - x) + 1.0f;
    m = x;
  } else {
    s += expf(x - m);
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
  if (!target_ok && threadIdx.x == 0) atomicExch(status, 1);
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
        s = s * expf(m - mx);
        m = mx;
      }
      s += (expf(v.x - m) + expf(v.y - m)) + (expf(v.z - m) + expf(v.w - m));
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) online_push(__ldg(x + i), m, s);
  }
  // combine (m, s) pairs: first the maximum, then rescaled sums
  const float row_max = block_reduce(m, red_m, MaxOp());
  const float mine = (s == 0.0f) ? 0.0f : s * expf(m - row_max);
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
      r.x = u * (rn_mul(expf(v.x - row_max), inv_sum) - (j + 0 == target ? 1.0f : 0.0f));
      r.y = u * (rn_mul(expf(v.y - row_max), inv_sum) - (j + 1 == target ? 1.0f : 0.0f));
      r.z = u * (rn_mul(expf(v.z - row_max), inv_sum) - (j + 2 == target ? 1.0f : 0.0f));
      r.w = u * (rn_mul(expf(v.w - row_max), inv_sum) - (j + 3 == target ? 1.0f : 0.0f));
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
      float r = u * (rn_mul(expf(v - row_max), inv_sum) - (j == target ? 1.0f : 0.0f));
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
                                 float* out) {
  __shared__ double red[32];
  double acc = 0.0;
  for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) acc += (double)loss[i];
  const double total = block_reduce(acc, red, AddOp());
  if (threadIdx.x == 0) *out = (float)(total / (double)rows);
}

// ---- AdamW ----------------------------------------------------------------

constexpr int kAdamThreads = 256;
constexpr int kAdamPerThread = 8;
constexpr int64_t kAdamChunk = (int64_t)kAdamThreads * kAdamPerThread;
constexpr int kAdamBatch = 4;

__device__ __forceinline__ int find_tensor(const uint64_t* prefix, int count, uint64_t e) {
  int lo = 0, hi = count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= e) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kAdamThreads)
adamw_kernel(const AdamwTensor* __restrict__ tensors, const uint64_t* __restrict__ prefix,
             int tensor_count, uint64_t total, float weight, float clip, int* status,
             const float* skip) {
  const uint64_t begin = (uint64_t)blockIdx.x * kAdamChunk;
  if (begin >= total) return;
  if (skip != nullptr && *skip != 0.0f) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(status + 2, 1);
    return;
  }
  float amax = 0.0f;  // max |value| of the tensors that record it
  const uint64_t end = min(total, begin + (uint64_t)kAdamChunk);
  int t = find_tensor(prefix, tensor_count, begin);
  bool bad = false;
  uint64_t seg = begin;
  while (seg < end) {
    while (t + 1 < tensor_count && prefix[t + 1] <= seg) t++;
    const AdamwTensor T = tensors[t];
    const uint64_t seg_end = min(end, prefix[t] + T.count);
    const uint64_t base = prefix[t];
    // kAdamBatch elements per thread per round, their loads issued together
    for (uint64_t e0 = seg + threadIdx.x; e0 < seg_end; e0 += (uint64_t)kAdamBatch * blockDim.x) {
      float gr[kAdamBatch], m0[kAdamBatch], v0[kAdamBatch], p0[kAdamBatch];
#pragma unroll
      for (int u = 0; u < kAdamBatch; u++) {
        const uint64_t e = e0 + (uint64_t)u * blockDim.x;
        const uint64_t i = e - base;
        const bool in = e < seg_end;
        gr[u] = in ? T.grad[i] : 0.0f;
        m0[u] = in ? T.exp_avg[i] : 0.0f;
        v0[u] = in ? T.exp_avg_sq[i] : 0.0f;
        p0[u] = in ? T.value[i] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kAdamBatch; u++) {
        const uint64_t e = e0 + (uint64_t)u * blockDim.x;
        if (e >= seg_end) continue;
        const uint64_t i = e - base;
        const float g = rn_mul(rn_div(gr[u], weight), clip);
        const float m = rn_add(rn_mul(T.beta1, m0[u]), rn_mul(T.one_minus_beta1, g));
        const float v = rn_add(rn_mul(T.beta2, v0[u]), rn_mul(T.one_minus_beta2, rn_mul(g, g)));
        const float mh = rn_div(m, T.bias1);
        const float vh = rn_div(v, T.bias2);
        const float den = rn_add(rn_sqrt(vh), T.epsilon);
        const float p = rn_sub(rn_mul(p0[u], T.decay), rn_div(rn_mul(T.lr, mh), den));
        bad |= !(isfinite(g) && isfinite(m) && isfinite(v) && isfinite(p));
        T.value[i] = p;
        T.exp_avg[i] = m;
        T.exp_avg_sq[i] = v;
        if (T.value_sc.f16) {
          amax = fmaxf(amax, fabsf(p));
          f16_split(p * exp2_int(*T.value_sc.exp), reinterpret_cast<uint16_t*>(T.value_hi)[i],
                    reinterpret_cast<uint16_t*>(T.value_lo)[i]);
        } else if (T.value_hi != nullptr) {
          float h, l;
          tf32_split(p, h, l);
          T.value_hi[i] = h;
          T.value_lo[i] = l;
        }
      }
    }
    seg = seg_end;
  }
  // (a single max slot per launch: the first tensor's)
  if (tensors[0].value_sc.amax != nullptr) amax_record_warp(tensors[0].value_sc.amax, amax);
  if (bad) atomicExch(status + 1, 1);
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
  if (bad) atomicExch(status, 1);
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

void mean_loss(const float* loss, size_t rows, float* out, cudaStream_t stream) {
  mean_loss_kernel<<<1, 1024, 0, stream>>>(loss, (int64_t)rows, out);
  count_launch();
}

void adamw_multi(const AdamwTensor* tensors, const uint64_t* prefix, int tensor_count,
                 uint64_t total, float weight, float clip, int* status, cudaStream_t stream,
                 const float* skip) {
  if (total == 0) return;
  const unsigned blocks = (unsigned)((total + kAdamChunk - 1) / kAdamChunk);
  adamw_kernel<<<blocks, kAdamThreads, 0, stream>>>(tensors, prefix, tensor_count, total,
                                                    weight, clip, status, skip);
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
