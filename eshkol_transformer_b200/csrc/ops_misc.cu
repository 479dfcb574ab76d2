// N2-family bandwidth kernels: LayerNorm, GELU/ReLU, residual, embedding,
// column sums (bias gradients), the TF32 residual split and standalone RoPE.
//
// Rounding points follow native/n2_primitives_provider.c:313-622 where the
// operation is elementwise (GELU, residual, RoPE rotation, embedding sums),
// so those outputs differ from the reference only through the device libm
// (erff/expf) and not through contraction.  Row and column reductions use a
// fixed-order tree, so every result is deterministic run to run.
#include <cub/cub.cuh>

#include "ops.cuh"

namespace etb {

namespace {

// ---- LayerNorm --------------------------------------------------------------

constexpr int kLnWarps = 4;

// One warp per row; the row is re-read from L1 for each of the three sweeps
// (mean, centred variance, output) so HBM sees one read and one write.
__global__ void __launch_bounds__(kLnWarps * 32)
ln_forward_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                  const float* __restrict__ beta, float epsilon, float* __restrict__ y,
                  float* __restrict__ mean_out, float* __restrict__ rstd_out,
                  int64_t rows, int64_t d, float* __restrict__ y_lo, OperandScale sc) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * d;
  const float dim = (float)d;
  float s = 0.0f;
  for (int64_t j = lane; j < d; j += 32) s += xr[j];
  s = warp_sum(s);
  const float mean = rn_div(s, dim);
  float v = 0.0f;
  for (int64_t j = lane; j < d; j += 32) {
    const float delta = rn_sub(xr[j], mean);
    v += rn_mul(delta, delta);
  }
  v = warp_sum(v);
  const float variance = rn_div(v, dim);
  const float rstd = rn_div(1.0f, rn_sqrt(rn_add(variance, epsilon)));
  float* yr = y + row * d;
  // split-f16: y and y_lo hold binary16 hi / lo of y 2^e
  const float s16 = sc.f16 ? exp2_int(*sc.exp) : 1.0f;
  uint16_t* yh = reinterpret_cast<uint16_t*>(y) + row * d;
  uint16_t* yl = reinterpret_cast<uint16_t*>(y_lo) + row * d;
  float amax = 0.0f;
  for (int64_t j = lane; j < d; j += 32) {
    const float normalized = rn_mul(rn_sub(xr[j], mean), rstd);
    float val = rn_add(rn_mul(normalized, gamma[j]), beta[j]);
    amax = fmaxf(amax, fabsf(val));
    if (sc.f16) {
      f16_split(val * s16, yh[j], yl[j]);
      continue;
    }
    if (y_lo != nullptr) tf32_split(val, val, y_lo[row * d + j]);
    yr[j] = val;
  }
  if (sc.amax != nullptr) amax_record_warp(sc.amax, amax);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

// Register-row variant for d = 128 NV (d <= 1024): one warp per row, lane l
// holding columns 4 l + 128 i (float4), so the row is read from HBM once with
// 128-bit loads and the mean / variance / output sweeps run from registers;
// outputs leave as float4 (f32, TF32 pair) or 8-byte binary16 quads.  Same
// per-element arithmetic as ln_forward_kernel; the row sums add in the lane
// order of this layout.
template <int NV>
__global__ void __launch_bounds__(kLnWarps * 32)
ln_forward_rows_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                       const float* __restrict__ beta, float epsilon, float* __restrict__ y,
                       float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t rows,
                       float* __restrict__ y_lo, OperandScale sc) {
  constexpr int D = 128 * NV;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * D);
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) v[i] = __ldg(xr + lane + 32 * i);
  const float dim = (float)D;
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    s += v[i].x; s += v[i].y; s += v[i].z; s += v[i].w;
  }
  s = warp_sum(s);
  const float mean = rn_div(s, dim);
  float var = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    float dlt;
    dlt = rn_sub(v[i].x, mean); var += rn_mul(dlt, dlt);
    dlt = rn_sub(v[i].y, mean); var += rn_mul(dlt, dlt);
    dlt = rn_sub(v[i].z, mean); var += rn_mul(dlt, dlt);
    dlt = rn_sub(v[i].w, mean); var += rn_mul(dlt, dlt);
  }
  var = warp_sum(var);
  const float variance = rn_div(var, dim);
  const float rstd = rn_div(1.0f, rn_sqrt(rn_add(variance, epsilon)));
  const float s16 = sc.f16 ? exp2_int(*sc.exp) : 1.0f;
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int c = lane + 32 * i;
    const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c);
    const float4 b = __ldg(reinterpret_cast<const float4*>(beta) + c);
    float4 o;
    o.x = rn_add(rn_mul(rn_mul(rn_sub(v[i].x, mean), rstd), g.x), b.x);
    o.y = rn_add(rn_mul(rn_mul(rn_sub(v[i].y, mean), rstd), g.y), b.y);
    o.z = rn_add(rn_mul(rn_mul(rn_sub(v[i].z, mean), rstd), g.z), b.z);
    o.w = rn_add(rn_mul(rn_mul(rn_sub(v[i].w, mean), rstd), g.w), b.w);
    amax = abs_max4(amax, o);
    const int64_t off = row * D + 4 * c;
    if (sc.f16) {
      f16_store4(reinterpret_cast<uint16_t*>(y), reinterpret_cast<uint16_t*>(y_lo), off, o, s16);
    } else if (y_lo != nullptr) {
      float4 l;
      tf32_split(o.x, o.x, l.x);
      tf32_split(o.y, o.y, l.y);
      tf32_split(o.z, o.z, l.z);
      tf32_split(o.w, o.w, l.w);
      *reinterpret_cast<float4*>(y + off) = o;
      *reinterpret_cast<float4*>(y_lo + off) = l;
    } else {
      *reinterpret_cast<float4*>(y + off) = o;
    }
  }
  if (sc.amax != nullptr) amax_record_warp(sc.amax, amax);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

int ln_backward_blocks(size_t rows) {
  const size_t want = (rows + kLnWarps - 1) / kLnWarps;
  const size_t cap = (size_t)sm_count() * 4;
  return (int)(want < cap ? want : cap);
}

// dx per row (n2_primitives_provider.c:490-512):
//   h = dy * gamma, n = (x - mean) rstd,
//   dx = (rstd / d) * ((d h - sum h) - n * sum(h n))
// and per-block column partials of dy * n (dgamma) and dy (dbeta), reduced
// over the block's warps in a fixed order.
__global__ void __launch_bounds__(kLnWarps * 32)
ln_backward_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                   const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                   const float* __restrict__ dy, float* __restrict__ dx, int accumulate,
                   float* __restrict__ partial, int64_t rows, int64_t d,
                   float* __restrict__ dx_hi, float* __restrict__ dx_lo) {
  extern __shared__ float sm[];  // [kLnWarps][2][d]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* pg = sm + (size_t)warp * 2 * d;
  float* pb = pg + d;
  for (int64_t j = lane; j < d; j += 32) { pg[j] = 0.0f; pb[j] = 0.0f; }
  const float dim = (float)d;
  const float inv_dim = rn_div(1.0f, dim);
  for (int64_t row = (int64_t)blockIdx.x * kLnWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kLnWarps) {
    const float* xr = x + row * d;
    const float* gr = dy + row * d;
    const float mean = mean_in[row], rstd = rstd_in[row];
    float sh = 0.0f, shn = 0.0f;
    for (int64_t j = lane; j < d; j += 32) {
      const float n = rn_mul(rn_sub(xr[j], mean), rstd);
      const float h = rn_mul(gr[j], gamma[j]);
      sh += h;
      shn += rn_mul(h, n);
      pg[j] += rn_mul(gr[j], n);
      pb[j] += gr[j];
    }
    sh = warp_sum(sh);
    shn = warp_sum(shn);
    const float factor = rn_mul(rstd, inv_dim);
    float* dr = dx + row * d;
    for (int64_t j = lane; j < d; j += 32) {
      const float n = rn_mul(rn_sub(xr[j], mean), rstd);
      const float h = rn_mul(gr[j], gamma[j]);
      const float val = rn_mul(factor, rn_sub(rn_sub(rn_mul(dim, h), sh), rn_mul(n, shn)));
      const float out = accumulate ? rn_add(dr[j], val) : val;
      dr[j] = out;
      if (dx_lo != nullptr) tf32_split(out, dx_hi[row * d + j], dx_lo[row * d + j]);
    }
  }
  __syncthreads();
  float* out = partial + (size_t)blockIdx.x * 2 * d;
  for (int64_t j = threadIdx.x; j < d; j += blockDim.x) {
    float g = 0.0f, b = 0.0f;
    for (int w = 0; w < kLnWarps; w++) {
      g += sm[(size_t)w * 2 * d + j];
      b += sm[(size_t)w * 2 * d + d + j];
    }
    out[j] = g;
    out[d + j] = b;
  }
}

// Register-resident variant for d = 128 NV (d <= 1024): each warp owns whole
// rows; lane l holds columns 4 l + 128 i (float4).  x, dy and (when
// accumulating) the incoming dx of a row are loaded together up front, so one
// memory latency covers the row; the column partials (dgamma, dbeta and, with
// dsum, the column sum of the final dx) accumulate in the warp's slice of
// shared memory, which keeps the registers low enough for two blocks per SM.
// Each block adds its warps' sums in warp order and writes one partial row
// per quantity; reduce_partials adds the blocks' rows.
constexpr int kLnbWarps = 8;

template <int NV>
__global__ void __launch_bounds__(kLnbWarps * 32, 2)
ln_backward_rows_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                        const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                        const float* __restrict__ dy, float* __restrict__ dx, int accumulate,
                        float* __restrict__ dx_hi, float* __restrict__ dx_lo,
                        float* __restrict__ partial, int with_sum, int64_t rows,
                        OperandScale sc) {
  constexpr int D = 128 * NV;
  const float s16 = sc.f16 ? exp2_int(*sc.exp) : 1.0f;
  float amax = 0.0f;
  extern __shared__ float4 lnb_acc[];  // [kLnbWarps][3][32 NV] partials, then gamma [32 NV]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4* acc = lnb_acc + warp * 3 * 32 * NV;
  float4* g = lnb_acc + kLnbWarps * 3 * 32 * NV;
  for (int i = threadIdx.x; i < 32 * NV; i += kLnbWarps * 32)
    g[i] = reinterpret_cast<const float4*>(gamma)[i];
#pragma unroll
  for (int i = 0; i < NV; i++)
    acc[lane + 32 * i] = acc[32 * NV + lane + 32 * i] = acc[64 * NV + lane + 32 * i] =
        make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  const float dim = (float)D;
  const float inv_dim = rn_div(1.0f, dim);
  for (int64_t row = (int64_t)blockIdx.x * kLnbWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kLnbWarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * D);
    const float4* gr = reinterpret_cast<const float4*>(dy + row * D);
    float4* dr = reinterpret_cast<float4*>(dx + row * D);
    float4 xv[NV], gv[NV], dv[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
      xv[i] = xr[lane + 32 * i];
      gv[i] = gr[lane + 32 * i];
      dv[i] = accumulate ? dr[lane + 32 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float mean = mean_in[row], rstd = rstd_in[row];
    float sh = 0.0f, shn = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      float4 ag = acc[lane + 32 * i], ab = acc[32 * NV + lane + 32 * i];
      const float4 gi = g[lane + 32 * i];
#define LNB_ACC(c)                                                  \
  {                                                                 \
    const float n = rn_mul(rn_sub(xv[i].c, mean), rstd);            \
    const float h = rn_mul(gv[i].c, gi.c);                          \
    sh += h;                                                        \
    shn += rn_mul(h, n);                                            \
    ag.c += rn_mul(gv[i].c, n);                                     \
    ab.c += gv[i].c;                                                \
  }
      LNB_ACC(x) LNB_ACC(y) LNB_ACC(z) LNB_ACC(w)
#undef LNB_ACC
      acc[lane + 32 * i] = ag;
      acc[32 * NV + lane + 32 * i] = ab;
    }
    sh = warp_sum(sh);
    shn = warp_sum(shn);
    const float factor = rn_mul(rstd, inv_dim);
#pragma unroll
    for (int i = 0; i < NV; i++) {
      float4 out;
      const float4 gi = g[lane + 32 * i];
#define LNB_OUT(c)                                                                         \
  {                                                                                        \
    const float n = rn_mul(rn_sub(xv[i].c, mean), rstd);                                   \
    const float h = rn_mul(gv[i].c, gi.c);                                                 \
    out.c = rn_mul(factor, rn_sub(rn_sub(rn_mul(dim, h), sh), rn_mul(n, shn)));            \
  }
      LNB_OUT(x) LNB_OUT(y) LNB_OUT(z) LNB_OUT(w)
#undef LNB_OUT
      if (accumulate) {
        out.x = rn_add(dv[i].x, out.x); out.y = rn_add(dv[i].y, out.y);
        out.z = rn_add(dv[i].z, out.z); out.w = rn_add(dv[i].w, out.w);
      }
      dr[lane + 32 * i] = out;
      if (with_sum) {
        float4 as = acc[64 * NV + lane + 32 * i];
        as.x += out.x; as.y += out.y; as.z += out.z; as.w += out.w;
        acc[64 * NV + lane + 32 * i] = as;
      }
      amax = abs_max4(amax, out);
      if (sc.f16) {  // dx_hi / dx_lo hold binary16 hi / lo of dx 2^e
        f16_store4(reinterpret_cast<uint16_t*>(dx_hi), reinterpret_cast<uint16_t*>(dx_lo),
                   row * D + 4 * (lane + 32 * i), out, s16);
      } else if (dx_lo != nullptr) {
        float4 h4, l4;
        tf32_split(out.x, h4.x, l4.x);
        tf32_split(out.y, h4.y, l4.y);
        tf32_split(out.z, h4.z, l4.z);
        tf32_split(out.w, h4.w, l4.w);
        reinterpret_cast<float4*>(dx_hi + row * D)[lane + 32 * i] = h4;
        reinterpret_cast<float4*>(dx_lo + row * D)[lane + 32 * i] = l4;
      }
    }
  }
  if (sc.amax != nullptr) amax_record_warp(sc.amax, amax);
  // the block's partial row per quantity: the warps' sums added in warp order
  __syncthreads();
  const int nq = with_sum ? 3 : 2;
  float4* out = reinterpret_cast<float4*>(partial + (int64_t)blockIdx.x * nq * D);
  for (int idx = threadIdx.x; idx < nq * 32 * NV; idx += kLnbWarps * 32) {
    float4 t = lnb_acc[idx];
#pragma unroll
    for (int w = 1; w < kLnbWarps; w++) {
      const float4 o = lnb_acc[w * 3 * 32 * NV + idx];
      t.x += o.x; t.y += o.y; t.z += o.z; t.w += o.w;
    }
    out[idx] = t;
  }
}

int ln_backward_rows_blocks(size_t rows) {
  const size_t want = (rows + kLnbWarps - 1) / kLnbWarps;
  const size_t cap = (size_t)sm_count() * 4;
  return (int)(want < cap ? want : cap);
}

// ---- GELU backward with column sums ----------------------------------------------

constexpr int kGcRows = 512;  // rows per block

// Block (c, r): columns [128 c, 128 c + 128) (float4 per lane) of rows
// [kGcRows r, ...), one row per warp at a time; each warp writes its column
// partial row of dx.
__global__ void __launch_bounds__(256)
gelu_backward_colsum_kernel(const float* __restrict__ x, const float* dy,
                            float* dx, float* __restrict__ dx_lo,
                            float* __restrict__ partial, int64_t rows, int64_t n) {
  const float inv_sqrt_2 = 0x1.6a09e6p-1f, inv_sqrt_2pi = 0x1.988454p-2f;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 128 + 4 * lane;
  const int64_t r0 = (int64_t)blockIdx.y * kGcRows, r1 = min(rows, r0 + kGcRows);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col < n) {
    for (int64_t r = r0 + warp; r < r1; r += 8) {
      const int64_t i = r * n + col;
      const float4 v = *reinterpret_cast<const float4*>(x + i);
      const float4 g = *reinterpret_cast<const float4*>(dy + i);
      float4 o, lo;
#define GC_ONE(c)                                                                       \
  {                                                                                     \
    const float cdf = rn_mul(0.5f, rn_add(1.0f, erff(rn_mul(v.c, inv_sqrt_2))));        \
    const float density = rn_mul(expf(-rn_mul(0.5f, rn_mul(v.c, v.c))), inv_sqrt_2pi); \
    const float slope = rn_add(cdf, rn_mul(v.c, density));                              \
    o.c = rn_mul(g.c, slope);                                                           \
    acc.c += o.c;                                                                       \
    if (dx_lo != nullptr) tf32_split(o.c, o.c, lo.c);                                   \
  }
      GC_ONE(x) GC_ONE(y) GC_ONE(z) GC_ONE(w)
#undef GC_ONE
      *reinterpret_cast<float4*>(dx + i) = o;
      if (dx_lo != nullptr) *reinterpret_cast<float4*>(dx_lo + i) = lo;
    }
    *reinterpret_cast<float4*>(partial + ((int64_t)blockIdx.y * 8 + warp) * n + col) = acc;
  }
}

// Column sums of `count` partial rows: quantity q = blockIdx.y reads columns
// [q width, q width + width) of each row (row stride `stride`) and writes
// out[q].  A block covers 32 columns; warp w sums rows w, w + 8, ... (each
// warp load is one 128-byte row segment), then the 8 warp sums are added in
// warp order, so the result does not depend on timing.
struct PartialOuts {
  float* out[3];
};
__global__ void __launch_bounds__(256)
reduce_partials_kernel(const float* __restrict__ partial, int count, int64_t width,
                       int64_t stride, PartialOuts outs) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int q = blockIdx.y;
  const int64_t j = (int64_t)blockIdx.x * 32 + tx;
  float s = 0.0f;
  if (j < width) {
    const float* col = partial + (int64_t)q * width + j;
#pragma unroll 4
    for (int b = ty; b < count; b += 8) s += col[(int64_t)b * stride];
  }
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && j < width) {
    float t = red[0][tx];
#pragma unroll
    for (int w = 1; w < 8; w++) t += red[w][tx];
    float* o = q == 0 ? outs.out[0] : (q == 1 ? outs.out[1] : outs.out[2]);
    o[j] = t;
  }
}


// ---- activations -------------------------------------------------------------

// Exact-erf GELU with the reference's binary32 constants
// (n2_primitives_provider.c:545-583).
__global__ void gelu_forward_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                                    float* __restrict__ y_lo) {
  const float inv_sqrt_2 = 0x1.6a09e6p-1f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float e = erff(rn_mul(v, inv_sqrt_2));
    float r = rn_mul(rn_mul(0.5f, v), rn_add(1.0f, e));
    if (y_lo != nullptr) tf32_split(r, r, y_lo[i]);
    y[i] = r;
  }
}

__global__ void gelu_backward_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                     float* __restrict__ dx, int64_t n, float* __restrict__ dx_lo) {
  const float inv_sqrt_2 = 0x1.6a09e6p-1f, inv_sqrt_2pi = 0x1.988454p-2f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float cdf = rn_mul(0.5f, rn_add(1.0f, erff(rn_mul(v, inv_sqrt_2))));
    const float density = rn_mul(expf(-rn_mul(0.5f, rn_mul(v, v))), inv_sqrt_2pi);
    const float slope = rn_add(cdf, rn_mul(v, density));
    float r = rn_mul(dy[i], slope);
    if (dx_lo != nullptr) tf32_split(r, r, dx_lo[i]);
    dx[i] = r;
  }
}

__global__ void relu_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                            float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    out[i] = v > 0.0f ? (dy ? dy[i] : v) : 0.0f;
  }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = rn_add(a[i], b[i]);
}

__global__ void copy_kernel(const float* __restrict__ a, float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = a[i];
}

__global__ void split_tf32_kernel(const float* x, float* hi_out, float* __restrict__ lo,
                                  int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    // hi: v rounded to the nearest TF32 value (10 explicit mantissa bits,
    // ties away from zero), so |lo| <= 2^-11 |v|; the add cannot carry past
    // the exponent except into the next binade, which is still exact.
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7f800000u) != 0x7f800000u) {
      const uint32_t r = (b + 0x1000u) & 0xffffe000u;
      b = ((r & 0x7f800000u) == 0x7f800000u) ? (b & 0xffffe000u) : r;  // no overflow to inf
    }
    const float hi = __uint_as_float(b);
    lo[i] = v - hi;  // exact: |v - hi| fits in the low mantissa bits
    hi_out[i] = hi;
  }
}

// max |x| over n values, one atomicMax per warp
__global__ void abs_max_kernel(const float* __restrict__ x, int64_t n, unsigned* amax) {
  float m = 0.0f;
  const int64_t n4 = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) ? n >> 2 : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t i = first; i < n4; i += stride)
    m = abs_max4(m, __ldg(reinterpret_cast<const float4*>(x) + i));
  for (int64_t i = 4 * n4 + first; i < n; i += stride) m = fmaxf(m, fabsf(x[i]));
  amax_record_warp(amax, m);
}

// exp[i] from amax[i] = f 2^k (f in [0.5, 1)): e = target - k, so that
// amax 2^e lies in [2^(target-1), 2^target); clamped to [-60, 60].  A zero or
// nonfinite amax keeps exp[i]: after a step whose operands overflowed, the
// overflowing tensors' maxima (taken before scaling) are finite and rescale
// them, while tensors computed from the overflowed values keep the scale of
// the last good step.  amax[i] is cleared when reset.
__global__ void scale_from_amax_kernel(unsigned* amax, int* exp, int count, int target,
                                       int reset) {
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const float a = __uint_as_float(amax[i]);
    if (isfinite(a) && a > 0.0f) {
      int k;
      frexpf(a, &k);
      exp[i] = max(-60, min(60, target - k));
    }
    if (reset) amax[i] = 0u;
  }
}

// binary16 operand pair of v = x (+ xlo) scaled by 2^(*exp); max |v| to amax
__global__ void split_f16_kernel(const float* __restrict__ x, const float* __restrict__ xlo,
                                 int64_t n4, uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                                 const int* __restrict__ exp, unsigned* amax) {
  const float s = exp2_int(*exp);
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    if (xlo != nullptr) {
      const float4 l = __ldg(reinterpret_cast<const float4*>(xlo) + i);
      v.x += l.x; v.y += l.y; v.z += l.z; v.w += l.w;
    }
    m = abs_max4(m, v);
    f16_store4(hi, lo, 4 * i, v, s);
  }
  amax_record_warp(amax, m);
}
__global__ void split_f16_tail_kernel(const float* x, const float* xlo, int64_t begin, int64_t n,
                                      uint16_t* hi, uint16_t* lo, const int* exp, unsigned* amax) {
  const float s = exp2_int(*exp);
  float m = 0.0f;
  for (int64_t i = begin + threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i] + (xlo != nullptr ? xlo[i] : 0.0f);
    m = fmaxf(m, fabsf(v));
    f16_split(v * s, hi[i], lo[i]);
  }
  amax_record_warp(amax, m);
}

// flag[0] = 1 when any slot's amax 2^exp reached binary16's largest finite
// value 65504 (or is NaN), else 0; amax[reset_slot] is then cleared.
__global__ void operand_range_kernel(unsigned* amax, const int* exp, int count, int reset_slot,
                                     float* flag) {
  bool bad = false;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const float v = __uint_as_float(amax[i]) * exp2_int(exp[i]);
    bad |= !(v < 65504.0f);
  }
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    if (bad) flag[0] += 1.0f;  // (the flag may already hold other step-void marks)
    if (reset_slot >= 0) amax[reset_slot] = 0u;
  }
}

__global__ void finite_kernel(const float* __restrict__ x, int64_t n, int* flag) {
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    bad |= !isfinite(x[i]);
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicExch(flag, 1);
}

// ---- embedding --------------------------------------------------------------

__global__ void embedding_forward_kernel(const int64_t* __restrict__ ids, const float* __restrict__ w,
                                         float* __restrict__ y, int64_t rows, int64_t V, int64_t d,
                                         int* status) {
  const int64_t row = blockIdx.x;
  const int64_t id = ids[row];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) atomicOr(status, 1);
    return;
  }
  const float* src = w + id * d;
  float* dst = y + row * d;
  for (int64_t j = threadIdx.x; j < d; j += blockDim.x) dst[j] = src[j];
}

__global__ void ids_to_keys_kernel(const int64_t* __restrict__ ids, uint32_t* __restrict__ keys,
                                   uint32_t* __restrict__ vals, int64_t rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) {
    keys[i] = (uint32_t)ids[i];
    vals[i] = (uint32_t)i;
  }
}

// One block per vocabulary row: locate its run in the sorted keys, then sum
// the matching token rows in ascending row order starting from +0 and add it
// to the base (the tied head gradient), exactly as the reference orders it.
__global__ void embedding_backward_kernel(const uint32_t* __restrict__ keys,
                                          const uint32_t* __restrict__ rows_sorted,
                                          const float* __restrict__ dy,
                                          const float* __restrict__ base, float* __restrict__ dw,
                                          int64_t rows, int64_t d) {
  const uint32_t v = blockIdx.x;
  __shared__ int64_t range[2];
  if (threadIdx.x == 0) {
    int64_t lo = 0, hi = rows;
    while (lo < hi) {  // first key >= v
      const int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < v) lo = mid + 1; else hi = mid;
    }
    int64_t lo2 = lo, hi2 = rows;
    while (lo2 < hi2) {  // first key > v
      const int64_t mid = (lo2 + hi2) >> 1;
      if (keys[mid] <= v) lo2 = mid + 1; else hi2 = mid;
    }
    range[0] = lo;
    range[1] = lo2;
  }
  __syncthreads();
  const int64_t a = range[0], b = range[1];
  for (int64_t j = threadIdx.x; j < d; j += blockDim.x) {
    float acc = 0.0f;
    for (int64_t p = a; p < b; p++) acc = rn_add(acc, dy[(int64_t)rows_sorted[p] * d + j]);
    dw[(int64_t)v * d + j] = base ? rn_add(base[(int64_t)v * d + j], acc) : acc;
  }
}

// ---- column sums ------------------------------------------------------------

constexpr int kColRowsChunk = 256;

__global__ void colsum_partial_kernel(const float* __restrict__ dy, const float* __restrict__ dy_lo,
                                      float* __restrict__ partial, int64_t rows, int64_t n) {
  __shared__ float sm[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const int64_t r0 = (int64_t)blockIdx.y * kColRowsChunk;
  const int64_t r1 = min(rows, r0 + kColRowsChunk);
  float acc = 0.0f;
  if (col < n)
    for (int64_t r = r0 + warp; r < r1; r += 8)
      acc += dy_lo != nullptr ? dy[r * n + col] + dy_lo[r * n + col] : dy[r * n + col];
  sm[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && col < n) {
    float s = 0.0f;
    for (int w = 0; w < 8; w++) s += sm[w][lane];
    partial[(int64_t)blockIdx.y * n + col] = s;
  }
}

// ---- RoPE -------------------------------------------------------------------

// Pair rotation with the reference's rounding points
// (a2_attention_provider.c:792-804): forward (a - b, c + d), backward
// (a + b, -c + d), a = x0 cos, b = x1 sin, c = x0 sin, d = x1 cos.
__global__ void rope_kernel(const float* __restrict__ x, float* __restrict__ y,
                            const float* __restrict__ ct, const float* __restrict__ st,
                            int64_t N, int64_t H, int64_t T, int64_t half, int backward) {
  const int64_t total = N * H * T * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pair = i % half;
    const int64_t t = (i / half) % T;
    const int64_t n = i / (half * T * H);
    const float c = ct[(n * T + t) * half + pair];
    const float s = st[(n * T + t) * half + pair];
    const float x0 = x[2 * i], x1 = x[2 * i + 1];
    const float a = rn_mul(x0, c), b = rn_mul(x1, s), cc = rn_mul(x0, s), dd = rn_mul(x1, c);
    y[2 * i] = backward ? rn_add(a, b) : rn_sub(a, b);
    y[2 * i + 1] = backward ? rn_add(-cc, dd) : rn_add(cc, dd);
  }
}

unsigned grid_for(int64_t n, int threads) {
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 16;
  return (unsigned)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

// Launches reduce_partials_kernel for 1 to 3 quantities (o1, o2 optional).
void reduce_partials(const float* partial, int count, int64_t width, int64_t stride, float* o0,
                     float* o1, float* o2, cudaStream_t stream) {
  PartialOuts outs{{o0, o1, o2}};
  const unsigned nq = o2 ? 3u : (o1 ? 2u : 1u);
  dim3 grid(ceil_div(width, 32), nq);
  reduce_partials_kernel<<<grid, 256, 0, stream>>>(partial, count, width, stride, outs);
  count_launch();
}

void layer_norm_forward(const float* x, const float* gamma, const float* beta, float epsilon,
                        float* y, float* mean, float* rstd, size_t rows, size_t d,
                        cudaStream_t stream, float* y_lo, OperandScale sc) {
  if (rows == 0) return;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(y_lo) | reinterpret_cast<uintptr_t>(gamma) |
                         reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
  if (aligned && d % 128 == 0 && d <= 1024) {
    switch (d / 128) {
#define LNF_CASE(nv)                                                                        \
  case nv:                                                                                  \
    ln_forward_rows_kernel<nv><<<ceil_div(rows, kLnWarps), kLnWarps * 32, 0, stream>>>(      \
        x, gamma, beta, epsilon, y, mean, rstd, (int64_t)rows, y_lo, sc);                   \
    break;
      LNF_CASE(1) LNF_CASE(2) LNF_CASE(3) LNF_CASE(4) LNF_CASE(5) LNF_CASE(6) LNF_CASE(7)
      LNF_CASE(8)
#undef LNF_CASE
    }
    count_launch();
    return;
  }
  ln_forward_kernel<<<ceil_div(rows, kLnWarps), kLnWarps * 32, 0, stream>>>(
      x, gamma, beta, epsilon, y, mean, rstd, (int64_t)rows, (int64_t)d, y_lo, sc);
  count_launch();
}

size_t ln_workspace_floats(size_t rows, size_t d) {
  const size_t simt = (size_t)ln_backward_blocks(rows) * 2 * d;
  const size_t regs = (size_t)ln_backward_rows_blocks(rows) * 3 * d;
  const size_t cols = colsum_workspace_floats(rows, d);
  return std::max(std::max(simt, regs), cols);
}

void layer_norm_backward(const float* x, const float* gamma, const float* mean, const float* rstd,
                         const float* dy, float* dx, int accumulate, float* dgamma, float* dbeta,
                         float* workspace, size_t rows, size_t d, cudaStream_t stream,
                         float* dx_hi, float* dx_lo, float* dsum, OperandScale sc) {
  if (rows == 0) return;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                         reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(gamma) |
                         reinterpret_cast<uintptr_t>(dx_hi) | reinterpret_cast<uintptr_t>(dx_lo)) &
                        15) == 0;
  if (aligned && d % 128 == 0 && d <= 1024) {
    const int blocks = ln_backward_rows_blocks(rows);
    const int nq = dsum ? 3 : 2;
    const int with_sum = dsum ? 1 : 0;
    float* hi = dx_lo ? dx_hi : nullptr;
    switch (d / 128) {
#define LNB_CASE(nv)                                                                          \
  case nv: {                                                                                  \
    const int smem = (kLnbWarps * 3 + 1) * 32 * (nv) * (int)sizeof(float4);                  \
    if (smem > 48 * 1024)                                                                     \
      cudaFuncSetAttribute(ln_backward_rows_kernel<nv>,                                       \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                \
    ln_backward_rows_kernel<nv><<<blocks, kLnbWarps * 32, smem, stream>>>(                    \
        x, gamma, mean, rstd, dy, dx, accumulate, hi, dx_lo, workspace, with_sum, (int64_t)rows, \
        sc);                                                                                  \
    break;                                                                                    \
  }
      LNB_CASE(1) LNB_CASE(2) LNB_CASE(3) LNB_CASE(4) LNB_CASE(5) LNB_CASE(6) LNB_CASE(7)
      LNB_CASE(8)
#undef LNB_CASE
    }
    count_launch();
    reduce_partials(workspace, blocks, (int64_t)d, (int64_t)nq * d, dgamma, dbeta, dsum, stream);
    return;
  }
  if (sc.f16 || sc.amax != nullptr) {  // operand scales exist on the register-row path only
    fprintf(stderr, "et_b200: LayerNorm backward with d = %zu has no split-f16 output\n", d);
    static const int one = 1;
    cudaMemcpy(device_error_word(), &one, sizeof(int), cudaMemcpyHostToDevice);
    return;
  }
  const int blocks = ln_backward_blocks(rows);
  const size_t smem = (size_t)kLnWarps * 2 * d * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(ln_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  ln_backward_kernel<<<blocks, kLnWarps * 32, smem, stream>>>(
      x, gamma, mean, rstd, dy, dx, accumulate, workspace, (int64_t)rows, (int64_t)d,
      dx_lo ? dx_hi : nullptr, dx_lo);
  count_launch();
  reduce_partials(workspace, blocks, (int64_t)d, (int64_t)(2 * d), dgamma, dbeta, nullptr, stream);
  if (dsum) column_sum(dx, dsum, rows, d, workspace, stream);
}

void gelu_forward(const float* x, float* y, size_t count, cudaStream_t stream, float* y_lo) {
  gelu_forward_kernel<<<grid_for(count, 256), 256, 0, stream>>>(x, y, (int64_t)count, y_lo);
  count_launch();
}
void gelu_backward(const float* x, const float* dy, float* dx, size_t count, cudaStream_t stream,
                   float* dx_lo) {
  gelu_backward_kernel<<<grid_for(count, 256), 256, 0, stream>>>(x, dy, dx, (int64_t)count, dx_lo);
  count_launch();
}
void relu_forward(const float* x, float* y, size_t count, cudaStream_t stream) {
  relu_kernel<<<grid_for(count, 256), 256, 0, stream>>>(x, nullptr, y, (int64_t)count);
  count_launch();
}
void relu_backward(const float* x, const float* dy, float* dx, size_t count, cudaStream_t stream) {
  relu_kernel<<<grid_for(count, 256), 256, 0, stream>>>(x, dy, dx, (int64_t)count);
  count_launch();
}
void add_tensors(const float* a, const float* b, float* out, size_t count, cudaStream_t stream) {
  add_kernel<<<grid_for(count, 256), 256, 0, stream>>>(a, b, out, (int64_t)count);
  count_launch();
}
void copy_tensor(const float* a, float* out, size_t count, cudaStream_t stream) {
  copy_kernel<<<grid_for(count, 256), 256, 0, stream>>>(a, out, (int64_t)count);
  count_launch();
}
void split_tf32(const float* x, float* hi, float* lo, size_t count, cudaStream_t stream) {
  if (count == 0) return;
  split_tf32_kernel<<<grid_for(count, 256), 256, 0, stream>>>(x, hi, lo, (int64_t)count);
  count_launch();
}
void abs_max(const float* x, size_t count, unsigned* amax, cudaStream_t stream) {
  if (count == 0) return;
  abs_max_kernel<<<grid_for((count + 3) / 4, 256), 256, 0, stream>>>(x, (int64_t)count, amax);
  count_launch();
}
void scale_from_amax(unsigned* amax, int* exp, int count, int target, int reset,
                     cudaStream_t stream) {
  if (count <= 0) return;
  scale_from_amax_kernel<<<1, 256, 0, stream>>>(amax, exp, count, target, reset);
  count_launch();
}
void split_f16(const float* x, const float* xlo, size_t count, uint16_t* hi, uint16_t* lo,
               const int* exp, unsigned* amax, cudaStream_t stream) {
  if (count == 0) return;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = al(x) && (xlo == nullptr || al(xlo)) &&
                   (reinterpret_cast<uintptr_t>(hi) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(lo) & 7) == 0;
  const int64_t n4 = vec ? (int64_t)(count / 4) : 0;
  if (n4 > 0) {
    split_f16_kernel<<<grid_for((size_t)n4, 256), 256, 0, stream>>>(x, xlo, n4, hi, lo, exp, amax);
    count_launch();
  }
  if ((size_t)(4 * n4) < count) {
    split_f16_tail_kernel<<<1, 256, 0, stream>>>(x, xlo, 4 * n4, (int64_t)count, hi, lo, exp,
                                                 amax);
    count_launch();
  }
}
void operand_range_check(unsigned* amax, const int* exp, int count, int reset_slot, float* flag,
                         cudaStream_t stream) {
  operand_range_kernel<<<1, 256, 0, stream>>>(amax, exp, count, reset_slot, flag);
  count_launch();
}
void check_finite(const float* x, size_t count, int* flag, cudaStream_t stream) {
  if (count == 0) return;
  finite_kernel<<<grid_for(count, 256), 256, 0, stream>>>(x, (int64_t)count, flag);
  count_launch();
}

void embedding_forward(const int64_t* ids, const float* w, float* y, size_t rows, size_t V,
                       size_t d, int* status, cudaStream_t stream) {
  if (rows == 0) return;
  embedding_forward_kernel<<<(unsigned)rows, 128, 0, stream>>>(ids, w, y, (int64_t)rows,
                                                               (int64_t)V, (int64_t)d, status);
  count_launch();
}

static size_t cub_sort_bytes(size_t rows) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (const uint32_t*)nullptr, (uint32_t*)nullptr, (int)rows);
  return (bytes + 255) & ~(size_t)255;
}

size_t embedding_scratch_bytes(size_t rows, size_t V) {
  (void)V;
  const size_t arr = ((rows * sizeof(uint32_t)) + 255) & ~(size_t)255;
  return 4 * arr + cub_sort_bytes(rows);
}

void embedding_backward(const int64_t* ids, const float* dy, const float* base, float* dw,
                        size_t rows, size_t V, size_t d, void* scratch, cudaStream_t stream) {
  const size_t arr = ((rows * sizeof(uint32_t)) + 255) & ~(size_t)255;
  uint8_t* p = (uint8_t*)scratch;
  uint32_t* keys_in = (uint32_t*)p;
  uint32_t* keys_out = (uint32_t*)(p + arr);
  uint32_t* vals_in = (uint32_t*)(p + 2 * arr);
  uint32_t* vals_out = (uint32_t*)(p + 3 * arr);
  void* temp = p + 4 * arr;
  size_t temp_bytes = cub_sort_bytes(rows);
  int end_bit = 1;
  while (end_bit < 32 && (1ull << end_bit) < V) end_bit++;
  if (rows > 0) {
    ids_to_keys_kernel<<<ceil_div(rows, 256), 256, 0, stream>>>(ids, keys_in, vals_in, (int64_t)rows);
    cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, vals_in, vals_out,
                                    (int)rows, 0, end_bit, stream);
    count_launch(2);
  }
  embedding_backward_kernel<<<(unsigned)V, 128, 0, stream>>>(keys_out, vals_out, dy, base, dw,
                                                             (int64_t)rows, (int64_t)d);
  count_launch();
}

size_t gelu_colsum_workspace_floats(size_t rows, size_t n) {
  return ((rows + kGcRows - 1) / kGcRows) * 8 * n;
}

void gelu_backward_colsum(const float* x, const float* dy, float* dx, float* dx_lo, float* dsum,
                          float* workspace, size_t rows, size_t n, cudaStream_t stream) {
  if (rows == 0) {
    cudaMemsetAsync(dsum, 0, n * sizeof(float), stream);
    return;
  }
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                         reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dx_lo)) &
                        15) == 0;
  if (!aligned || n % 128 != 0) {
    gelu_backward(x, dy, dx, rows * n, stream, dx_lo);
    column_sum(dx, dsum, rows, n, workspace, stream, dx_lo);
    return;
  }
  const unsigned chunks = ceil_div(rows, kGcRows);
  dim3 grid((unsigned)(n / 128), chunks);
  gelu_backward_colsum_kernel<<<grid, 256, 0, stream>>>(x, dy, dx, dx_lo, workspace, (int64_t)rows,
                                                        (int64_t)n);
  count_launch();
  reduce_partials(workspace, (int)chunks * 8, (int64_t)n, (int64_t)n, dsum, nullptr, nullptr,
                  stream);
}

size_t colsum_workspace_floats(size_t rows, size_t n) {
  return ((rows + kColRowsChunk - 1) / kColRowsChunk) * n;
}

void column_sum(const float* dy, float* out, size_t rows, size_t n, float* workspace,
                cudaStream_t stream, const float* dy_lo) {
  const unsigned chunks = ceil_div(rows, kColRowsChunk);
  if (chunks == 0) {
    cudaMemsetAsync(out, 0, n * sizeof(float), stream);
    return;
  }
  dim3 grid(ceil_div(n, 32), chunks);
  colsum_partial_kernel<<<grid, 256, 0, stream>>>(dy, dy_lo, workspace, (int64_t)rows, (int64_t)n);
  count_launch();
  reduce_partials(workspace, (int)chunks, (int64_t)n, (int64_t)n, out, nullptr, nullptr, stream);
}

void rope_apply(const float* x, float* y, const float* cos_table, const float* sin_table, size_t N,
                size_t H, size_t T, size_t Dh, int backward, cudaStream_t stream) {
  const int64_t total = (int64_t)(N * H * T * (Dh / 2));
  if (total == 0) return;
  rope_kernel<<<grid_for(total, 256), 256, 0, stream>>>(x, y, cos_table, sin_table, (int64_t)N,
                                                        (int64_t)H, (int64_t)T, (int64_t)(Dh / 2),
                                                        backward);
  count_launch();
}

}  // namespace etb
