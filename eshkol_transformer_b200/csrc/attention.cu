// A2 causal attention, forward and backward (FP32 FFMA flash tiles).
//
// Semantics follow native/a2_attention_provider.c:221-368 and 669-790:
//   s = (q . k) * (1 / sqrtf(Dh)) over admitted keys
//       (keep[b, tq, tk] != 0 and kpos[b, tk] <= qpos[b, tq]);
//   o = sum_k softmax(s)_k v_k; a row with no admitted key gives o = +0;
//   dq/dk/dv from ds = p (dO . v - sum_k p dO . v); dk/dv of a KV head sum
//   over its query-head group (GQA, kv head = hq / (Hq / Hkv)).
// RoPE (a2_attention_provider.c:792-804) is applied in registers as Q/K tiles
// are loaded, and its backward rotation to dQ/dK before they are stored, with
// cos/sin tables built on the host by libm so the rotation is bit-identical.
//
// Forward: one CTA per (64-query tile, b, hq) with online softmax; it stores
// the row max m and the row sum l so backward recomputes p = exp(s - m) / l.
// Backward is deterministic (no atomics): one kernel owns a 64-key tile and
// accumulates dK/dV over every query tile and head of its group; a second
// owns a 64-query tile and accumulates dQ over the key tiles.  Tiles entirely
// above the causal diagonal (first key position > last query position) are
// skipped.
#include "ops.cuh"

namespace etb {

namespace {

constexpr int BM = 64;
constexpr int BN = 64;
constexpr int kThreads = 256;
constexpr int PAD = 4;

struct RopeTable {
  const float* cos_t;
  const float* sin_t;
};

// Loads rows [t0, t0+rows) of one (b, h) slice into smem [rows][DH+PAD],
// zero-padding past Dh and past the sequence end; applies the forward RoPE
// rotation when a table is given (table row = b * T + t).
template <int DH>
__device__ __forceinline__ void load_tile(float* dst, const float* base, int64_t st, int t0,
                                          int T, int Dh, RopeTable rope, int b) {
  const int half = Dh >> 1;
  for (int idx = threadIdx.x; idx < BM * (DH / 2); idx += kThreads) {
    const int r = idx / (DH / 2);
    const int pair = idx % (DH / 2);
    const int t = t0 + r;
    float x0 = 0.0f, x1 = 0.0f;
    const int c0 = 2 * pair;
    if (t < T) {
      const float* row = base + (int64_t)t * st;
      if (c0 < Dh) x0 = row[c0];
      if (c0 + 1 < Dh) x1 = row[c0 + 1];
      if (rope.cos_t != nullptr && c0 + 1 < Dh) {
        const int64_t ti = ((int64_t)b * T + t) * half + pair;
        const float c = rope.cos_t[ti], s = rope.sin_t[ti];
        const float a = rn_mul(x0, c), bb = rn_mul(x1, s), cc = rn_mul(x0, s), dd = rn_mul(x1, c);
        x0 = rn_sub(a, bb);
        x1 = rn_add(cc, dd);
      }
    }
    dst[r * (DH + PAD) + c0] = x0;
    dst[r * (DH + PAD) + c0 + 1] = x1;
  }
}

// S[BM x BN] = A[BM][DH] . B[BN][DH]^T for this thread's 4x4 block
// (rows ty*4+i, cols tx + 16*j).
template <int DH>
__device__ __forceinline__ void tile_dot(float acc[4][4], const float* A, const float* B, int ty,
                                         int tx) {
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
#pragma unroll 4
  for (int d = 0; d < DH; d += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
      a[i] = *reinterpret_cast<const float4*>(A + (ty * 4 + i) * (DH + PAD) + d);
#pragma unroll
    for (int j = 0; j < 4; j++)
      b[j] = *reinterpret_cast<const float4*>(B + (tx + 16 * j) * (DH + PAD) + d);
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
        acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
        acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
        acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
      }
  }
}

__device__ __forceinline__ bool admitted(const AttnParams& p, int b, int tq, int tk) {
  if (tq >= p.Tq || tk >= p.Tk) return false;
  if (p.kpos[(int64_t)b * p.Tk + tk] > p.qpos[(int64_t)b * p.Tq + tq]) return false;
  return p.mask == nullptr || p.mask[((int64_t)b * p.Tq + tq) * p.Tk + tk] != 0;
}

// Index of the last key tile that can hold an admitted key for query rows
// [q0, q0+BM): keys beyond the first position greater than the last query
// position are never admitted (positions are strictly increasing).
__device__ __forceinline__ int key_tile_end(const AttnParams& p, int b, int q0) {
  const int qlast = min(q0 + BM, p.Tq) - 1;
  const int64_t qmax = p.qpos[(int64_t)b * p.Tq + qlast];
  const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
  int lo = 0, hi = p.Tk;  // first tk with kpos > qmax
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (kp[mid] <= qmax) lo = mid + 1; else hi = mid;
  }
  return (lo + BN - 1) / BN;
}

// First query tile whose last row may admit key position kmin.
__device__ __forceinline__ int query_tile_begin(const AttnParams& p, int b, int k0) {
  const int64_t kmin = p.kpos[(int64_t)b * p.Tk + k0];
  const int64_t* qp = p.qpos + (int64_t)b * p.Tq;
  int lo = 0, hi = p.Tq;  // first tq with qpos >= kmin
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (qp[mid] < kmin) lo = mid + 1; else hi = mid;
  }
  return lo / BM;
}

template <int DH>
__global__ void __launch_bounds__(kThreads)
attn_fwd_kernel(AttnParams p, AttnOut o, float* __restrict__ row_max, float* __restrict__ row_sum,
                int q_rope_bstride, int k_rope_bstride) {
  extern __shared__ __align__(16) float smem[];
  float* Qs = smem;
  float* Ks = Qs + BM * (DH + PAD);
  float* Vs = Ks + BN * (DH + PAD);
  float* Ps = Vs + BN * (DH + PAD);  // [BM][BN+1]
  constexpr int CPT = DH / 16;       // output columns per thread
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int q0 = blockIdx.x * BM;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / (p.Hq / p.Hkv);
  const float* qb = p.q.ptr + b * p.q.sb + hq * p.q.sh;
  const float* kb = p.k.ptr + b * p.k.sb + hkv * p.k.sh;
  const float* vb = p.v.ptr + b * p.v.sb + hkv * p.v.sh;
  RopeTable qr{p.q_cos, p.q_sin}, kr{p.k_cos, p.k_sin};
  load_tile<DH>(Qs, qb, p.q.st, q0, p.Tq, p.Dh, qr, q_rope_bstride ? b : 0);

  float m[4], l[4], acc[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPT; c++) acc[i][c] = 0.0f;
  }
  const int kt_end = key_tile_end(p, b, q0);
  for (int kt = 0; kt < kt_end; kt++) {
    const int k0 = kt * BN;
    __syncthreads();
    load_tile<DH>(Ks, kb, p.k.st, k0, p.Tk, p.Dh, kr, k_rope_bstride ? b : 0);
    load_tile<DH>(Vs, vb, p.v.st, k0, p.Tk, p.Dh, RopeTable{nullptr, nullptr}, 0);
    __syncthreads();
    float s[4][4];
    tile_dot<DH>(s, Qs, Ks, ty, tx);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int tq = q0 + ty * 4 + i;
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int tk = k0 + tx + 16 * j;
        s[i][j] = admitted(p, b, tq, tk) ? rn_mul(s[i][j], p.scale) : -INFINITY;
        tmax = fmaxf(tmax, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mnew = fmaxf(m[i], tmax);
      const float corr = (mnew == -INFINITY) ? 1.0f : expf(m[i] - mnew);
      float psum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float e = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - mnew);
        Ps[(ty * 4 + i) * (BN + 1) + tx + 16 * j] = e;
        psum += e;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l[i] = l[i] * corr + psum;
      m[i] = mnew;
#pragma unroll
      for (int c = 0; c < CPT; c++) acc[i][c] *= corr;
    }
    __syncthreads();
    for (int k = 0; k < BN; k++) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) pv[i] = Ps[(ty * 4 + i) * (BN + 1) + k];
      const float* vrow = Vs + k * (DH + PAD) + tx * CPT;
#pragma unroll
      for (int c = 0; c < CPT; c++) {
        const float vv = vrow[c];
#pragma unroll
        for (int i = 0; i < 4; i++) acc[i][c] = fmaf(pv[i], vv, acc[i][c]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int tq = q0 + ty * 4 + i;
    if (tq >= p.Tq) continue;
    const bool empty = l[i] == 0.0f;
    float* orow = o.ptr + b * o.sb + hq * o.sh + (int64_t)tq * o.st;
#pragma unroll
    for (int c = 0; c < CPT; c++) {
      const int col = tx * CPT + c;
      if (col < p.Dh) orow[col] = empty ? 0.0f : rn_div(acc[i][c], l[i]);
    }
    if (tx == 0) {
      const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
      row_max[ri] = empty ? 0.0f : m[i];
      row_sum[ri] = l[i];
    }
  }
}

// delta[b, hq, tq] = sum_j dO[j] O[j]  (equals the reference's mean_dp)
__global__ void attn_delta_kernel(AttnParams p, AttnTensor o, const float* __restrict__ o_lo,
                                  AttnTensor dout, float* __restrict__ delta) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t rows = (int64_t)p.B * p.Hq * p.Tq;
  if (row >= rows) return;
  const int tq = (int)(row % p.Tq);
  const int hq = (int)((row / p.Tq) % p.Hq);
  const int b = (int)(row / ((int64_t)p.Tq * p.Hq));
  const int64_t ooff = b * o.sb + hq * o.sh + (int64_t)tq * o.st;
  const float* orow = o.ptr + ooff;
  const float* lrow = o_lo ? o_lo + ooff : nullptr;
  const float* grow = dout.ptr + b * dout.sb + hq * dout.sh + (int64_t)tq * dout.st;
  float s = 0.0f;
  for (int j = lane; j < p.Dh; j += 32) s = fmaf(grow[j], lrow ? orow[j] + lrow[j] : orow[j], s);
  s = warp_sum(s);
  if (lane == 0) delta[row] = s;
}

// Stores a [64][DH] register tile (rows ty*4+i, cols tx*CPT+c) through smem,
// applying the RoPE backward rotation when a table is given.
template <int DH>
__device__ __forceinline__ void store_tile(float (*acc)[DH / 16], float* stage, AttnOut out, int b,
                                           int h, int t0, int T, int Dh, RopeTable rope,
                                           int rope_b, float scale_mul) {
  constexpr int CPT = DH / 16;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int c = 0; c < CPT; c++)
      stage[(ty * 4 + i) * (DH + PAD) + tx * CPT + c] = rn_mul(acc[i][c], scale_mul);
  __syncthreads();
  const int half = Dh >> 1;
  for (int idx = tid; idx < BM * (DH / 2); idx += kThreads) {
    const int r = idx / (DH / 2), pair = idx % (DH / 2);
    const int t = t0 + r, c0 = 2 * pair;
    if (t >= T || c0 >= Dh) continue;
    float x0 = stage[r * (DH + PAD) + c0];
    float x1 = stage[r * (DH + PAD) + c0 + 1];
    float* row = out.ptr + b * out.sb + h * out.sh + (int64_t)t * out.st;
    if (rope.cos_t != nullptr && c0 + 1 < Dh) {
      const int64_t ti = ((int64_t)rope_b * T + t) * half + pair;
      const float c = rope.cos_t[ti], s = rope.sin_t[ti];
      const float a = rn_mul(x0, c), bb = rn_mul(x1, s), cc = rn_mul(x0, s), dd = rn_mul(x1, c);
      x0 = rn_add(a, bb);
      x1 = rn_add(-cc, dd);
    }
    row[c0] = x0;
    if (c0 + 1 < Dh) row[c0 + 1] = x1;
  }
}

// dK / dV for one 64-key tile of (b, hkv).
template <int DH>
__global__ void __launch_bounds__(kThreads)
attn_bwd_kv_kernel(AttnParams p, AttnTensor dout, const float* __restrict__ row_max,
                   const float* __restrict__ row_sum, const float* __restrict__ delta,
                   AttnOut dk, AttnOut dv, int q_rope_bstride, int k_rope_bstride) {
  extern __shared__ __align__(16) float smem[];
  float* Ks = smem;
  float* Vs = Ks + BN * (DH + PAD);
  float* Qs = Vs + BN * (DH + PAD);
  float* Gs = Qs + BM * (DH + PAD);   // dO tile
  float* Ps = Gs + BM * (DH + PAD);   // [BM][BN+1] probabilities
  float* Ds = Ps + BM * (BN + 1);     // [BM][BN+1] dS
  float* stat = Ds + BM * (BN + 1);   // m, l, delta for BM rows
  constexpr int CPT = DH / 16;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int k0 = blockIdx.x * BN;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int group = p.Hq / p.Hkv;
  const float* kb = p.k.ptr + b * p.k.sb + hkv * p.k.sh;
  const float* vb = p.v.ptr + b * p.v.sb + hkv * p.v.sh;
  RopeTable qr{p.q_cos, p.q_sin}, kr{p.k_cos, p.k_sin};
  load_tile<DH>(Ks, kb, p.k.st, k0, p.Tk, p.Dh, kr, k_rope_bstride ? b : 0);
  load_tile<DH>(Vs, vb, p.v.st, k0, p.Tk, p.Dh, RopeTable{nullptr, nullptr}, 0);

  float adk[4][CPT], adv[4][CPT];  // rows = keys ty*4+i
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int c = 0; c < CPT; c++) adk[i][c] = adv[i][c] = 0.0f;

  const int qt_begin = (k0 < p.Tk) ? query_tile_begin(p, b, k0) : 0;
  const int qt_count = (p.Tq + BM - 1) / BM;
  for (int hq = hkv * group; hq < (hkv + 1) * group; hq++) {
    const float* qb = p.q.ptr + b * p.q.sb + hq * p.q.sh;
    const float* gb = dout.ptr + b * dout.sb + hq * dout.sh;
    for (int qt = qt_begin; qt < qt_count; qt++) {
      const int q0 = qt * BM;
      __syncthreads();
      load_tile<DH>(Qs, qb, p.q.st, q0, p.Tq, p.Dh, qr, q_rope_bstride ? b : 0);
      load_tile<DH>(Gs, gb, dout.st, q0, p.Tq, p.Dh, RopeTable{nullptr, nullptr}, 0);
      for (int r = tid; r < BM; r += kThreads) {
        const int tq = q0 + r;
        const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
        stat[r] = tq < p.Tq ? row_max[ri] : 0.0f;
        stat[BM + r] = tq < p.Tq ? row_sum[ri] : 0.0f;
        stat[2 * BM + r] = tq < p.Tq ? delta[ri] : 0.0f;
      }
      __syncthreads();
      float s[4][4], dp[4][4];
      tile_dot<DH>(s, Qs, Ks, ty, tx);   // rows = queries, cols = keys
      tile_dot<DH>(dp, Gs, Vs, ty, tx);  // dP = dO V^T
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int r = ty * 4 + i, tq = q0 + r;
        const float mrow = stat[r], lrow = stat[BM + r], drow = stat[2 * BM + r];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int c = tx + 16 * j, tk = k0 + c;
          float pr = 0.0f;
          if (lrow != 0.0f && admitted(p, b, tq, tk))
            pr = rn_div(expf(rn_mul(s[i][j], p.scale) - mrow), lrow);
          Ps[r * (BN + 1) + c] = pr;
          Ds[r * (BN + 1) + c] = pr * (dp[i][j] - drow);
        }
      }
      __syncthreads();
      // dV[k] += sum_q P[q][k] dO[q];  dK[k] += sum_q dS[q][k] Q[q]
      for (int q = 0; q < BM; q++) {
        float pk[4], dk_[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          pk[i] = Ps[q * (BN + 1) + ty * 4 + i];
          dk_[i] = Ds[q * (BN + 1) + ty * 4 + i];
        }
        const float* grow = Gs + q * (DH + PAD) + tx * CPT;
        const float* qrow = Qs + q * (DH + PAD) + tx * CPT;
#pragma unroll
        for (int c = 0; c < CPT; c++) {
          const float gv = grow[c], qv = qrow[c];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            adv[i][c] = fmaf(pk[i], gv, adv[i][c]);
            adk[i][c] = fmaf(dk_[i], qv, adk[i][c]);
          }
        }
      }
    }
  }
  // reuse Qs as the staging buffer
  store_tile<DH>(adv, Qs, dv, b, hkv, k0, p.Tk, p.Dh, RopeTable{nullptr, nullptr}, 0, 1.0f);
  store_tile<DH>(adk, Qs, dk, b, hkv, k0, p.Tk, p.Dh, kr, k_rope_bstride ? b : 0, p.scale);
}

// dQ for one 64-query tile of (b, hq).
template <int DH>
__global__ void __launch_bounds__(kThreads)
attn_bwd_q_kernel(AttnParams p, AttnTensor dout, const float* __restrict__ row_max,
                  const float* __restrict__ row_sum, const float* __restrict__ delta, AttnOut dq,
                  int q_rope_bstride, int k_rope_bstride) {
  extern __shared__ __align__(16) float smem[];
  float* Qs = smem;
  float* Gs = Qs + BM * (DH + PAD);
  float* Ks = Gs + BM * (DH + PAD);
  float* Vs = Ks + BN * (DH + PAD);
  float* Ds = Vs + BN * (DH + PAD);  // [BM][BN+1]
  constexpr int CPT = DH / 16;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int q0 = blockIdx.x * BM;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / (p.Hq / p.Hkv);
  const float* qb = p.q.ptr + b * p.q.sb + hq * p.q.sh;
  const float* gb = dout.ptr + b * dout.sb + hq * dout.sh;
  const float* kb = p.k.ptr + b * p.k.sb + hkv * p.k.sh;
  const float* vb = p.v.ptr + b * p.v.sb + hkv * p.v.sh;
  RopeTable qr{p.q_cos, p.q_sin}, kr{p.k_cos, p.k_sin};
  load_tile<DH>(Qs, qb, p.q.st, q0, p.Tq, p.Dh, qr, q_rope_bstride ? b : 0);
  load_tile<DH>(Gs, gb, dout.st, q0, p.Tq, p.Dh, RopeTable{nullptr, nullptr}, 0);
  float mrow[4], lrow[4], drow[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int tq = q0 + ty * 4 + i;
    const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
    mrow[i] = tq < p.Tq ? row_max[ri] : 0.0f;
    lrow[i] = tq < p.Tq ? row_sum[ri] : 0.0f;
    drow[i] = tq < p.Tq ? delta[ri] : 0.0f;
  }
  float adq[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int c = 0; c < CPT; c++) adq[i][c] = 0.0f;
  const int kt_end = key_tile_end(p, b, q0);
  for (int kt = 0; kt < kt_end; kt++) {
    const int k0 = kt * BN;
    __syncthreads();
    load_tile<DH>(Ks, kb, p.k.st, k0, p.Tk, p.Dh, kr, k_rope_bstride ? b : 0);
    load_tile<DH>(Vs, vb, p.v.st, k0, p.Tk, p.Dh, RopeTable{nullptr, nullptr}, 0);
    __syncthreads();
    float s[4][4], dp[4][4];
    tile_dot<DH>(s, Qs, Ks, ty, tx);
    tile_dot<DH>(dp, Gs, Vs, ty, tx);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int r = ty * 4 + i, tq = q0 + r;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int c = tx + 16 * j, tk = k0 + c;
        float pr = 0.0f;
        if (lrow[i] != 0.0f && admitted(p, b, tq, tk))
          pr = rn_div(expf(rn_mul(s[i][j], p.scale) - mrow[i]), lrow[i]);
        Ds[r * (BN + 1) + c] = pr * (dp[i][j] - drow[i]);
      }
    }
    __syncthreads();
    for (int k = 0; k < BN; k++) {
      float dsv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) dsv[i] = Ds[(ty * 4 + i) * (BN + 1) + k];
      const float* krow = Ks + k * (DH + PAD) + tx * CPT;
#pragma unroll
      for (int c = 0; c < CPT; c++) {
        const float kv = krow[c];
#pragma unroll
        for (int i = 0; i < 4; i++) adq[i][c] = fmaf(dsv[i], kv, adq[i][c]);
      }
    }
  }
  store_tile<DH>(adq, Gs, dq, b, hq, q0, p.Tq, p.Dh, qr, q_rope_bstride ? b : 0, p.scale);
}

template <int DH>
size_t fwd_smem() { return (size_t)(BM + 2 * BN) * (DH + PAD) * 4 + (size_t)BM * (BN + 1) * 4; }
template <int DH>
size_t kv_smem() {
  return (size_t)(2 * BN + 2 * BM) * (DH + PAD) * 4 + 2 * (size_t)BM * (BN + 1) * 4 + 3 * BM * 4;
}
template <int DH>
size_t q_smem() { return (size_t)(2 * BM + 2 * BN) * (DH + PAD) * 4 + (size_t)BM * (BN + 1) * 4; }

template <int DH>
void launch_fwd(const AttnParams& p, AttnOut o, float* m, float* l, int qrb, int krb,
                cudaStream_t stream) {
  const size_t smem = fwd_smem<DH>();
  cudaFuncSetAttribute(attn_fwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((p.Tq + BM - 1) / BM, p.Hq, p.B);
  attn_fwd_kernel<DH><<<grid, kThreads, smem, stream>>>(p, o, m, l, qrb, krb);
  count_launch();
}

template <int DH>
void launch_bwd(const AttnParams& p, AttnTensor dout, const float* m, const float* l,
                const float* delta, AttnOut dq, AttnOut dk, AttnOut dv, int qrb, int krb,
                cudaStream_t stream) {
  const size_t s1 = kv_smem<DH>(), s2 = q_smem<DH>();
  cudaFuncSetAttribute(attn_bwd_kv_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1);
  cudaFuncSetAttribute(attn_bwd_q_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2);
  dim3 g1((p.Tk + BN - 1) / BN, p.Hkv, p.B);
  attn_bwd_kv_kernel<DH><<<g1, kThreads, s1, stream>>>(p, dout, m, l, delta, dk, dv, qrb, krb);
  dim3 g2((p.Tq + BM - 1) / BM, p.Hq, p.B);
  attn_bwd_q_kernel<DH><<<g2, kThreads, s2, stream>>>(p, dout, m, l, delta, dq, qrb, krb);
  count_launch(2);
}

}  // namespace

bool attention_forward(const AttnParams& p, AttnOut o, float* row_max, float* row_sum,
                       cudaStream_t stream) {
  if (p.B == 0 || p.Hq == 0 || p.Tq == 0) return false;
  if (attention_forward_tc(p, o, row_max, row_sum, stream)) return true;
  const int qb = p.q_rope_batched, kb = p.k_rope_batched;
  if (p.Dh <= 32) launch_fwd<32>(p, o, row_max, row_sum, qb, kb, stream);
  else if (p.Dh <= 64) launch_fwd<64>(p, o, row_max, row_sum, qb, kb, stream);
  else launch_fwd<128>(p, o, row_max, row_sum, qb, kb, stream);
  return false;
}

bool attention_backward(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                        const float* row_max,
                        const float* row_sum, float* delta, AttnOut dq, AttnOut dk, AttnOut dv,
                        cudaStream_t stream) {
  if (p.B == 0 || p.Hq == 0) return false;
  if (attention_backward_tc(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream))
    return true;
  const int64_t rows = (int64_t)p.B * p.Hq * p.Tq;
  if (rows > 0) {
    attn_delta_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(p, o, o_lo, dout, delta);
    count_launch();
  }
  const int qb = p.q_rope_batched, kb = p.k_rope_batched;
  if (p.Dh <= 32) launch_bwd<32>(p, dout, row_max, row_sum, delta, dq, dk, dv, qb, kb, stream);
  else if (p.Dh <= 64) launch_bwd<64>(p, dout, row_max, row_sum, delta, dq, dk, dv, qb, kb, stream);
  else launch_bwd<128>(p, dout, row_max, row_sum, delta, dq, dk, dv, qb, kb, stream);
  return false;
}

}  // namespace etb
