// Pieces shared by the tcgen05 attention kernels (attention_tc.cu forward,
// attention_bwd_tc.cu backward): the workspace layout, the TF32 hi/lo split
// of scores and probabilities, base-2 exponentials and the kind::tf32
// instruction descriptor.
#pragma once

#include "ops.cuh"
#include "tcgen05.cuh"

namespace etb {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Head-major [B, H, T, Dh] operand copies in the attention workspace: RoPE'd
// Q and K and plain V split into TF32 hi and residual lo, dO split the same
// way (backward), and per-row base-2 log-sum-exp lse2 = (m + ln l) log2(e)
// (backward; +inf for a row with no admitted key).  The binary16-pair
// backward (attention_bwd_f16.cu) keeps its dO and Q pairs (uint16 hi, lo
// arrays) where the TF32 dO pair would be, its K and V pairs behind lse2,
// and the four operand maxima (f32 bits) last.
struct AttnWs {
  float *qh, *ql, *kh, *kl, *vh, *vl, *doh, *dol, *lse2;
  uint16_t *g16h, *g16l, *q16h, *q16l, *k16h, *k16l, *v16h, *v16l;
  unsigned* amax16;
  // dK/dV chunk sums of the backward: `chunk_slots` slots of
  // kBwdChunkFloats floats (one per CTA holding one), each slot's flag in
  // slot_flags (0 free, 1 taken; cleared before every backward launch)
  int* slot_flags;
  float* chunks;
  int chunk_slots;
};
// dK and dV rows of a 128-key tile at head_dim <= 128, f32.
constexpr int kBwdChunkFloats = 2 * 128 * 128;
// Slots: every CTA that sums dK/dV in chunks holds one while it runs, and at
// most one such CTA is resident per SM (each holds all 512 TMEM columns and
// takes its slot after allocating them); twice the SM count leaves margin.
inline int attn_chunk_slots() { return 2 * sm_count(); }
inline AttnWs attn_ws(const AttnParams& p) {
  const size_t nq = (size_t)p.B * p.Hq * p.Tq * p.Dh, nk = (size_t)p.B * p.Hkv * p.Tk * p.Dh;
  const size_t rows = (size_t)p.B * p.Hq * p.Tq;
  AttnWs w;
  w.qh = p.ws;
  w.ql = w.qh + nq;
  w.kh = w.ql + nq;
  w.kl = w.kh + nk;
  w.vh = w.kl + nk;
  w.vl = w.vh + nk;
  w.doh = p.ws_grad != nullptr ? p.ws_grad : w.vl + nk;
  w.dol = w.doh + nq;
  w.lse2 = w.dol + nq;
  w.g16h = reinterpret_cast<uint16_t*>(w.doh);
  w.g16l = w.g16h + nq;
  w.q16h = reinterpret_cast<uint16_t*>(w.dol);
  w.q16l = w.q16h + nq;
  w.k16h = reinterpret_cast<uint16_t*>(w.lse2 + ((rows + 63) & ~(size_t)63));
  w.k16l = w.k16h + nk;
  w.v16h = w.k16l + nk;
  w.v16l = w.v16h + nk;
  w.amax16 = reinterpret_cast<unsigned*>(w.v16l + nk);
  if (p.pairs16) {
    // the producers' binary16 Q / K / V pairs live in the Q / K / V part (in
    // place of the TF32 pairs), so the backward finds them after the forward
    w.q16h = reinterpret_cast<uint16_t*>(p.ws);
    w.q16l = w.q16h + nq;
    w.k16h = w.q16l + nq;
    w.k16l = w.k16h + nk;
    w.v16h = w.k16l + nk;
    w.v16l = w.v16h + nk;
  }
  w.chunk_slots = attn_chunk_slots();
  w.slot_flags = reinterpret_cast<int*>(w.amax16 + 64);
  w.chunks = reinterpret_cast<float*>(w.slot_flags + ((w.chunk_slots + 63) & ~63));
  return w;
}

// Writes qh/ql, kh/kl, vh/vl of the workspace (3 launches).
void attention_prepare_qkv(const AttnParams& p, const AttnWs& w, cudaStream_t stream);

// Nearest TF32 value of a probability in [0, 1].
__device__ __forceinline__ float tf32_round(float v) {
  return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xffffe000u);
}
// Nearest TF32 value of a finite operand; magnitudes that would round up to
// infinity are truncated instead, so hi stays finite and lo = x - hi exact.
__device__ __forceinline__ float tf32_hi(float v) {
  const uint32_t u = __float_as_uint(v);
  uint32_t r = (u + 0x1000u) & 0xffffe000u;
  if ((r & 0x7f800000u) == 0x7f800000u) r = u & 0xffffe000u;
  return __uint_as_float(r);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// kind::tf32 instruction descriptor: f32 accumulate, M = 128, N = n, A
// K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1).
__host__ __device__ constexpr uint32_t idesc_tf32_m128(int n, int b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// K-major operand tile staged by TMA with the 128-byte swizzle: 32-column
// chunks of `rows` rows x 128 B.  Descriptor of K-slice j (8 columns).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int rows, int j) {
  return sdesc(base + (uint32_t)(j >> 2) * (uint32_t)rows * 128u + (uint32_t)(j & 3) * 32u, 16u,
               1024u, 2u);
}
// MN-major operand tile (128-byte swizzle, 32-byte atoms) of `krows` K-rows
// per 32-wide MN chunk.  Descriptor of K-slice j (8 K-rows).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int krows, int j) {
  return sdesc(base + 1024u * (uint32_t)j, (uint32_t)krows * 128u, 512u, 1u);
}
// The same descriptors from a slice-0 descriptor plus a constant: the start
// address field holds address >> 4 and shared-memory addresses stay below
// 2^18, so adding (offset >> 4) never carries out of the field.
template <int ROWS>
__device__ __forceinline__ uint64_t kslice(uint64_t d0, int j) {
  return d0 + (uint64_t)((((uint32_t)(j >> 2) * ROWS * 128u) + (uint32_t)(j & 3) * 32u) >> 4);
}
__device__ __forceinline__ uint64_t mslice(uint64_t d0, int j) { return d0 + (uint64_t)(64 * j); }

// Row `row` of a 128-row K-major tile staged by TMA with the 128-byte swizzle
// (32-column chunks of 128 rows x 128 B) -> 32 TMEM columns per chunk of this
// thread's lane, starting at column `col` of `trow`.
template <int COLS>
__device__ __forceinline__ void tile_row_to_tmem(uint32_t tile, int row, uint32_t trow,
                                                 uint32_t col) {
#pragma unroll
  for (int c = 0; c < COLS / 32; c++) {
    float v[32];
    const uint32_t rp = tile + (uint32_t)c * 128u * 128u + (uint32_t)row * 128u;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const float4 x = lds128(rp + (((uint32_t)u ^ (uint32_t)(row & 7)) << 4));
      v[4 * u] = x.x; v[4 * u + 1] = x.y; v[4 * u + 2] = x.z; v[4 * u + 3] = x.w;
    }
    tmem_st32(trow + col + 32 * c, v);
  }
}

// Output rows are staged in shared memory as [128][cols + 4] floats (the pad
// spreads a row-per-lane float4 store over all banks) and copied out with
// coalesced float4 stores: `nthreads` threads starting at thread `t`.
__device__ __forceinline__ void stage_row32(uint32_t stage, int cols, int row, int col,
                                            const float (&v)[32], int first, int n) {
  const uint32_t rp = stage + ((uint32_t)row * (uint32_t)(cols + 4) + (uint32_t)col) * 4u;
#pragma unroll
  for (int i = 0; i < n; i += 4)
    sts128(rp + 4u * (uint32_t)i, make_float4(v[first + i], v[first + i + 1], v[first + i + 2],
                                              v[first + i + 3]));
}
__device__ __forceinline__ void store_staged_rows(uint32_t stage, int cols, int rows_valid,
                                                  float* base, int64_t row_stride, int t,
                                                  int nthreads) {
  const int per_row = cols / 4;
  const bool vec = ((reinterpret_cast<uintptr_t>(base) | (uintptr_t)(row_stride * 4)) & 15) == 0;
  for (int idx = t; idx < rows_valid * per_row; idx += nthreads) {
    const int r = idx / per_row, c4 = idx - r * per_row;
    const float4 v = lds128(stage + ((uint32_t)r * (uint32_t)(cols + 4) + 4u * (uint32_t)c4) * 4u);
    float* dst = base + (int64_t)r * row_stride + 4 * c4;
    if (vec) {
      *reinterpret_cast<float4*>(dst) = v;
    } else {
      dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
    }
  }
}

// Writes `rows_valid` staged rows ([128][cols + 4] floats at `stage`) with
// coalesced stores: thread t of `nthreads` takes float4s t, t + nthreads, ...
// (row r = i / (cols / 4), column 4 (i % (cols / 4))), applies f(r, c4, v) in
// place, then stores v to hi (lo null), its TF32 hi part to hi and the
// residual to lo, or (sc.f16) the binary16 pair of v 2^(*sc.exp) to hi / lo
// as uint16 arrays.  Row r goes to element off + r * row_stride of hi / lo.
// Returns the sum of the thread's v (its rows of columns 4 (t % (cols / 4))
// .. when nthreads is a multiple of cols / 4); amax takes max |v|.
template <typename F>
__device__ __forceinline__ float4 store_rows_split(uint32_t stage, int cols, int rows_valid,
                                                   float* hi, float* lo, int64_t off0,
                                                   int64_t row_stride, int t, int nthreads, F f,
                                                   const OperandScale& sc, float& amax) {
  float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
  const int per_row = cols / 4;
  if (sc.f16) {
    // 8-byte stores: hi / lo 8-byte aligned and row_stride % 4 == 0 (host-checked)
    uint16_t* hb = reinterpret_cast<uint16_t*>(hi) + off0;
    uint16_t* lb = reinterpret_cast<uint16_t*>(lo) + off0;
    const float s = exp2_int(*sc.exp);
#pragma unroll 4
    for (int idx = t; idx < rows_valid * per_row; idx += nthreads) {
      const int r = idx / per_row, c4 = idx - r * per_row;
      float4 v = lds128(stage + ((uint32_t)r * (uint32_t)(cols + 4) + 4u * (uint32_t)c4) * 4u);
      f(r, c4, v);
      sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
      amax = abs_max4(amax, v);
      f16_store4(hb, lb, (int64_t)r * row_stride + 4 * c4, v, s);
    }
    return sum;
  }
  float* hi_base = hi + off0;
  float* lo_base = lo != nullptr ? lo + off0 : nullptr;
  const uintptr_t bits = reinterpret_cast<uintptr_t>(hi_base) |
                         reinterpret_cast<uintptr_t>(lo_base) | (uintptr_t)(row_stride * 4);
  const bool vec = (bits & 15) == 0;
#pragma unroll 4
  for (int idx = t; idx < rows_valid * per_row; idx += nthreads) {
    const int r = idx / per_row, c4 = idx - r * per_row;
    float4 v = lds128(stage + ((uint32_t)r * (uint32_t)(cols + 4) + 4u * (uint32_t)c4) * 4u);
    f(r, c4, v);
    sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
    if (sc.amax != nullptr) amax = abs_max4(amax, v);
    float4 lo4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lo_base != nullptr) {
      tf32_split(v.x, v.x, lo4.x);
      tf32_split(v.y, v.y, lo4.y);
      tf32_split(v.z, v.z, lo4.z);
      tf32_split(v.w, v.w, lo4.w);
    }
    const int64_t off = (int64_t)r * row_stride + 4 * c4;
    if (vec) {
      *reinterpret_cast<float4*>(hi_base + off) = v;
      if (lo_base != nullptr) *reinterpret_cast<float4*>(lo_base + off) = lo4;
    } else {
      float* h = hi_base + off;
      h[0] = v.x; h[1] = v.y; h[2] = v.z; h[3] = v.w;
      if (lo_base != nullptr) {
        float* l = lo_base + off;
        l[0] = lo4.x; l[1] = lo4.y; l[2] = lo4.z; l[3] = lo4.w;
      }
    }
  }
  return sum;
}

// Column sums of a written tile from the threads' store_rows_split sums: each
// thread puts its sum into shared scratch `red` (nthreads float4) before a
// barrier of the nthreads threads (colsum_put), then the first cols / 4
// threads add the groups in thread order and store 4 columns each
// (colsum_get).
__device__ __forceinline__ void colsum_put(uint32_t red, int t, float4 sum) {
  sts128(red + (uint32_t)t * 16u, sum);
}
__device__ __forceinline__ void colsum_get(uint32_t red, int t, int nthreads, int cols,
                                           float* out) {
  const int per_row = cols / 4;
  if (t >= per_row) return;
  float4 s = lds128(red + (uint32_t)t * 16u);
  for (int g = 1; g < nthreads / per_row; g++) {
    const float4 v = lds128(red + (uint32_t)(g * per_row + t) * 16u);
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  *reinterpret_cast<float4*>(out + 4 * t) = s;
}

// Gradient scaling and RoPE backward rotation of columns 4 c4 .. 4 c4 + 3 of
// a row (pairs 2 c4, 2 c4 + 1 at table entries trow + 2 c4, + 1): x = v
// scale, then (x0, x1) -> (x0 c + x1 s, -x0 s + x1 c) when ct is set.  The
// tables are read-only for the kernel (non-coherent loads, which the
// compiler may issue ahead of the output stores), as one float2 per table
// when both are 8-byte aligned (trow and 2 c4 are even).
__device__ __forceinline__ void grad_rotate4(float4& v, float scale, const float* ct,
                                             const float* st, int64_t trow, int c4) {
  float x[4] = {rn_mul(v.x, scale), rn_mul(v.y, scale), rn_mul(v.z, scale), rn_mul(v.w, scale)};
  if (ct != nullptr) {
    float cv[2], sv[2];
    const int64_t t0 = trow + 2 * c4;
    if (((reinterpret_cast<uintptr_t>(ct) | reinterpret_cast<uintptr_t>(st)) & 7) == 0) {
      const float2 c2 = __ldg(reinterpret_cast<const float2*>(ct + t0));
      const float2 s2 = __ldg(reinterpret_cast<const float2*>(st + t0));
      cv[0] = c2.x; cv[1] = c2.y; sv[0] = s2.x; sv[1] = s2.y;
    } else {
      cv[0] = __ldg(ct + t0); cv[1] = __ldg(ct + t0 + 1);
      sv[0] = __ldg(st + t0); sv[1] = __ldg(st + t0 + 1);
    }
#pragma unroll
    for (int pr = 0; pr < 2; pr++) {
      const float c = cv[pr], s = sv[pr];
      const float x0 = x[2 * pr], x1 = x[2 * pr + 1];
      x[2 * pr] = rn_add(rn_mul(x0, c), rn_mul(x1, s));
      x[2 * pr + 1] = rn_add(-rn_mul(x0, s), rn_mul(x1, c));
    }
  }
  v = make_float4(x[0], x[1], x[2], x[3]);
}

// The RoPE tables' rows [tab_row0, tab_row0 + rows) (rows x dh / 2 floats
// each, contiguous in the tables) copied into shared memory: cos at dst, sin
// at dst + 128 * dh / 2 floats, by `nthreads` threads with 16-byte loads,
// four of a thread's loads per table in flight before its stores (one memory
// round trip per four rows of dh = 64 per thread, instead of one dependent
// load per float4 of the gradient).  False (nothing copied) when the tables
// are absent or not 16-byte aligned; the caller then reads them from
// global memory.
__device__ __forceinline__ bool rope_rows_to_smem(uint32_t dst, const float* ct, const float* st,
                                                  int64_t tab_row0, int rows, int dh, int t,
                                                  int nthreads) {
  if (ct == nullptr || ((reinterpret_cast<uintptr_t>(ct) | reinterpret_cast<uintptr_t>(st)) & 15))
    return false;
  const int half = dh / 2, n4 = rows * half / 4;
  const float4* c4 = reinterpret_cast<const float4*>(ct + tab_row0 * half);
  const float4* s4 = reinterpret_cast<const float4*>(st + tab_row0 * half);
  const uint32_t sin_dst = dst + (uint32_t)(128 * half * 4);
  for (int i0 = t; i0 < n4; i0 += 4 * nthreads) {
    float4 c[4], sn[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int i = i0 + u * nthreads;
      if (i < n4) {
        c[u] = __ldg(c4 + i);
        sn[u] = __ldg(s4 + i);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int i = i0 + u * nthreads;
      if (i < n4) {
        sts128(dst + 16u * (uint32_t)i, c[u]);
        sts128(sin_dst + 16u * (uint32_t)i, sn[u]);
      }
    }
  }
  return true;
}
// grad_rotate4 with the table entries of row r (pairs 2 c4, 2 c4 + 1) read
// from a rope_rows_to_smem copy; the same arithmetic.
__device__ __forceinline__ void grad_rotate4_smem(float4& v, float scale, uint32_t tab, int r,
                                                  int c4, int half) {
  float x[4] = {rn_mul(v.x, scale), rn_mul(v.y, scale), rn_mul(v.z, scale), rn_mul(v.w, scale)};
  const uint32_t off = 4u * (uint32_t)(r * half + 2 * c4);
  float2 c, sn;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(c.x), "=f"(c.y) : "r"(tab + off));
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];"
               : "=f"(sn.x), "=f"(sn.y)
               : "r"(tab + (uint32_t)(128 * half * 4) + off));
  const float cv[2] = {c.x, c.y}, sv[2] = {sn.x, sn.y};
#pragma unroll
  for (int pr = 0; pr < 2; pr++) {
    const float x0 = x[2 * pr], x1 = x[2 * pr + 1];
    x[2 * pr] = rn_add(rn_mul(x0, cv[pr]), rn_mul(x1, sv[pr]));
    x[2 * pr + 1] = rn_add(-rn_mul(x0, sv[pr]), rn_mul(x1, cv[pr]));
  }
  v = make_float4(x[0], x[1], x[2], x[3]);
}

// Number of entries of the ascending array a[0..n) that are <= x (le) or < x
// (!le), found by a 32-ary search of the calling warp (every lane gets the
// result): each round loads 32 entries at once and narrows the bracket 32-fold,
// two dependent load rounds for n <= 1024.
__device__ __forceinline__ int warp_count(const int64_t* a, int n, int64_t x, bool le) {
  const int lane = threadIdx.x & 31;
  int lo = 0, hi = n;  // the count lies in [lo, hi]
  while (hi - lo > 32) {
    const int step = (hi - lo + 31) / 32;
    const int idx = lo + lane * step;
    const bool in = idx < hi;
    const int64_t v = in ? a[idx] : 0;
    const unsigned below = __ballot_sync(0xffffffffu, in && (le ? v <= x : v < x));
    const int c = __popc(below);  // a prefix of the lanes, as a is ascending
    if (c == 0) return lo;        // a[lo] already fails
    const int last = lo + (c - 1) * step;
    lo = last + 1;
    hi = min(hi, last + step);
  }
  const int idx = lo + lane;
  const bool in = idx < hi;
  const int64_t v = in ? a[idx] : 0;
  return lo + __popc(__ballot_sync(0xffffffffu, in && (le ? v <= x : v < x)));
}

// Part `part` of a 3xTF32 operand pair: the TF32 hi value (part 0) or the
// residual (part 1) of every element, in place.
template <int N>
__device__ __forceinline__ void split_part(float (&v)[N], int part) {
#pragma unroll
  for (int i = 0; i < N; i++) {
    float h, l;
    tf32_split(v[i], h, l);
    v[i] = part == 0 ? h : l;
  }
}

// Named barrier over the first `threads` threads (warps 0..threads/32-1).
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Bounded wait that also gives up when another role of the CTA has aborted
// (*abort set); on a timeout it records the error and raises *abort.
__device__ __forceinline__ bool role_wait(uint32_t bar, uint32_t parity, int* error,
                                          volatile int* abort) {
  if (mbar_try(bar, parity)) return true;
  const long long start = clock64();
  for (int n = 0;; n++) {
    if (mbar_try(bar, parity)) return true;
    if ((n & 63) == 63) {
      if (*abort) return false;
      if (clock64() - start > kWaitCycles) {
        atomicExch(error, 0x6e6d);
        *abort = 1;
        return false;
      }
    }
  }
}

}  // namespace etb
