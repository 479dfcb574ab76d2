// Binary16-pair tcgen05 pieces shared by the attention kernels that carry
// their operands as binary16 hi / lo pairs with per-tensor power-of-two
// scales (attention_f16.cu forward, attention_bwd_f16.cu backward).
#pragma once

#include <cuda_fp16.h>

#include "attention_tc.cuh"

namespace etb {
namespace f16att {

// ---- binary16 tcgen05 helpers -----------------------------------------------------

// kind::f16 instruction descriptor: f16 A and B, f32 accumulate, M = 128,
// N = n, A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1).
__host__ __device__ constexpr uint32_t idesc_f16_m128(int n, int b_mn) {
  return (1u << 4) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// A from TMEM (two binary16 elements per column), B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

// A binary16 [rows, DH] tile staged by TMA with the 128-byte swizzle: DH/64
// chunks of `rows` rows x 128 B.  K-major view (K = DH): slice j (16 k) at
// chunk j / 4, byte 32 (j % 4) of each row; 8-row groups 1 KB apart.
template <int ROWS>
__device__ __forceinline__ uint64_t kdesc16(uint32_t tile, int j) {
  return sdesc(tile + (uint32_t)(j >> 2) * (uint32_t)ROWS * 128u + (uint32_t)(j & 3) * 32u, 16u,
               1024u, 2u);
}
// MN-major view of the same tile (MN = DH, K = rows): per 64-wide MN chunk
// `rows` k-rows of 128 B, chunks ROWS x 128 B apart (LBO), 8-row groups 1 KB
// apart (SBO); slice j (16 k-rows) at +2 KB j.
template <int ROWS>
__device__ __forceinline__ uint64_t mdesc16(uint32_t tile, int j) {
  return sdesc(tile + 2048u * (uint32_t)j, (uint32_t)ROWS * 128u, 1024u, 2u);
}

// hi / lo binary16 pair of (a, b) (already scaled), two elements per word,
// the first in the low half.
__device__ __forceinline__ void pair2(float a, float b, float& hi, float& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
  hi = __uint_as_float(*reinterpret_cast<const uint32_t*>(&h));
  lo = __uint_as_float(*reinterpret_cast<const uint32_t*>(&l));
}
// 32 values (scaled by s) -> their packed hi (16 words) and lo (16 words).
__device__ __forceinline__ void pack_pairs(const float (&v)[32], float s, float (&hi)[16],
                                           float (&lo)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i++) pair2(v[2 * i] * s, v[2 * i + 1] * s, hi[i], lo[i]);
}

// Row `row` of a binary16 [128, DH] tile (DH/64 chunks of 128 rows x 128 B,
// 128-byte swizzle) -> DH/2 TMEM columns of this thread's lane from `col`.
template <int DH>
__device__ __forceinline__ void tile_row16_to_tmem(uint32_t tile, int row, uint32_t trow,
                                                   uint32_t col) {
#pragma unroll
  for (int c = 0; c < DH / 64; c++) {
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

// ---- exponents --------------------------------------------------------------------

// 2^e with max |x| 2^e in [2^14, 2^15) (e = 0 for a zero or non-finite max),
// clamped to [-60, 60] like the linear GEMMs' operand scales.
__device__ __forceinline__ int pair_exponent(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 0;
  int k;
  frexpf(amax, &k);
  return max(-60, min(60, 15 - k));
}
struct Exps {
  int q, k, v, g, ds;
};
// amax[0..3]: max |x| of Q, K, V, dO (f32 bits).  fixed (non-null): the
// producers chose the exponents of Q, K, V, dO (fixed[0..3]); dS's still
// comes from this call's maxima of V and dO, which bound it.
__device__ __forceinline__ Exps exps_of(const unsigned* amax, int dh,
                                       const int* fixed = nullptr) {
  const float aq = __uint_as_float(amax[0]), ak = __uint_as_float(amax[1]);
  const float av = __uint_as_float(amax[2]), ag = __uint_as_float(amax[3]);
  Exps x;
  if (fixed != nullptr) {
    x.q = fixed[0];
    x.k = fixed[1];
    x.v = fixed[2];
    x.g = fixed[3];
  } else {
    x.q = pair_exponent(aq);
    x.k = pair_exponent(ak);
    x.v = pair_exponent(av);
    x.g = pair_exponent(ag);
  }
  // bound 2^e in [2^13, 2^14)
  x.ds = pair_exponent(2.0f * (float)dh * ag * av) - 1;
  return x;
}

// VEC consecutive floats: with VLOAD one 16-byte (VEC 4) or 8-byte (VEC 2)
// load, the address aligned to it; without, one float at a time.
template <int VEC, bool VLOAD = true>
__device__ __forceinline__ void load_vec(const float* src, float (&v)[VEC]) {
  if constexpr (!VLOAD) {
#pragma unroll
    for (int u = 0; u < VEC; u++) v[u] = src[u];
  } else if constexpr (VEC == 4) {
    const float4 f = *reinterpret_cast<const float4*>(src);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else if constexpr (VEC == 2) {
    const float2 f = *reinterpret_cast<const float2*>(src);
    v[0] = f.x; v[1] = f.y;
  } else {
#pragma unroll
    for (int u = 0; u < VEC; u++) v[u] = src[u];
  }
}

}  // namespace f16att

// Whether rows of t (and of `lo`, same strides) can be read as float4: the
// base and every stride 16-byte aligned (head_dim a multiple of 4 is implied
// by the binary16 kernels' 64 / 128).
inline bool rows_vec4(const AttnTensor& t, const float* lo) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(t.ptr) | reinterpret_cast<uintptr_t>(lo) |
                         (uintptr_t)(t.sb * 4) | (uintptr_t)(t.sh * 4) | (uintptr_t)(t.st * 4);
  return (bits & 15) == 0;
}
// The same for 8-byte (float2) reads; otherwise the kernels read one float
// at a time.
inline bool rows_vec2(const AttnTensor& t, const float* lo) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(t.ptr) | reinterpret_cast<uintptr_t>(lo) |
                         (uintptr_t)(t.sb * 4) | (uintptr_t)(t.sh * 4) | (uintptr_t)(t.st * 4);
  return (bits & 7) == 0;
}

}  // namespace etb
