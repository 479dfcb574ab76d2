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
// (backward; +inf for a row with no admitted key).
struct AttnWs {
  float *qh, *ql, *kh, *kl, *vh, *vl, *doh, *dol, *lse2;
};
inline AttnWs attn_ws(const AttnParams& p) {
  const size_t nq = (size_t)p.B * p.Hq * p.Tq * p.Dh, nk = (size_t)p.B * p.Hkv * p.Tk * p.Dh;
  AttnWs w;
  w.qh = p.ws;
  w.ql = w.qh + nq;
  w.kh = w.ql + nq;
  w.kl = w.kh + nk;
  w.vh = w.kl + nk;
  w.vl = w.vh + nk;
  w.doh = w.vl + nk;
  w.dol = w.doh + nq;
  w.lse2 = w.dol + nq;
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

}  // namespace etb
