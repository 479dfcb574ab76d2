// Shared host/device helpers for libet_b200 (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "eshkol_b200/et_b200.h"

namespace etb {

// Kernels launched by this library since load; sampled by callers to count
// the launches inside a timed region.
extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

inline int32_t set_error(et_kernel_error *e, uint32_t category, uint32_t code,
                         const char *operation, const char *message) {
  if (e != nullptr) {
    memset(e, 0, sizeof(*e));
    e->category = category;
    e->code = code;
    snprintf(e->operation, sizeof(e->operation), "%s", operation ? operation : "et-b200");
    snprintf(e->message, sizeof(e->message), "%s", message ? message : "error");
  }
  return (int32_t)category;
}

inline int32_t cuda_error(et_kernel_error *e, cudaError_t status, const char *operation) {
  char text[160];
  snprintf(text, sizeof(text), "CUDA: %s", cudaGetErrorString(status));
  return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_PROVIDER_REJECTED, operation, text);
}

inline unsigned ceil_div(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

// Number of SMs of the current device (cached per device id).
int sm_count();

// Device word (one per GPU) that bounded device-side waits set when they
// give up; host entry points read and clear it.
int* device_error_word();

// ---- correctly rounded f32 arithmetic without contraction (device) -----
__device__ __forceinline__ float rn_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float rn_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float rn_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float rn_div(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float rn_sqrt(float a) { return __fsqrt_rn(a); }

// v = hi + lo exactly, hi = v rounded to the nearest TF32 value (10 explicit
// mantissa bits; magnitudes that would round up to infinity are truncated
// instead), the operand pair of the 3xTF32 tensor-core GEMMs.
__device__ __forceinline__ void tf32_split(float v, float& hi, float& lo) {
  uint32_t b = __float_as_uint(v);
  if ((b & 0x7f800000u) != 0x7f800000u) {
    const uint32_t r = (b + 0x1000u) & 0xffffe000u;
    b = ((r & 0x7f800000u) == 0x7f800000u) ? (b & 0xffffe000u) : r;
  }
  hi = __uint_as_float(b);
  lo = v - hi;
}

// ---- split-f16 operand pairs ---------------------------------------------
// A GEMM operand x may be stored as two IEEE binary16 arrays (hi, lo) with
// x 2^e = hi + lo + r, |r| <= 2^-22 |x 2^e| while x 2^e stays within binary16's
// normal range: hi = x 2^e rounded to binary16 (11 significant bits) and lo =
// the rounded remainder (another 11).  e is a per-tensor power-of-two scale
// read from device memory; the GEMM multiplies its accumulator by
// 2^-(e_A + e_B), which is exact.  Three tcgen05 kind::f16 products
// (hi hi + hi lo + lo hi, the split-f16 scheme of Ootomo & Yokota, 2022)
// then carry the same ~2^-22 operand accuracy as the 3xTF32 scheme at twice
// its tensor-core rate.
struct OperandScale {
  const int* exp;   // e of the output tensor (f16 != 0)
  unsigned* amax;   // optional: max |x| over the tensor (f32 bits, atomicMax)
  int f16;          // 1: write a binary16 pair, 0: the TF32 (hi, lo) f32 pair
};
// 2^e for e in [-126, 127] (exact).
__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }
__device__ __forceinline__ void f16_split(float xs, uint16_t& hi, uint16_t& lo) {
  const __half h = __float2half_rn(xs);
  hi = __half_as_ushort(h);
  lo = __half_as_ushort(__float2half_rn(xs - __half2float(h)));
}
// Four consecutive values: x 2^e as binary16 hi / lo quads (8-byte stores).
// (packed conversions, two values per instruction; each value rounded exactly
// as f16_split rounds it)
__device__ __forceinline__ void f16_store4(uint16_t* hi, uint16_t* lo, int64_t off, float4 x,
                                           float s) {
  const float a = x.x * s, b = x.y * s, c = x.z * s, d = x.w * s;
  const __half2 h01 = __floats2half2_rn(a, b), h23 = __floats2half2_rn(c, d);
  const float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
  const __half2 l01 = __floats2half2_rn(a - b01.x, b - b01.y);
  const __half2 l23 = __floats2half2_rn(c - b23.x, d - b23.y);
  *reinterpret_cast<uint2*>(hi + off) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
  *reinterpret_cast<uint2*>(lo + off) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
}
// binary16 values in the low / high half of a 32-bit word
__device__ __forceinline__ float half_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float half_hi(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ float abs_max4(float m, float4 x) {
  return fmaxf(fmaxf(m, fmaxf(fabsf(x.x), fabsf(x.y))), fmaxf(fabsf(x.z), fabsf(x.w)));
}
// Warp-wide max of m (non-negative, NaN propagating as the largest value)
// into *slot; every lane of the warp must call it.
__device__ __forceinline__ void amax_record_warp(unsigned* slot, float m) {
  unsigned b = (m != m) ? 0x7fffffffu : __float_as_uint(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
  if ((threadIdx.x & 31) == 0 && slot != nullptr && b != 0u) atomicMax(slot, b);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reduction helpers (blockDim.x multiple of 32, <= 1024); lanes
// past the warp count contribute Op's identity.
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* scratch, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < warps ? scratch[lane] : Op::template identity<T>();
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) scratch[0] = v;
  }
  __syncthreads();
  T r = scratch[0];
  __syncthreads();
  return r;
}

struct AddOp {
  template <typename T> __device__ __forceinline__ T operator()(T a, T b) const { return a + b; }
  template <typename T> __device__ __forceinline__ static T identity() { return T(0); }
};
struct MaxOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
  template <typename T> __device__ __forceinline__ static T identity() { return -INFINITY; }
};

}  // namespace etb
