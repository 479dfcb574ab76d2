// N2/N3K linear contractions: C[m,n] = sum_k A(m,k) B(n,k) (+ bias) (+ C).
//
// The three linear products of native/n2_primitives_provider.c:347-419 map
// onto this one operation with different operand majorness:
//   forward  y  = x W^T : A = x  (K-major), B = W  (K-major)
//   backward dX = dY W  : A = dY (K-major), B = W  (N-major)
//   backward dW = dY^T x: A = dY (M-major), B = x  (N-major)
//
// Tensor-core paths (sm_100a), persistent and warp-specialised:
// * gemm_tc2_kernel (the f32-grade modes): clusters of two CTAs on the two
//   SMs of a TPC compute 256 x 256 tiles with tcgen05.mma.cta_group::2; warp
//   0 issues TMA loads (128-byte swizzle, no multicast) into a 3-deep ring of
//   64 KB per SM, warp 1 allocates the pair's TMEM and the leader's lane 0
//   issues the MMAs, warps 2-9 drain the double-buffered accumulator through
//   a shared-memory transpose and apply the fused epilogue (plain, residual,
//   GELU forward / backward, QKV attention operands, dO operands).  Operands
//   are (hi, lo) pairs and every algorithmic product is three MMAs (A B +
//   A B_lo + A_lo B): TF32 pairs with kind::tf32 (K 8 per instruction, 32 k
//   per 128-byte row) or binary16 pairs scaled by a per-tensor power of two
//   with kind::f16 (K 16, 64 k per row; twice the rate, the same accuracy;
//   the epilogue multiplies by 2^-(e_A + e_B)).  One instance per epilogue
//   mode keeps each kernel's unrolled epilogue small.
// * gemm_tc_kernel: the single-CTA 128 x 256 kernel of the single-TF32 mode.
// Two TMEM accumulators (2 x BN columns) let the epilogue of one tile overlap
// the main loop of the next.  Every mbarrier wait is bounded (about two
// seconds of clock) and reports through the device error word instead of
// hanging.
//
// FFMA path: a plain 128x128 register-tiled kernel, used for the f32 mode and
// for shapes the tensor-core path does not take (unaligned strides, K = 0).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "ops.cuh"
#include "tcgen05.cuh"

namespace etb {



namespace {

// ============================================================== FFMA path

constexpr int SB_M = 128, SB_N = 128, SB_K = 8;

__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmArgs g) {
  __shared__ __align__(16) float As[SB_K][SB_M];
  __shared__ __align__(16) float Bs[SB_K][SB_N];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < g.K; k0 += SB_K) {
    for (int i = tid; i < SB_M * SB_K; i += 256) {
      int mm, kk;
      if (g.a_kmajor) { mm = i / SB_K; kk = i % SB_K; } else { kk = i / SB_M; mm = i % SB_M; }
      const int m = m0 + mm, k = k0 + kk;
      float v = 0.0f;
      if (m < g.M && k < g.K) {
        const int64_t at = g.a_kmajor ? (int64_t)m * g.lda + k : (int64_t)k * g.lda + m;
        v = g.A[at];
        if (g.A_lo) v += g.A_lo[at];  // hi + lo restores the f32 operand exactly
      }
      As[kk][mm] = v;
    }
    for (int i = tid; i < SB_N * SB_K; i += 256) {
      int nn, kk;
      if (g.b_kmajor) { nn = i / SB_K; kk = i % SB_K; } else { kk = i / SB_N; nn = i % SB_N; }
      const int n = n0 + nn, k = k0 + kk;
      float v = 0.0f;
      if (n < g.N && k < g.K) {
        const int64_t at = g.b_kmajor ? (int64_t)n * g.ldb + k : (int64_t)k * g.ldb + n;
        v = g.B[at];
        if (g.B_lo) v += g.B_lo[at];
      }
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SB_K; kk++) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4 + 64]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int m = m0 + ty * 8 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int n = n0 + tx * 4 + (j & 3) + (j >> 2) * 64;
      if (n >= g.N) continue;
      float v = acc[i][j];
      if (g.bias) v += g.bias[n];
      float* c = g.C + (int64_t)m * g.ldc + n;
      if (g.accumulate) v += *c;
      *c = v;
    }
  }
}

// ============================================================== tcgen05 path

constexpr int TC_BM = 128;
constexpr int TC_THREADS = 192;
constexpr int TC2_THREADS = 320;  // pair kernel: producer, MMA and 8 epilogue warps

// Operand tiles of one K block of BK f32 (BK = 32: 128-byte rows; BK = 16:
// 64-byte rows).  Descriptor of K-slice j (8 k) of a staged tile:
//   K-major : 8-row swizzle atoms of BK*4-byte rows (SBO = 8 rows); the
//             128-byte swizzle for BK 32, the 64-byte swizzle for BK 16;
//             slice j at +32j bytes within the row.
//   MN-major: per 32-wide MN chunk BK k-rows of 128 B (32-byte-atom 128-byte
//             swizzle), chunks BK*128 bytes apart (LBO), 4-row groups 512 B
//             apart (SBO); slice j (8 k-rows) at +1024j bytes.
template <int BK>
__device__ __forceinline__ uint64_t tile_desc(uint32_t base, int mn_major, int j) {
  if (mn_major) return sdesc(base + 1024u * j, (uint32_t)BK * 128u, 512u, 1u);
  return BK == 32 ? sdesc(base + 32u * j, 16u, 1024u, 2u) : sdesc(base + 32u * j, 16u, 512u, 4u);
}

struct TcArgs {
  int M, N, K;
  float* C;
  int64_t ldc;
  const float* bias;
  int accumulate;
  int a_mn, b_mn;
  int tiles_m, tiles_n;
  // split-K: work unit u covers tile u % tiles over K blocks
  // [s * kb_per_split, min(nkb, (s + 1) * kb_per_split)), s = u / tiles, and
  // writes its raw sum to partial + s * M * N (row stride N)
  int splits, kb_per_split;
  // K blocks per accumulation chunk (>= kb_per_split: one chunk); the
  // epilogue warps add the chunks of a tile in f32 in chunk_ws (per CTA 8
  // warps x 32 lanes x BN / 2 floats)
  int chunk_kb;
  float* chunk_ws;
  float* partial;
  // fused epilogue (pair kernel): mode, auxiliary input, extra outputs, and
  // the per-(tile, warp) column partials of the GELU_BWD mode
  int epilogue;
  const float* aux;
  float* out2;
  float* out3;
  float* colpart;
  // pair kernel: every row pointer and ldc allow float4 access and N % 4 == 0,
  // so the epilogue goes through the shared-memory transpose (coalesced rows)
  int staged;
  QkvPrep qkv;          // GEMM_EPI_QKV (staged epilogue only)
  AttnGradPrep dprep;   // GEMM_EPI_ATTN_DO (staged epilogue only)
  int* error;
  // split-f16 operands (pair kernel): binary16 (hi, lo) tiles, 64 k per
  // 128-byte row, and the accumulator scaled by 2^-(*exp_a + *exp_b)
  int f16;
  const int* exp_a;
  const int* exp_b;
  // GELU_FWD / GELU_BWD operand-pair outputs: binary16 with this scale, and
  // their max |x| (either format)
  OperandScale out_sc;
  // QKV / ATTN_DO: C itself is not stored (the attention operands are its
  // only consumers)
  int skip_c;
  // GELU_FWD: C = GELU'(u) instead of u; GELU_BWD: aux holds GELU'(u)
  int gelu_slope_c;
};

__device__ __forceinline__ float gelu_value(float v) {  // n2_primitives_provider.c:545-583
  const float inv_sqrt_2 = 0x1.6a09e6p-1f;
  const float e = erff(rn_mul(v, inv_sqrt_2));
  return rn_mul(rn_mul(0.5f, v), rn_add(1.0f, e));
}
// GELU(v) and GELU'(v) with one erf: the same operations as gelu_value and
// gelu_slope, so the results are identical to theirs.
__device__ __forceinline__ void gelu_both(float v, float& g, float& slope) {
  const float inv_sqrt_2 = 0x1.6a09e6p-1f, inv_sqrt_2pi = 0x1.988454p-2f;
  const float e = erff(rn_mul(v, inv_sqrt_2));
  g = rn_mul(rn_mul(0.5f, v), rn_add(1.0f, e));
  const float cdf = rn_mul(0.5f, rn_add(1.0f, e));
  const float density = rn_mul(expf(-rn_mul(0.5f, rn_mul(v, v))), inv_sqrt_2pi);
  slope = rn_add(cdf, rn_mul(v, density));
}
__device__ __forceinline__ float gelu_slope(float v) {
  const float inv_sqrt_2 = 0x1.6a09e6p-1f, inv_sqrt_2pi = 0x1.988454p-2f;
  const float cdf = rn_mul(0.5f, rn_add(1.0f, erff(rn_mul(v, inv_sqrt_2))));
  const float density = rn_mul(expf(-rn_mul(0.5f, rn_mul(v, v))), inv_sqrt_2pi);
  return rn_add(cdf, rn_mul(v, density));
}

// One halving stage of warp_column_sums: lanes with bit K set keep the upper
// K of their first 2K values, the others the lower K, and add the partner's.
template <int K>
__device__ __forceinline__ void column_sum_stage(float (&v)[32], int lane) {
  const bool upper = (lane & K) != 0;
#pragma unroll
  for (int i = 0; i < K; i++) {
    const float send = upper ? v[i] : v[i + K];
    const float keep = upper ? v[i + K] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, K);
  }
}
// Lane l of the warp receives the sum over the 32 lanes of v[l] (a
// reduce-scatter: 31 shuffles for 32 columns).
__device__ __forceinline__ float warp_column_sums(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
  column_sum_stage<16>(v, lane);
  column_sum_stage<8>(v, lane);
  column_sum_stage<4>(v, lane);
  column_sum_stage<2>(v, lane);
  column_sum_stage<1>(v, lane);
  return v[0];
}

// Grouped rasterisation: 16 M-tiles per group so the CTAs in flight share
// their A row blocks and B column blocks through L2.
__device__ __forceinline__ void raster(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  constexpr int G = 16;
  const int per_group = G * tiles_n;
  const int group = tile / per_group;
  const int first = group * G;
  const int gm = min(tiles_m - first, G);
  const int in = tile % per_group;
  tm = first + in % gm;
  tn = in / gm;
}

template <int BN, int STAGES, bool THREE, int BK>
struct TcLayout {
  static constexpr int A_BYTES = TC_BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int OPS = THREE ? 2 : 1;
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * OPS;
  static constexpr int RING_BYTES = STAGE_BYTES * STAGES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = RING_BYTES + BAR_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
};

template <int BN, int STAGES, bool THREE, int BK>
__global__ void __launch_bounds__(TC_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap ta_lo,
               const __grid_constant__ CUtensorMap tb, const __grid_constant__ CUtensorMap tb_lo,
               TcArgs args) {
  using L = TcLayout<BN, STAGES, THREE, BK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::RING_BYTES);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2]; then the TMEM slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + 2);

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int nkb = (args.K + BK - 1) / BK;
  const int tiles = args.tiles_m * args.tiles_n;
  const int units = tiles * args.splits;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t armed = 0;  // bitmask of stages with an armed phase in flight
      uint32_t armed_phase[STAGES];
      for (int s = 0; s < STAGES; s++) armed_phase[s] = 0;
      for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
        const int tile = unit % tiles, split = unit / tiles;
        int tm, tn;
        raster(tile, args.tiles_m, args.tiles_n, tm, tn);
        const int m0 = tm * TC_BM, n0 = tn * BN;
        const int kb_end = min(nkb, (split + 1) * args.kb_per_split);
        for (int kb = split * args.kb_per_split; kb < kb_end; kb++) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, args.error)) { ok = false; break; }
          const uint32_t full = full0 + 8 * stage;
          mbar_expect_tx(full, L::STAGE_BYTES);
          armed |= 1u << stage;
          armed_phase[stage] = phase;
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
          const int k0 = kb * BK;
#pragma unroll
          for (int op = 0; op < L::OPS; op++) {
            const CUtensorMap* mA = op == 0 ? &ta : &ta_lo;
            const CUtensorMap* mB = op == 0 ? &tb : &tb_lo;
            const uint32_t da = sa + op * (L::A_BYTES + L::B_BYTES);
            const uint32_t db = sb + op * (L::A_BYTES + L::B_BYTES);
            if (args.a_mn) {
              for (int c = 0; c < TC_BM / 32; c++)
                tma_load_2d(da + (uint32_t)BK * 128u * c, mA, full, m0 + 32 * c, k0);
            } else {
              tma_load_2d(da, mA, full, k0, m0);
            }
            if (args.b_mn) {
              for (int c = 0; c < BN / 32; c++)
                tma_load_2d(db + (uint32_t)BK * 128u * c, mB, full, n0 + 32 * c, k0);
            } else {
              tma_load_2d(db, mB, full, k0, n0);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // drain: let every armed copy land before the CTA can exit
        for (int s = 0; s < STAGES; s++)
          if (armed & (1u << s)) mbar_wait(full0 + 8 * s, armed_phase[s], args.error);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)args.a_mn << 15) |
                             ((uint32_t)args.b_mn << 16) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(TC_BM >> 4) << 24);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
        const int split = unit / tiles;
        if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1u, args.error)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int kb_begin = split * args.kb_per_split;
        const int kb_end = min(nkb, kb_begin + args.kb_per_split);
        for (int kb = kb_begin; kb < kb_end; kb++) {
          if (!mbar_wait(full0 + 8 * stage, phase, args.error)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int j = 0; j < BK / 8; j++) {
            const uint64_t a = tile_desc<BK>(sa, args.a_mn, j);
            const uint64_t b = tile_desc<BK>(sb, args.b_mn, j);
            umma_tf32(d_tmem, a, b, idesc, (kb > kb_begin || j > 0) ? 1u : 0u);
            if (THREE) {
              const uint32_t lo = L::A_BYTES + L::B_BYTES;
              const uint64_t alo = tile_desc<BK>(sa + lo, args.a_mn, j);
              const uint64_t blo = tile_desc<BK>(sb + lo, args.b_mn, j);
              umma_tf32(d_tmem, a, blo, idesc, 1u);
              umma_tf32(d_tmem, alo, b, idesc, 1u);
            }
          }
          umma_commit(empty0 + 8 * stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(tfull0 + 8 * acc);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5 own TMEM lanes 32*(warp%4)..
    const int lane_base = 32 * (warp & 3);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
      const int tile = unit % tiles, split = unit / tiles;
      // one lane observes the phase; the warp stays converged for tcgen05.ld
      int ok = 1;
      if (lane == 0) ok = mbar_wait(tfull0 + 8 * acc, acc_phase, args.error) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      int tm, tn;
      raster(tile, args.tiles_m, args.tiles_n, tm, tn);
      const int m = tm * TC_BM + lane_base + lane;
      const int n_tile = tn * BN;
      // split-K units write their raw sum to their partial buffer
      const bool part = args.splits > 1;
      float* cbase = part ? args.partial + (int64_t)split * args.M * args.N : args.C;
      const int64_t ldc = part ? (int64_t)args.N : args.ldc;
      const float* bias = part ? nullptr : args.bias;
      const int accumulate = part ? 0 : args.accumulate;
      float* crow = cbase + (int64_t)m * ldc;
      const bool vec = ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(cbase) & 15) == 0);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN + c), v);
        if (m < args.M) {
          const int n0 = n_tile + c;
          if (vec && n0 + 32 <= args.N) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 r = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
              if (bias) {
                r.x += bias[n0 + i];
                r.y += bias[n0 + i + 1];
                r.z += bias[n0 + i + 2];
                r.w += bias[n0 + i + 3];
              }
              float4* dst = reinterpret_cast<float4*>(crow + n0 + i);
              if (accumulate) {
                const float4 o = *dst;
                r.x += o.x; r.y += o.y; r.z += o.z; r.w += o.w;
              }
              *dst = r;
            }
          } else {
            for (int i = 0; i < 32; i++) {
              const int n = n0 + i;
              if (n >= args.N) break;
              float r = v[i];
              if (bias) r += bias[n];
              if (accumulate) r += crow[n];
              crow[n] = r;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
}

// Section (0 Q, 1 K, 2 V), head and column within the head of qkv column n.
__device__ __forceinline__ void qkv_column(const QkvPrep& q, int n, int& sec, int& h, int& j) {
  const int dq = q.Hq * q.Dh, dk = q.Hkv * q.Dh;
  int hc;
  if (n < dq) { sec = 0; hc = n; }
  else if (n < dq + dk) { sec = 1; hc = n - dq; }
  else { sec = 2; hc = n - dq - dk; }
  h = hc / q.Dh;
  j = hc - h * q.Dh;
}
// Attention operands of qkv columns [n, n + 4) (section sec, head h, column
// j of the head; j % 4 == 0) of token t of sequence b, from the values x = y +
// bias as stored to C: head-major TF32 hi / lo copies, with the RoPE rotation
// of the pairs (j, j + 1), (j + 2, j + 3) for Q and K (attention_tc.cu
// attn_prepare_kernel computes the same values), or with q.q16h the binary16
// pair of the rotated values times s (2^exps[sec]).  The host tables' two
// entries are one aligned float2 (Dh / 2 even).  Returns max |x| of the four
// stored values.
__device__ __forceinline__ float qkv_prep_store(const QkvPrep& q, int sec, int h, int j, int b,
                                                int t, float4 x, float s16) {
  const float* ct = sec == 0 ? q.q_cos : (sec == 1 ? q.k_cos : nullptr);
  if (ct != nullptr) {
    const float* st = sec == 0 ? q.q_sin : q.k_sin;
    const int batched = sec == 0 ? q.q_rope_batched : q.k_rope_batched;
    const int64_t ti = (int64_t)(batched ? b * q.T + t : t) * (q.Dh >> 1) + (j >> 1);
    const float2 c = __ldg(reinterpret_cast<const float2*>(ct + ti));
    const float2 s = __ldg(reinterpret_cast<const float2*>(st + ti));
    const float x0 = rn_sub(rn_mul(x.x, c.x), rn_mul(x.y, s.x));
    const float x1 = rn_add(rn_mul(x.x, s.x), rn_mul(x.y, c.x));
    const float x2 = rn_sub(rn_mul(x.z, c.y), rn_mul(x.w, s.y));
    const float x3 = rn_add(rn_mul(x.z, s.y), rn_mul(x.w, c.y));
    x = make_float4(x0, x1, x2, x3);
  }
  const int H = sec == 0 ? q.Hq : q.Hkv;
  const int64_t o = (((int64_t)b * H + h) * q.T + t) * q.Dh + j;
  if (q.q16h != nullptr) {
    uint16_t* hi = sec == 0 ? q.q16h : (sec == 1 ? q.k16h : q.v16h);
    uint16_t* lo = sec == 0 ? q.q16l : (sec == 1 ? q.k16l : q.v16l);
    f16_store4(hi, lo, o, x, s16);
    return abs_max4(0.0f, x);
  }
  float* hi = sec == 0 ? q.qh : (sec == 1 ? q.kh : q.vh);
  float* lo = sec == 0 ? q.ql : (sec == 1 ? q.kl : q.vl);
  float4 h4, l4;
  tf32_split(x.x, h4.x, l4.x);
  tf32_split(x.y, h4.y, l4.y);
  tf32_split(x.z, h4.z, l4.z);
  tf32_split(x.w, h4.w, l4.w);
  *reinterpret_cast<float4*>(hi + o) = h4;
  *reinterpret_cast<float4*>(lo + o) = l4;
  return abs_max4(0.0f, x);
}

// dO columns [j, j + 4) of head h, token t of sequence b, as the attention
// backward's head-major TF32 hi / lo operands (attention_bwd_tc.cu
// attn_bwd_prepare_kernel writes the same values), or with g.g16h the
// binary16 pair of dO s16 (s16 = 2^(*g_exp)).
__device__ __forceinline__ void attn_do_store(const AttnGradPrep& g, int h, int j, int b, int t,
                                              float4 x, float s16) {
  const int64_t o = (((int64_t)b * g.H + h) * g.T + t) * g.Dh + j;
  if (g.g16h != nullptr) {
    f16_store4(g.g16h, g.g16l, o, x, s16);
    return;
  }
  float4 h4, l4;
  tf32_split(x.x, h4.x, l4.x);
  tf32_split(x.y, h4.y, l4.y);
  tf32_split(x.z, h4.z, l4.z);
  tf32_split(x.w, h4.w, l4.w);
  *reinterpret_cast<float4*>(g.doh + o) = h4;
  *reinterpret_cast<float4*>(g.dol + o) = l4;
}

// ---- 2-SM (CTA pair) 3xTF32 kernel ---------------------------------------------
//
// A cluster of two CTAs on the two SMs of a TPC computes a 256 x BN output
// tile with tcgen05.mma.cta_group::2 (M = 256): CTA r holds A rows
// [128 r, 128 r + 128) and B rows [BN/2 r, BN/2 r + BN/2) of every K block in
// its own shared memory, and its TMEM receives output rows [128 r, 128 r + 128).
// Each SM's ring stage is then 64 KB instead of 96 KB, so three stages fit
// and hide the TMA latency that a two-stage 128 x 256 ring exposes.
//   both CTAs  warp 0: TMA into its own shared memory; the copies complete on
//              the leader CTA's full barrier (the leader expects both CTAs'
//              bytes); warp 1 allocates TMEM (cta_group::2, both CTAs);
//              warps 2-9: epilogue of its own 128 rows (warp w: TMEM lane
//              quadrant w % 4, column half (w - 2) / 4), then an arrive on the
//              leader's accumulator-empty barrier
//   leader     warp 1 lane 0 issues the MMAs and commits to the empty /
//              accumulator-full barriers of both CTAs (one commit per CTA)
// No TMA load uses cluster multicast.  All waits are bounded; after a
// timeout every thread still reaches the closing cluster barrier.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// TMA tile load whose completion may be signalled on the peer CTA's barrier.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t a, uint64_t b,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a, uint64_t b,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// binary16 tiles of 64 k (128-byte rows).  K-major: as the f32 tiles, slice j
// (16 k) at +32j bytes.  MN-major: per 64-wide MN chunk 64 k-rows of 128 B
// with the 128-byte swizzle; chunks 8 KB apart (LBO), 8-row groups 1 KB apart
// (SBO), slice j (16 k-rows) at +2 KB j.
__device__ __forceinline__ uint64_t tile_desc_f16(uint32_t base, int mn_major, int j) {
  if (mn_major) return sdesc(base + 2048u * j, 8192u, 1024u, 2u);
  return sdesc(base + 32u * j, 16u, 1024u, 2u);
}
// Arrives on `bar_cluster` (either CTA of the pair) once all prior MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

template <int BN, int STAGES>
struct Tc2Layout {
  static constexpr int BK = 32;
  static constexpr int A_BYTES = TC_BM * BK * 4;        // this CTA's 128 A rows
  static constexpr int B_BYTES = (BN / 2) * BK * 4;      // this CTA's BN/2 B rows
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * 2;  // hi and lo
  static constexpr int RING_BYTES = STAGE_BYTES * STAGES;
  // per epilogue warp a 32 x 32 f32 transpose buffer (16-byte chunks XOR-swizzled by row)
  static constexpr int STAGE_OUT_BYTES = 8 * 4096;
  static constexpr int SMEM_BYTES = RING_BYTES + 256 + STAGE_OUT_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  static_assert(SMEM_BYTES <= 232448, "shared memory above the 227 KB per-CTA limit");
};

// EPI: the fused epilogue mode this instance carries besides plain and
// residual (GEMM_EPI_PLAIN: none).  One instance per mode keeps each kernel's
// code (and registers) to what its epilogue needs: the epilogue warps' loop
// is unrolled, and a kernel holding every mode overflowed the instruction
// cache (ncu: "no_instruction" stalls).  VAR fixes the GELU modes' options
// at compile time for the same reason: bit 0 gelu_slope_c, bit 1 a binary16
// operand-pair output; kVarRuntime reads both from the arguments.
// The K chunks of one tile, for one epilogue warp of the pair kernel (its
// 32 TMEM lanes, BN / 2 columns from taddr0).  Each chunk's accumulator
// buffer is added into an f32 running sum and handed back to the MMA warp;
// the last chunk's buffer receives the total, and `acc` / `phase` are left on
// it for the epilogue.  The running sum lives in this warp's 16 KB of the
// global chunk scratch `run`, lane-major (column group q of lane l at
// run[(q * 32 + l) * 4]) so that each warp access is 512 contiguous bytes:
// the first chunk is stored, the middle ones are added with fire-and-forget
// reductions (red.add: round to nearest, applied in this thread's program
// order, since every element has one owner), and the last chunk reads the
// sum back once.  Returns false when a bounded wait gave up.
__device__ __forceinline__ void red_add4(float4* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}
__device__ __forceinline__ float4 ld_relaxed4(const float4* p) {
  float4 v;
  asm volatile("ld.relaxed.gpu.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
template <int BN>
__device__ __forceinline__ bool sum_k_chunks(uint32_t taddr0, int nchunks, uint32_t tfull0,
                                             uint32_t tempty_leader, int& acc,
                                             uint32_t& acc_phase, int* error, float* run) {
  static_assert(BN % 64 == 0, "pairs of 16-column groups");
  const int lane = threadIdx.x & 31;
  float4* r4 = reinterpret_cast<float4*>(run) + lane;
  for (int ch = 0; ch < nchunks; ch++) {
    const bool last = ch == nchunks - 1;
    // the last chunk: the running sums of the first two 16-column groups
    // load while its MMAs finish; later ones are issued one pair ahead
    float4 pa[4], pb[4];
    if (last) {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        pa[q] = ld_relaxed4(r4 + q * 32);
        pb[q] = ld_relaxed4(r4 + (4 + q) * 32);
      }
    }
    int ok = 1;
    if (lane == 0) ok = mbar_wait(tfull0 + 8 * acc, acc_phase, error) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return false;
    __syncwarp();
    tc_fence_after();
    const uint32_t taddr = taddr0 + (uint32_t)(acc * BN);
#pragma unroll 1
    for (int g = 0; g < BN / 32; g += 2) {
      float va[16], vb[16];
      tmem_ld16(taddr + 16u * g, va);
      tmem_ld16(taddr + 16u * (g + 1), vb);
      if (last) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          va[4 * q] = pa[q].x + va[4 * q];
          va[4 * q + 1] = pa[q].y + va[4 * q + 1];
          va[4 * q + 2] = pa[q].z + va[4 * q + 2];
          va[4 * q + 3] = pa[q].w + va[4 * q + 3];
          vb[4 * q] = pb[q].x + vb[4 * q];
          vb[4 * q + 1] = pb[q].y + vb[4 * q + 1];
          vb[4 * q + 2] = pb[q].z + vb[4 * q + 2];
          vb[4 * q + 3] = pb[q].w + vb[4 * q + 3];
        }
        if (g + 2 < BN / 32) {
#pragma unroll
          for (int q = 0; q < 4; q++) {
            pa[q] = ld_relaxed4(r4 + (4 * (g + 2) + q) * 32);
            pb[q] = ld_relaxed4(r4 + (4 * (g + 3) + q) * 32);
          }
        }
        tmem_st16(taddr + 16u * g, va);
        tmem_st16(taddr + 16u * (g + 1), vb);
      } else if (ch == 0) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          r4[(4 * g + q) * 32] = make_float4(va[4 * q], va[4 * q + 1], va[4 * q + 2], va[4 * q + 3]);
          r4[(4 * (g + 1) + q) * 32] =
              make_float4(vb[4 * q], vb[4 * q + 1], vb[4 * q + 2], vb[4 * q + 3]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          red_add4(r4 + (4 * g + q) * 32, va[4 * q], va[4 * q + 1], va[4 * q + 2], va[4 * q + 3]);
          red_add4(r4 + (4 * (g + 1) + q) * 32, vb[4 * q], vb[4 * q + 1], vb[4 * q + 2],
                   vb[4 * q + 3]);
        }
      }
    }
    if (last) break;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(tempty_leader + 8 * acc);
    if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
  }
  tmem_wait_st();
  return true;
}

constexpr int kVarRuntime = 4;
template <int BN, int STAGES, int EPI, int VAR>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC2_THREADS, 1)
gemm_tc2_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap ta_lo,
                const __grid_constant__ CUtensorMap tb, const __grid_constant__ CUtensorMap tb_lo,
                TcArgs args) {
  constexpr bool ATTN = EPI == GEMM_EPI_QKV || EPI == GEMM_EPI_ATTN_DO;
  constexpr bool K_QKV = EPI == GEMM_EPI_QKV, K_DO = EPI == GEMM_EPI_ATTN_DO;
  constexpr bool K_GF = EPI == GEMM_EPI_GELU_FWD, K_GB = EPI == GEMM_EPI_GELU_BWD;
  using L = Tc2Layout<BN, STAGES>;
  constexpr int BK = L::BK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::RING_BYTES);
  // bars: full[STAGES] (leader's used), empty[STAGES], tfull[2], tempty[2] (leader's used)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + 2);

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 16);  // 8 epilogue warps in each CTA
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's TMEM
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const bool f16 = args.f16 != 0;
  const int bke = f16 ? 2 * BK : BK;  // k per 128-byte row of a stage
  const int nkb = (args.K + bke - 1) / bke;
  const int tiles = args.tiles_m * args.tiles_n;  // tiles_m counts 256-row blocks
  const int units = tiles * args.splits;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  bool failed = false;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (both CTAs)
      const uint32_t full_leader = map_to_rank(full0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = cluster; ok && unit < units; unit += nclusters) {
        const int tile = unit % tiles, split = unit / tiles;
        int tm, tn;
        raster(tile, args.tiles_m, args.tiles_n, tm, tn);
        const int m0 = tm * 2 * TC_BM + (int)rank * TC_BM, n0 = tn * BN + (int)rank * (BN / 2);
        const int kb_end = min(nkb, (split + 1) * args.kb_per_split);
        for (int kb = split * args.kb_per_split; kb < kb_end; kb++) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, args.error)) { ok = false; break; }
          if (leader) mbar_expect_tx(full0 + 8 * stage, 2 * L::STAGE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
          const uint32_t fb = full_leader + 8 * stage;
          const int k0 = kb * bke;
          // MN-major tiles: one load per 128-byte-wide MN chunk of bke k-rows
          const int cw = f16 ? 64 : 32;
#pragma unroll
          for (int op = 0; op < 2; op++) {
            const CUtensorMap* mA = op == 0 ? &ta : &ta_lo;
            const CUtensorMap* mB = op == 0 ? &tb : &tb_lo;
            const uint32_t da = sa + op * (L::A_BYTES + L::B_BYTES);
            const uint32_t db = sb + op * (L::A_BYTES + L::B_BYTES);
            if (args.a_mn) {
              for (int c = 0; c < TC_BM / cw; c++)
                tma_load_2d_pair(da + (uint32_t)bke * 128u * c, mA, fb, m0 + cw * c, k0);
            } else {
              tma_load_2d_pair(da, mA, fb, k0, m0);
            }
            if (args.b_mn) {
              for (int c = 0; c < (BN / 2) / cw; c++)
                tma_load_2d_pair(db + (uint32_t)bke * 128u * c, mB, fb, n0 + cw * c, k0);
            } else {
              tma_load_2d_pair(db, mB, fb, k0, n0);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      failed = !ok;
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA)
      // operand format 0 = f16, 2 = tf32 (bits 7-9 A, 10-12 B); f32 accumulator
      const uint32_t fmt = f16 ? 0u : 2u;
      const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)args.a_mn << 15) |
                             ((uint32_t)args.b_mn << 16) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)((2 * TC_BM) >> 4) << 24);
      const uint32_t peer = 1;
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int unit = cluster; ok && unit < units; unit += nclusters) {
        const int split = unit / tiles;
        const int kb_begin = split * args.kb_per_split;
        const int kb_end = min(nkb, kb_begin + args.kb_per_split);
        // one accumulator buffer per K chunk (the epilogue warps add the
        // chunks in f32 registers: the tensor-pipe accumulation truncates, so
        // its error grows with the K it sums)
        for (int c0 = kb_begin; ok && c0 < kb_end; c0 += args.chunk_kb) {
          const int c1 = min(kb_end, c0 + args.chunk_kb);
          if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1u, args.error)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          for (int kb = c0; kb < c1; kb++) {
            if (!mbar_wait(full0 + 8 * stage, phase, args.error)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
            const uint32_t sb = sa + L::A_BYTES;
            const uint32_t lo = L::A_BYTES + L::B_BYTES;
            if (f16) {
#pragma unroll
              for (int j = 0; j < 4; j++) {  // 16 k per instruction
                const uint64_t a = tile_desc_f16(sa, args.a_mn, j);
                const uint64_t b = tile_desc_f16(sb, args.b_mn, j);
                const uint64_t alo = tile_desc_f16(sa + lo, args.a_mn, j);
                const uint64_t blo = tile_desc_f16(sb + lo, args.b_mn, j);
                umma_f16_pair(d_tmem, a, b, idesc, (kb > c0 || j > 0) ? 1u : 0u);
                umma_f16_pair(d_tmem, a, blo, idesc, 1u);
                umma_f16_pair(d_tmem, alo, b, idesc, 1u);
              }
            } else {
#pragma unroll
              for (int j = 0; j < BK / 8; j++) {  // 8 k per instruction
                const uint64_t a = tile_desc<BK>(sa, args.a_mn, j);
                const uint64_t b = tile_desc<BK>(sb, args.b_mn, j);
                const uint64_t alo = tile_desc<BK>(sa + lo, args.a_mn, j);
                const uint64_t blo = tile_desc<BK>(sb + lo, args.b_mn, j);
                umma_tf32_pair(d_tmem, a, b, idesc, (kb > c0 || j > 0) ? 1u : 0u);
                umma_tf32_pair(d_tmem, a, blo, idesc, 1u);
                umma_tf32_pair(d_tmem, alo, b, idesc, 1u);
              }
            }
            umma_commit_pair(empty0 + 8 * stage);
            umma_commit_pair(map_to_rank(empty0 + 8 * stage, peer));
            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          umma_commit_pair(tfull0 + 8 * acc);
          umma_commit_pair(map_to_rank(tfull0 + 8 * acc, peer));
          if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
      }
      failed = !ok;
    }
  } else {
    // ---------------- epilogue: warps 2..9 own TMEM lanes 32*(warp%4).. of this CTA
    // and columns [col_begin, col_begin + BN / 2) of the tile
    const int lane_base = 32 * (warp & 3);
    const int col_begin = ((warp - 2) >> 2) * (BN / 2);
    const uint32_t tempty_leader = map_to_rank(tempty0, 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    // split-f16: accumulator scale 2^-(e_A + e_B); operand-pair output scale
    const float unscale =
        f16 ? exp2_int(-((args.exp_a ? *args.exp_a : 0) + (args.exp_b ? *args.exp_b : 0))) : 1.0f;
    const bool out16 = VAR == kVarRuntime ? args.out_sc.f16 != 0 : (VAR & 2) != 0;
    const bool slope_c = VAR == kVarRuntime ? args.gelu_slope_c != 0 : (VAR & 1) != 0;
    const float out_s = out16 ? exp2_int(*args.out_sc.exp) : 1.0f;
    // ATTN_DO with o as a binary16 pair: its scale 2^-e
    const float o_inv =
        (K_DO && args.dprep.o_exp != nullptr) ? exp2_int(-*args.dprep.o_exp) : 1.0f;
    float amax = 0.0f;  // max |x| of the operand-pair output this warp wrote
    // attention operands as binary16 pairs: the scales of Q, K, V (QKV) or dO
    // (ATTN_DO), and max |x| of each operand this lane wrote
    const float s16_q = (K_QKV && args.qkv.q16h != nullptr) ? exp2_int(args.qkv.exps[0]) : 1.0f;
    const float s16_k = (K_QKV && args.qkv.q16h != nullptr) ? exp2_int(args.qkv.exps[1]) : 1.0f;
    const float s16_v = (K_QKV && args.qkv.q16h != nullptr) ? exp2_int(args.qkv.exps[2]) : 1.0f;
    const float s16_g = (K_DO && args.dprep.g16h != nullptr) ? exp2_int(*args.dprep.g_exp) : 1.0f;
    float am_q = 0.0f, am_k = 0.0f, am_v = 0.0f, am_g = 0.0f;
    for (int unit = cluster; unit < units; unit += nclusters) {
      const int tile = unit % tiles, split = unit / tiles;
      int ok = 1;
      {
        // K chunks (the plain / residual instance; the host gives the fused
        // modes, whose K is d_model, one chunk): every chunk but the last is
        // added into the f32 running sum in chunk order and its buffer handed
        // back to the MMA warp; the last chunk's buffer receives the total,
        // which the epilogue below then reads as a single accumulator.
        const int kb_begin = split * args.kb_per_split;
        const int nchunks =
            EPI != GEMM_EPI_PLAIN ? 1
            : (min(nkb, kb_begin + args.kb_per_split) - kb_begin + args.chunk_kb - 1) /
                  args.chunk_kb;
        if (nchunks > 1) {
          ok = sum_k_chunks<BN>(tmem_base + ((uint32_t)lane_base << 16) + (uint32_t)col_begin,
                                nchunks, tfull0, tempty_leader, acc, acc_phase, args.error,
                                args.chunk_ws + ((int64_t)blockIdx.x * 8 + (warp - 2)) *
                                                    (32 * (BN / 2)));
          if (!ok) { failed = true; break; }
        }
        if (nchunks <= 1) {
          if (lane == 0) ok = mbar_wait(tfull0 + 8 * acc, acc_phase, args.error) ? 1 : 0;
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) { failed = true; break; }
        }
      }
      __syncwarp();
      tc_fence_after();
      int tm, tn;
      raster(tile, args.tiles_m, args.tiles_n, tm, tn);
      const int m = tm * 2 * TC_BM + (int)rank * TC_BM + lane_base + lane;
      const int n_tile = tn * BN;
      const bool part = args.splits > 1;
      float* cbase = part ? args.partial + (int64_t)split * args.M * args.N : args.C;
      const int64_t ldc = part ? (int64_t)args.N : args.ldc;
      const float* bias = part ? nullptr : args.bias;
      const int accumulate = part ? 0 : args.accumulate;
      int epi = part ? 0 : args.epilogue;
      if (epi != GEMM_EPI_PLAIN && epi != GEMM_EPI_RESIDUAL && epi != EPI) epi = GEMM_EPI_PLAIN;
      const int64_t roff = (int64_t)m * ldc;
      const bool vec = ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(cbase) & 15) == 0);
      // the warp's column-partial row of the GELU_BWD mode
      float* colpart = args.colpart + ((int64_t)(tm * 2 + (int)rank) * 4 + (warp & 3)) * args.N;
      if (args.staged) {
        // Each 32-column chunk of the warp's 32 rows goes through shared memory:
        // lane l writes row l, then lane l handles 4 consecutive columns
        // (4 (l & 7)) of rows 4 i + (l >> 3), so every global load and store of
        // the warp covers four whole 128-byte row segments.
        const uint32_t stage = smem_u32(smem + L::RING_BYTES + 256) + (uint32_t)(warp - 2) * 4096u;
        const int sub = lane >> 3, q = lane & 7;
        const int row0 = m - lane;
        // attention-operand modes: sequence and token of row0 + sub
        int seq0 = 0, tok0 = 0, seqT = 1;
        if (ATTN && (epi == GEMM_EPI_QKV || epi == GEMM_EPI_ATTN_DO)) {
          seqT = epi == GEMM_EPI_QKV ? args.qkv.T : args.dprep.T;
          seq0 = (row0 + sub) / seqT;
          tok0 = row0 + sub - seq0 * seqT;
        }
        const bool has_aux = epi == GEMM_EPI_RESIDUAL || (K_GB && epi == GEMM_EPI_GELU_BWD);
        // ATTN_DO: per row of the warp, the running dO . O sum of the current head
        float dacc[8];
#pragma unroll
        for (int it = 0; it < 8; it++) dacc[it] = 0.0f;
#pragma unroll 1
        for (int c = col_begin; c < col_begin + BN / 2; c += 32) {
          const int n = n_tile + c + 4 * q;
          const bool col_ok = n < args.N;  // N % 4 == 0: the 4 columns are all in or all out
          // attention-operand modes: the lane's section / head / column
          int a_sec = 0, a_h = 0, a_j = 0;
          if (K_QKV && epi == GEMM_EPI_QKV && col_ok) qkv_column(args.qkv, n, a_sec, a_h, a_j);
          if (K_DO && epi == GEMM_EPI_ATTN_DO) {
            a_h = n / args.dprep.Dh;
            a_j = n - a_h * args.dprep.Dh;
          }
          // the auxiliary rows of the chunk, loaded before the accumulator wait
          float4 pre[8];
          // ATTN_DO with o as a binary16 pair: every row's pair is requested
          // before any is converted (one memory round trip per chunk)
          uint4 raw[8];
          if (K_DO && epi == GEMM_EPI_ATTN_DO && args.dprep.o_exp != nullptr) {
#pragma unroll
            for (int it = 0; it < 8; it++) {
              const int row = row0 + 4 * it + sub;
              raw[it] = make_uint4(0u, 0u, 0u, 0u);
              if (row < args.M && col_ok) {
                const int64_t oo = (int64_t)row * (args.dprep.H * args.dprep.Dh) + n;
                const uint2 h = __ldg(reinterpret_cast<const uint2*>(
                    reinterpret_cast<const uint16_t*>(args.dprep.o) + oo));
                const uint2 l = __ldg(reinterpret_cast<const uint2*>(
                    reinterpret_cast<const uint16_t*>(args.dprep.o_lo) + oo));
                raw[it] = make_uint4(h.x, h.y, l.x, l.y);
              }
            }
          }
#pragma unroll
          for (int it = 0; it < 8; it++) {
            const int row = row0 + 4 * it + sub;
            pre[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (has_aux && row < args.M && col_ok)
              pre[it] = __ldg(reinterpret_cast<const float4*>(args.aux + (int64_t)row * ldc + n));
            if (K_DO && epi == GEMM_EPI_ATTN_DO && row < args.M && col_ok) {
              // the forward output o = hi + lo (exact), same layout as dO
              const int64_t oo = (int64_t)row * (args.dprep.H * args.dprep.Dh) + n;
              if (args.dprep.o_exp != nullptr) {  // binary16 pair of o 2^e
                const uint4 r = raw[it];
                pre[it] = make_float4((half_lo(r.x) + half_lo(r.z)) * o_inv,
                                      (half_hi(r.x) + half_hi(r.z)) * o_inv,
                                      (half_lo(r.y) + half_lo(r.w)) * o_inv,
                                      (half_hi(r.y) + half_hi(r.w)) * o_inv);
              } else {
                const float4 oh = __ldg(reinterpret_cast<const float4*>(args.dprep.o + oo));
                float4 ol = make_float4(0.f, 0.f, 0.f, 0.f);
                if (args.dprep.o_lo != nullptr)
                  ol = __ldg(reinterpret_cast<const float4*>(args.dprep.o_lo + oo));
                pre[it] = make_float4(oh.x + ol.x, oh.y + ol.y, oh.z + ol.z, oh.w + ol.w);
              }
            }

          }
          float v[32];
          tmem_ld32(tmem_base + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN + c), v);
          if (f16) {
#pragma unroll
            for (int u = 0; u < 32; u++) v[u] *= unscale;
          }
#pragma unroll
          for (int u = 0; u < 8; u++)
            sts128(stage + (uint32_t)lane * 128u + (((uint32_t)u ^ (uint32_t)(lane & 7)) << 4),
                   make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]));
          __syncwarp();
          float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
          if (bias != nullptr && col_ok) b4 = *reinterpret_cast<const float4*>(bias + n);
          float4 cs = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int it = 0; it < 8; it++) {
            const int r = 4 * it + sub;
            float4 x = lds128(stage + (uint32_t)r * 128u + (((uint32_t)q ^ (uint32_t)(r & 7)) << 4));
            const int row = row0 + r;
            if (K_DO && epi == GEMM_EPI_ATTN_DO) {
              // C = dO, its head-major hi / lo copies, and the row's dO . O over
              // these 32 columns (summed over the 8 lanes of the row)
              float dot = 0.0f;
              if (row < args.M && col_ok) {
                if (!args.skip_c) *reinterpret_cast<float4*>(cbase + (int64_t)row * ldc + n) = x;
                int tk = tok0 + 4 * it, sq = seq0;
                while (tk >= seqT) { tk -= seqT; ++sq; }
                attn_do_store(args.dprep, a_h, a_j, sq, tk, x, s16_g);
                am_g = abs_max4(am_g, x);
                const float4 o = pre[it];
                dot = fmaf(x.w, o.w, fmaf(x.z, o.z, fmaf(x.y, o.y, x.x * o.x)));
              }
              dot += __shfl_xor_sync(0xffffffffu, dot, 1);
              dot += __shfl_xor_sync(0xffffffffu, dot, 2);
              dot += __shfl_xor_sync(0xffffffffu, dot, 4);
              dacc[it] += dot;
              continue;
            }
            if (row >= args.M || !col_ok) continue;
            const int64_t off = (int64_t)row * ldc + n;
            if (K_GB && epi == GEMM_EPI_GELU_BWD) {
              // d = y GELU'(u), split into hi (C) and lo (out2); column sums
              // (aux holds u, or GELU'(u) itself with gelu_slope_c)
              const float4 u4 = pre[it];
              float4 d;
              if (slope_c) {
                d.x = rn_mul(x.x, u4.x);
                d.y = rn_mul(x.y, u4.y);
                d.z = rn_mul(x.z, u4.z);
                d.w = rn_mul(x.w, u4.w);
              } else {
                d.x = rn_mul(x.x, gelu_slope(u4.x));
                d.y = rn_mul(x.y, gelu_slope(u4.y));
                d.z = rn_mul(x.z, gelu_slope(u4.z));
                d.w = rn_mul(x.w, gelu_slope(u4.w));
              }
              cs.x += d.x; cs.y += d.y; cs.z += d.z; cs.w += d.w;
              amax = abs_max4(amax, d);
              if (out16) {
                f16_store4(reinterpret_cast<uint16_t*>(cbase), reinterpret_cast<uint16_t*>(args.out2),
                           off, d, out_s);
                continue;
              }
              if (args.out2 != nullptr) {
                float4 lo;
                tf32_split(d.x, d.x, lo.x);
                tf32_split(d.y, d.y, lo.y);
                tf32_split(d.z, d.z, lo.z);
                tf32_split(d.w, d.w, lo.w);
                *reinterpret_cast<float4*>(args.out2 + off) = lo;
              }
              *reinterpret_cast<float4*>(cbase + off) = d;
              continue;
            }
            if (bias != nullptr) {
              x.x += b4.x; x.y += b4.y; x.z += b4.z; x.w += b4.w;
            }
            float4* dst = reinterpret_cast<float4*>(cbase + off);
            if (epi == GEMM_EPI_RESIDUAL) {
              const float4 o = pre[it];
              x.x = rn_add(x.x, o.x); x.y = rn_add(x.y, o.y);
              x.z = rn_add(x.z, o.z); x.w = rn_add(x.w, o.w);
            } else if (accumulate) {
              const float4 o = *dst;
              x.x += o.x; x.y += o.y; x.z += o.z; x.w += o.w;
            }
            if (K_GF && epi == GEMM_EPI_GELU_FWD && slope_c) {
              // C = GELU'(u) for the backward (one erf shared with GELU(u))
              float4 g, sl;
              gelu_both(x.x, g.x, sl.x);
              gelu_both(x.y, g.y, sl.y);
              gelu_both(x.z, g.z, sl.z);
              gelu_both(x.w, g.w, sl.w);
              *dst = sl;
              amax = abs_max4(amax, g);
              if (out16) {
                f16_store4(reinterpret_cast<uint16_t*>(args.out2),
                           reinterpret_cast<uint16_t*>(args.out3), off, g, out_s);
              } else {
                float4 lo = make_float4(0.f, 0.f, 0.f, 0.f);
                if (args.out3 != nullptr) {
                  tf32_split(g.x, g.x, lo.x);
                  tf32_split(g.y, g.y, lo.y);
                  tf32_split(g.z, g.z, lo.z);
                  tf32_split(g.w, g.w, lo.w);
                  *reinterpret_cast<float4*>(args.out3 + off) = lo;
                }
                *reinterpret_cast<float4*>(args.out2 + off) = g;
              }
              continue;
            }
            if (!(ATTN && args.skip_c)) *dst = x;
            if (K_GF && epi == GEMM_EPI_GELU_FWD) {
              float4 g = make_float4(gelu_value(x.x), gelu_value(x.y), gelu_value(x.z),
                                     gelu_value(x.w));
              amax = abs_max4(amax, g);
              if (out16) {
                f16_store4(reinterpret_cast<uint16_t*>(args.out2),
                           reinterpret_cast<uint16_t*>(args.out3), off, g, out_s);
                continue;
              }
              if (args.out3 != nullptr) {
                float4 lo;
                tf32_split(g.x, g.x, lo.x);
                tf32_split(g.y, g.y, lo.y);
                tf32_split(g.z, g.z, lo.z);
                tf32_split(g.w, g.w, lo.w);
                *reinterpret_cast<float4*>(args.out3 + off) = lo;
              }
              *reinterpret_cast<float4*>(args.out2 + off) = g;
            } else if (K_QKV && epi == GEMM_EPI_QKV) {
              int tk = tok0 + 4 * it, sq = seq0;
              while (tk >= seqT) { tk -= seqT; ++sq; }
              const float m4 = qkv_prep_store(args.qkv, a_sec, a_h, a_j, sq, tk, x,
                                              a_sec == 0 ? s16_q : (a_sec == 1 ? s16_k : s16_v));
              if (a_sec == 0) am_q = fmaxf(am_q, m4);
              else if (a_sec == 1) am_k = fmaxf(am_k, m4);
              else am_v = fmaxf(am_v, m4);
            }
          }
          if (K_GB && epi == GEMM_EPI_GELU_BWD) {
            // rows sub, sub + 4, ... summed per lane; then over the 4 lanes of a column group
#pragma unroll
            for (int o = 8; o <= 16; o <<= 1) {
              cs.x += __shfl_xor_sync(0xffffffffu, cs.x, o);
              cs.y += __shfl_xor_sync(0xffffffffu, cs.y, o);
              cs.z += __shfl_xor_sync(0xffffffffu, cs.z, o);
              cs.w += __shfl_xor_sync(0xffffffffu, cs.w, o);
            }
            if (sub == 0 && col_ok) *reinterpret_cast<float4*>(colpart + n) = cs;
          }
          if (K_DO && epi == GEMM_EPI_ATTN_DO && (n_tile + c + 32) % args.dprep.Dh == 0) {
            // the chunk completes a head: one lane per row writes its delta and
            // its base-2 log-sum-exp (the attention backward's formula)
            const int h = (n_tile + c) / args.dprep.Dh;
            // the rows' forward statistics first (read-only loads, all eight
            // in flight together), then the stores
            int64_t ri[8];
            float lsum[8], lmax[8];
#pragma unroll
            for (int it = 0; it < 8; it++) {
              const int row = row0 + 4 * it + sub;
              const int b = row / args.dprep.T, t = row - b * args.dprep.T;
              ri[it] = ((int64_t)b * args.dprep.H + h) * args.dprep.T + t;
              const bool mine = q == 0 && row < args.M && n_tile + c < args.N;
              lsum[it] = mine ? __ldg(args.dprep.row_sum + ri[it]) : 0.0f;
              lmax[it] = mine ? __ldg(args.dprep.row_max + ri[it]) : 0.0f;
            }
#pragma unroll
            for (int it = 0; it < 8; it++) {
              const int row = row0 + 4 * it + sub;
              if (q == 0 && row < args.M && n_tile + c < args.N) {
                args.dprep.delta[ri[it]] = dacc[it];
                const float l = lsum[it];
                args.dprep.lse2[ri[it]] =
                    l > 0.0f ? (lmax[it] + logf(l)) * 1.4426950408889634f : INFINITY;
              }
              dacc[it] = 0.0f;
            }
          }
          __syncwarp();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader + 8 * acc);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        continue;
      }
#pragma unroll 1
      for (int c = col_begin; c < col_begin + BN / 2; c += 32) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN + c), v);
        if (f16) {  // (the host routes operand-pair outputs to the staged path)
#pragma unroll
          for (int u = 0; u < 32; u++) v[u] *= unscale;
        }
        const int n0 = n_tile + c;
        const bool row_ok = m < args.M;
        const bool full = vec && n0 + 32 <= args.N;
        if (K_GB && epi == GEMM_EPI_GELU_BWD) {
          // d = y GELU'(u); the columns' partial sums include every row of the warp
          float d[32];
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int n = n0 + i;
            d[i] = (row_ok && n < args.N) ? rn_mul(v[i], gelu_slope(args.aux[roff + n])) : 0.0f;
          }
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
              const int n = n0 + i;
              if (n < args.N) {
                float h = d[i], lo = 0.0f;
                if (args.out2 != nullptr) tf32_split(d[i], h, lo);
                cbase[roff + n] = h;
                if (args.out2 != nullptr) args.out2[roff + n] = lo;
              }
            }
          }
          float cs[32];
#pragma unroll
          for (int i = 0; i < 32; i++) cs[i] = d[i];
          const float colsum = warp_column_sums(cs);
          if (n0 + lane < args.N) colpart[n0 + lane] = colsum;
          continue;
        }
        if (!row_ok) continue;
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 r = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            if (bias) {
              r.x += bias[n0 + i];
              r.y += bias[n0 + i + 1];
              r.z += bias[n0 + i + 2];
              r.w += bias[n0 + i + 3];
            }
            float4* dst = reinterpret_cast<float4*>(cbase + roff + n0 + i);
            if (epi == GEMM_EPI_RESIDUAL) {
              const float4 o = *reinterpret_cast<const float4*>(args.aux + roff + n0 + i);
              r.x = rn_add(r.x, o.x); r.y = rn_add(r.y, o.y);
              r.z = rn_add(r.z, o.z); r.w = rn_add(r.w, o.w);
            } else if (accumulate) {
              const float4 o = *dst;
              r.x += o.x; r.y += o.y; r.z += o.z; r.w += o.w;
            }
            *dst = r;
            if (K_GF && epi == GEMM_EPI_GELU_FWD) {
              float4 g = make_float4(gelu_value(r.x), gelu_value(r.y), gelu_value(r.z),
                                     gelu_value(r.w));
              if (args.out3 != nullptr) {
                float4 lo;
                tf32_split(g.x, g.x, lo.x);
                tf32_split(g.y, g.y, lo.y);
                tf32_split(g.z, g.z, lo.z);
                tf32_split(g.w, g.w, lo.w);
                *reinterpret_cast<float4*>(args.out3 + roff + n0 + i) = lo;
              }
              *reinterpret_cast<float4*>(args.out2 + roff + n0 + i) = g;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int n = n0 + i;
            if (n < args.N) {
              float r = v[i];
              if (bias) r += bias[n];
              if (epi == GEMM_EPI_RESIDUAL) r = rn_add(r, args.aux[roff + n]);
              else if (accumulate) r += cbase[roff + n];
              cbase[roff + n] = r;
              if (K_GF && epi == GEMM_EPI_GELU_FWD) {
                float gv = gelu_value(r), lo = 0.0f;
                if (args.out3 != nullptr) tf32_split(gv, gv, lo);
                args.out2[roff + n] = gv;
                if (args.out3 != nullptr) args.out3[roff + n] = lo;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + 8 * acc);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    if (args.out_sc.amax != nullptr) amax_record_warp(args.out_sc.amax, amax);
    if (K_QKV && args.qkv.amax != nullptr) {
      amax_record_warp(args.qkv.amax, am_q);
      amax_record_warp(args.qkv.amax + 1, am_k);
      amax_record_warp(args.qkv.amax + 2, am_v);
    }
    if (K_DO && args.dprep.g_amax != nullptr) amax_record_warp(args.dprep.g_amax, am_g);
  }
  // After a timeout, give copies still in flight (whose completion this CTA
  // cannot observe when it lands on the peer's barrier) time to land.
  if (__syncthreads_or(failed)) {
    const long long start = clock64();
    while (clock64() - start < (1ll << 22)) {
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA of the pair leaves while the other still uses its memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
}

// ---- host side ---------------------------------------------------------------

// Operand map: K-major [rows, K] with box {BK k, tile rows} and the 16-byte-
// atom swizzle of BK*4-byte rows; MN-major [K, rows] with box {32 mn, BK k}
// (one load per 32-wide chunk) and the 32-byte-atom 128-byte swizzle.
bool operand_map(CUtensorMap* map, const float* p, bool kmajor, int rows, int K, int64_t ld,
                 int tile_rows, int bk) {
  if (kmajor)
    return make_map_box(map, p, (uint64_t)K, (uint64_t)rows, ld, (uint32_t)bk,
                        (uint32_t)tile_rows,
                        bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  return make_map_box(map, p, (uint64_t)rows, (uint64_t)K, ld, 32u, (uint32_t)bk,
                      CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}
// binary16 operand map: 64 k (128 bytes) per row.  K-major [rows, K] with box
// {64 k, tile rows}; MN-major [K, rows] with box {64 mn, 64 k} (one load per
// 64-wide chunk); both with the 128-byte swizzle.
bool operand_map_f16(CUtensorMap* map, const void* p, bool kmajor, int rows, int K, int64_t ld,
                     int tile_rows) {
  if (kmajor)
    return make_map_box(map, p, (uint64_t)K, (uint64_t)rows, ld, 64u, (uint32_t)tile_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B, true);
  return make_map_box(map, p, (uint64_t)rows, (uint64_t)K, ld, 64u, 64u,
                      CU_TENSOR_MAP_SWIZZLE_128B, true);
}

// A split-f16 GEMM the pair kernel cannot take has no other path: report it
// through the device error word (the model's step then fails loudly).
void gemm_f16_refused(const GemmArgs& g, const char* why) {
  fprintf(stderr, "et_b200: split-f16 GEMM %d x %d x %d refused (%s)\n", g.M, g.N, g.K, why);
  static const int one = 1;
  cudaMemcpy(device_error_word(), &one, sizeof(int), cudaMemcpyHostToDevice);
}

// K blocks summed per tensor-pipe accumulator by the pair kernel before the
// chunk is added into its f32 running sum: 1,024 k of binary16 pairs or 512 k
// of TF32 pairs, the same MMA time per chunk (about 24k cycles), long enough
// to hide the epilogue's read-modify-write of the running sum.
constexpr int kChunkKbF16 = 16;
constexpr int kChunkKbTf32 = 16;

// C = (accumulate ? C : 0) + bias + sum over s of partial[s] (s ascending).
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                     float* __restrict__ C, int64_t ldc,
                                     const float* __restrict__ bias, int accumulate) {
  const int64_t total = (int64_t)M * N;
  const int64_t plane = total;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i - (int64_t)m * N);
    float acc = partial[i];
    for (int s = 1; s < splits; s++) acc += partial[(int64_t)s * plane + i];
    float* c = C + (int64_t)m * ldc + n;
    if (bias) acc += bias[n];
    if (accumulate) acc += *c;
    *c = acc;
  }
}

// Splits that best fill whole waves of the GPU for `tiles` output tiles and
// nkb K blocks (each split keeps at least 32 K blocks); 1 when the tiles fill
// the GPU well already.
int choose_splits(int tiles, int nkb, int sms) {
  auto fill = [&](int s) {
    const int u = tiles * s;
    return (double)u / (double)(((u + sms - 1) / sms) * sms);
  };
  int best = 1;
  double best_fill = fill(1);
  if (tiles >= 4 * sms || best_fill >= 0.9) return 1;
  for (int s = 2; s <= 16 && nkb / s >= 32; s++) {
    const double f = fill(s);
    if (f > best_fill + 0.02) { best = s; best_fill = f; }
  }
  return best;
}

template <int BN, int STAGES, bool THREE, int BK>
void launch_tc(const GemmArgs& g, cudaStream_t stream) {
  using L = TcLayout<BN, STAGES, THREE, BK>;
  CUtensorMap ta, tb, ta_lo, tb_lo;
  bool ok = operand_map(&ta, g.A, g.a_kmajor, g.M, g.K, g.lda, TC_BM, BK) &&
            operand_map(&tb, g.B, g.b_kmajor, g.N, g.K, g.ldb, BN, BK);
  if (THREE) {
    ok = ok && operand_map(&ta_lo, g.A_lo, g.a_kmajor, g.M, g.K, g.lda, TC_BM, BK) &&
         operand_map(&tb_lo, g.B_lo, g.b_kmajor, g.N, g.K, g.ldb, BN, BK);
  } else {
    ta_lo = ta;
    tb_lo = tb;
  }
  if (!ok) {
    gemm_simt(g, stream);
    return;
  }
  cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES, THREE, BK>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES);
  TcArgs a{};
  a.M = g.M; a.N = g.N; a.K = g.K;
  a.C = g.C; a.ldc = g.ldc; a.bias = g.bias; a.accumulate = g.accumulate ? 1 : 0;
  a.a_mn = g.a_kmajor ? 0 : 1;
  a.b_mn = g.b_kmajor ? 0 : 1;
  a.tiles_m = (g.M + TC_BM - 1) / TC_BM;
  a.tiles_n = (g.N + BN - 1) / BN;
  a.error = device_error_word();
  const int tiles = a.tiles_m * a.tiles_n;
  const int nkb = (g.K + BK - 1) / BK;
  a.splits = 1;
  a.kb_per_split = nkb;
  a.chunk_kb = nkb;  // (the single-CTA kernel accumulates each split in one buffer)
  a.partial = nullptr;
  const int s = choose_splits(tiles, nkb, sm_count());
  if (s > 1 && g.workspace != nullptr &&
      g.workspace_floats >= (size_t)s * (size_t)g.M * (size_t)g.N) {
    a.kb_per_split = (nkb + s - 1) / s;
    a.splits = (nkb + a.kb_per_split - 1) / a.kb_per_split;
    a.partial = g.workspace;
  }
  const int units = tiles * a.splits;
  const int grid = units < sm_count() ? units : sm_count();
  gemm_tc_kernel<BN, STAGES, THREE, BK><<<grid, TC_THREADS, L::SMEM_BYTES, stream>>>(
      ta, ta_lo, tb, tb_lo, a);
  count_launch();
  if (a.splits > 1) {
    const int64_t total = (int64_t)g.M * g.N;
    const int64_t want = (total + 255) / 256;
    const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(a.partial, a.splits, g.M, g.N, g.C, g.ldc,
                                                      g.bias, g.accumulate ? 1 : 0);
    count_launch();
  }
}

}  // namespace

void gemm_simt(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0) return;
  dim3 grid((g.N + SB_N - 1) / SB_N, (g.M + SB_M - 1) / SB_M);
  gemm_simt_kernel<<<grid, 256, 0, stream>>>(g);
  count_launch();
}

size_t gemm_splitk_floats(int M, int N) { return (size_t)16 * (size_t)M * (size_t)N; }
size_t gemm_chunk_ws_floats() { return (size_t)sm_count() * 8 * 32 * 128; }

size_t gemm_epilogue_ws_floats(int M, int N) {
  const size_t pair_parts = (size_t)((M + 2 * TC_BM - 1) / (2 * TC_BM)) * 8 * (size_t)N;
  return std::max(pair_parts, gelu_colsum_workspace_floats((size_t)M, (size_t)N));
}

bool gemm_tc_supported(const GemmArgs& g) {
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return false;
  if ((g.lda & 3) || (g.ldb & 3)) return false;
  if (!aligned(g.A) || !aligned(g.B)) return false;
  if (g.A_lo && !aligned(g.A_lo)) return false;
  if (g.B_lo && !aligned(g.B_lo)) return false;
  // TMA global extents and strides must fit the descriptor limits
  if (g.lda > ((int64_t)1 << 36) || g.ldb > ((int64_t)1 << 36)) return false;
  return encode_fn() != nullptr;
}

// 3xTF32 on CTA pairs: 256 x BN tiles, 3-stage ring of 64 KB per SM.
template <int BN, int STAGES>
void launch_tc2(const GemmArgs& g, cudaStream_t stream) {
  using L = Tc2Layout<BN, STAGES>;
  CUtensorMap ta, tb, ta_lo, tb_lo;
  bool ok;
  if (g.f16)
    ok = operand_map_f16(&ta, g.A, g.a_kmajor, g.M, g.K, g.lda, TC_BM) &&
         operand_map_f16(&tb, g.B, g.b_kmajor, g.N, g.K, g.ldb, BN / 2) &&
         operand_map_f16(&ta_lo, g.A_lo, g.a_kmajor, g.M, g.K, g.lda, TC_BM) &&
         operand_map_f16(&tb_lo, g.B_lo, g.b_kmajor, g.N, g.K, g.ldb, BN / 2);
  else
    ok = operand_map(&ta, g.A, g.a_kmajor, g.M, g.K, g.lda, TC_BM, L::BK) &&
         operand_map(&tb, g.B, g.b_kmajor, g.N, g.K, g.ldb, BN / 2, L::BK) &&
         operand_map(&ta_lo, g.A_lo, g.a_kmajor, g.M, g.K, g.lda, TC_BM, L::BK) &&
         operand_map(&tb_lo, g.B_lo, g.b_kmajor, g.N, g.K, g.ldb, BN / 2, L::BK);
  if (!ok && g.f16) {
    gemm_f16_refused(g, "tensor map");
    return;
  }
  if (!ok) {
    gemm_simt(g, stream);
    return;
  }

  TcArgs a{};
  a.M = g.M; a.N = g.N; a.K = g.K;
  a.C = g.C; a.ldc = g.ldc; a.bias = g.bias; a.accumulate = g.accumulate ? 1 : 0;
  a.a_mn = g.a_kmajor ? 0 : 1;
  a.b_mn = g.b_kmajor ? 0 : 1;
  a.tiles_m = (g.M + 2 * TC_BM - 1) / (2 * TC_BM);
  a.tiles_n = (g.N + BN - 1) / BN;
  a.error = device_error_word();
  a.epilogue = g.epilogue;
  a.aux = g.aux;
  a.out2 = g.out2;
  a.out3 = g.out3;
  a.colpart = g.epi_ws;
  a.f16 = g.f16 ? 1 : 0;
  a.exp_a = g.exp_a;
  a.exp_b = g.exp_b;
  a.out_sc = g.out_sc;
  a.skip_c = g.skip_c && (g.epilogue == GEMM_EPI_QKV || g.epilogue == GEMM_EPI_ATTN_DO) ? 1 : 0;
  a.gelu_slope_c = g.gelu_slope_c ? 1 : 0;
  if (g.epilogue == GEMM_EPI_QKV) a.qkv = *g.qkv;
  if (g.epilogue == GEMM_EPI_ATTN_DO) a.dprep = *g.dprep;
  {
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    a.staged = (g.ldc % 4 == 0) && (g.N % 4 == 0) && al(g.C) && al(g.aux) && al(g.out2) &&
               al(g.out3) && al(g.bias) && al(g.epi_ws) && al(g.workspace);
    if (g.epilogue == GEMM_EPI_ATTN_DO)
      a.staged = a.staged && al(g.dprep->o) && al(g.dprep->o_lo) && al(g.dprep->doh) &&
                 al(g.dprep->dol) && g.dprep->Dh % 32 == 0 && g.N == g.dprep->H * g.dprep->Dh;
  }
  // split-f16 operand-pair outputs and their max |x| come from the staged epilogue only
  const bool pair_out = g.epilogue == GEMM_EPI_GELU_FWD || g.epilogue == GEMM_EPI_GELU_BWD;
  if (!a.staged && pair_out && (g.out_sc.f16 || g.out_sc.amax != nullptr || g.gelu_slope_c)) {
    gemm_f16_refused(g, "unstaged epilogue");
    return;
  }
  if (!pair_out) a.out_sc = OperandScale{};
  // the attention operands are written by the staged epilogue only
  const bool prep_after =
      (g.epilogue == GEMM_EPI_QKV || g.epilogue == GEMM_EPI_ATTN_DO) && !a.staged;
  if (prep_after && g.epilogue == GEMM_EPI_ATTN_DO && g.dprep->o_exp != nullptr) {
    gemm_f16_refused(g, "binary16 attention output needs the staged epilogue");
    return;
  }
  if (prep_after && ((g.epilogue == GEMM_EPI_QKV && g.qkv->q16h != nullptr) ||
                     (g.epilogue == GEMM_EPI_ATTN_DO && g.dprep->g16h != nullptr))) {
    gemm_f16_refused(g, "binary16 attention operands need the staged epilogue");
    return;
  }
  if (prep_after) {
    a.epilogue = GEMM_EPI_PLAIN;
    a.skip_c = 0;
  }
  const int tiles = a.tiles_m * a.tiles_n;
  const int nkb = (g.K + (g.f16 ? 2 * L::BK : L::BK) - 1) / (g.f16 ? 2 * L::BK : L::BK);
  const int pairs = sm_count() / 2;
  a.splits = 1;
  a.kb_per_split = nkb;
  a.partial = nullptr;
  const int s = g.epilogue == GEMM_EPI_PLAIN ? choose_splits(tiles, nkb, pairs) : 1;
  if (s > 1 && g.workspace != nullptr &&
      g.workspace_floats >= (size_t)s * (size_t)g.M * (size_t)g.N) {
    a.kb_per_split = (nkb + s - 1) / s;
    a.splits = (nkb + a.kb_per_split - 1) / a.kb_per_split;
    a.partial = g.workspace;
  }
  // The tensor pipe's f32 accumulation truncates, so its error grows with
  // the K summed into one accumulator (measured against f64 at K = 65,536:
  // about 5e-4 relative, against 7e-7 for an FFMA GEMM).  The kernel
  // therefore accumulates one chunk of K blocks at a time and adds the chunks
  // in f32 (round to nearest) through the caller's chunk scratch.
  const int units = tiles * a.splits;
  const int grid = 2 * (units < pairs ? units : pairs);
  a.chunk_kb = a.kb_per_split;
  a.chunk_ws = nullptr;
  if ((a.epilogue == GEMM_EPI_PLAIN || a.epilogue == GEMM_EPI_RESIDUAL) && g.chunk_ws != nullptr &&
      g.chunk_ws_floats >= (size_t)grid * 8 * 32 * (BN / 2)) {
    a.chunk_kb = g.f16 ? kChunkKbF16 : kChunkKbTf32;
    a.chunk_ws = g.chunk_ws;
  }
  // GELU options as a compile-time variant: (slope, binary16 out) of the
  // split-f16 models' steps (1, 1) / (1, 0) and of the others (0, 0)
  const int gvar = (a.gelu_slope_c ? 1 : 0) | (a.out_sc.f16 ? 2 : 0);
  auto launch = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES);
    kernel<<<grid, TC2_THREADS, L::SMEM_BYTES, stream>>>(ta, ta_lo, tb, tb_lo, a);
  };
  switch (a.epilogue) {
#define TC2_GELU(mode)                                                                     \
  case mode:                                                                               \
    if (gvar == 3) launch(gemm_tc2_kernel<BN, STAGES, mode, 3>);                           \
    else if (gvar == 1) launch(gemm_tc2_kernel<BN, STAGES, mode, 1>);                      \
    else if (gvar == 0) launch(gemm_tc2_kernel<BN, STAGES, mode, 0>);                      \
    else launch(gemm_tc2_kernel<BN, STAGES, mode, kVarRuntime>);                           \
    break;
    TC2_GELU(GEMM_EPI_GELU_FWD)
    TC2_GELU(GEMM_EPI_GELU_BWD)
#undef TC2_GELU
    case GEMM_EPI_QKV: launch(gemm_tc2_kernel<BN, STAGES, GEMM_EPI_QKV, kVarRuntime>); break;
    case GEMM_EPI_ATTN_DO: launch(gemm_tc2_kernel<BN, STAGES, GEMM_EPI_ATTN_DO, kVarRuntime>); break;
    default:  // plain and residual
      launch(gemm_tc2_kernel<BN, STAGES, GEMM_EPI_PLAIN, kVarRuntime>);
  }
  count_launch();
  if (g.epilogue == GEMM_EPI_GELU_BWD) {
    reduce_partials(g.epi_ws, a.tiles_m * 8, g.N, g.N, g.dsum, nullptr, nullptr, stream);
  }
  if (prep_after && g.epilogue == GEMM_EPI_QKV)
    attention_prepare_from_qkv(g.C, g.ldc, g.M, *g.qkv, stream);
  if (prep_after && g.epilogue == GEMM_EPI_ATTN_DO)
    attention_prepare_grad_from(g.C, g.ldc, g.M, *g.dprep, stream);
  if (a.splits > 1) {
    const int64_t total = (int64_t)g.M * g.N;
    const int64_t want = (total + 255) / 256;
    const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(a.partial, a.splits, g.M, g.N, g.C, g.ldc,
                                                      g.bias, g.accumulate ? 1 : 0);
    count_launch();
  }
}

void gemm_tc(const GemmArgs& g, bool three_pass, cudaStream_t stream) {
  if (three_pass) launch_tc2<256, 3>(g, stream);
  else launch_tc<256, 4, false, 32>(g, stream);
}

// The fused epilogues on paths other than the pair kernel: a plain GEMM into
// C, then the same elementwise operation as a separate pass (C holds an
// [M, N] matrix with ldc == N, as every caller of those modes has).
void epilogue_after(const GemmArgs& g, cudaStream_t stream) {
  const size_t count = (size_t)g.M * (size_t)g.N;
  switch (g.epilogue) {
    case GEMM_EPI_RESIDUAL: add_tensors(g.aux, g.C, g.C, count, stream); break;
    case GEMM_EPI_GELU_FWD: gelu_forward(g.C, g.out2, count, stream, g.out3); break;
    case GEMM_EPI_GELU_BWD:
      gelu_backward_colsum(g.aux, g.C, g.C, g.out2, g.dsum, g.epi_ws, (size_t)g.M, (size_t)g.N,
                           stream);
      break;
    case GEMM_EPI_QKV: attention_prepare_from_qkv(g.C, g.ldc, g.M, *g.qkv, stream); break;
    case GEMM_EPI_ATTN_DO: attention_prepare_grad_from(g.C, g.ldc, g.M, *g.dprep, stream); break;
    default: break;
  }
}

void gemm(const GemmArgs& g, int precision, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0) return;
  if (g.f16) {  // binary16 pairs exist for the pair kernel only
    const bool ok = gemm_tc_supported(g) && g.A_lo != nullptr && g.B_lo != nullptr &&
                    (g.lda % 8) == 0 && (g.ldb % 8) == 0;
    if (ok) launch_tc2<256, 3>(g, stream);
    else gemm_f16_refused(g, "operand layout");
    return;
  }
  const bool three = precision == ET_B200_PRECISION_TF32X3;
  const bool pair = three && gemm_tc_supported(g) && g.A_lo != nullptr && g.B_lo != nullptr;
  if (pair) {
    gemm_tc(g, true, stream);  // the pair kernel applies every epilogue mode itself
    return;
  }
  if (g.gelu_slope_c) {  // GELU'(u) in C exists on the pair kernel only
    gemm_f16_refused(g, "GELU slope output");
    return;
  }
  GemmArgs plain = g;
  plain.epilogue = GEMM_EPI_PLAIN;
  if (g.epilogue != GEMM_EPI_PLAIN) plain.accumulate = false;
  if (precision == ET_B200_PRECISION_F32 || !gemm_tc_supported(g) || three)
    gemm_simt(plain, stream);
  else
    gemm_tc(plain, false, stream);
  epilogue_after(g, stream);
}

}  // namespace etb
