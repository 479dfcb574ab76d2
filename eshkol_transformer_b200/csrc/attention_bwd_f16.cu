// A2 causal attention backward on tcgen05 tensor cores with binary16 operand
// pairs (sm_100a): head_dim 128, head_dim 64 from Tq Tk = 768^2 or on
// request, and the training step's split-f16 steps.
//
// Semantics are those of the SIMT backward in attention.cu
// (native/a2_attention_provider.c:416-666) and of the 3xTF32 kernels in
// attention_bwd_tc.cu, with the same two-kernel split and the same fixed
// summation order (no atomics): P = softmax(S) recomputed from the forward's
// statistics, dV = P^T dO, dP = dO V^T, dS = P (dP - delta), dQ = scale dS K,
// dK = scale dS^T Q, then the RoPE backward rotation of dQ and dK.
//
// Operands.  Every f32 operand x of a contraction is carried as the binary16
// pair hi = f16(x 2^e), lo = f16(x 2^e - hi), and each product is
// hi hi + hi lo + lo hi on kind::f16 with f32 accumulation (the split-f16
// scheme the linear GEMMs use): about 22 significant bits of every element,
// down to an absolute floor near 2^-39 of the tensor's largest magnitude.
// The exponent e is one power of two per tensor: for Q, K, V and dO it puts
// the tensor's max |x| into [2^14, 2^15) (a prepass measures the maxima; in
// the training step the producing GEMM epilogues write the pairs with their
// slot's exponent instead); for
// P (in [0, 1]) it is 14; for dS it comes from the bound
// |dS| <= |dP| + |delta| <= 2 Dh max|dO| max|V| (|dP_qk| = |dO_q . V_k| and
// delta_q = dO_q . O_q with O_q a convex combination of V rows).  Scaling by a
// power of two is exact, and every accumulator is multiplied back by
// 2^-(e_A + e_B) before use.  Binary16 tiles are half the bytes of the TF32
// pairs, so the head_dim-128 tiles fit shared memory and TMEM, one tile in
// shared memory serves as both the K-major and the MN-major operand, and each
// MMA instruction covers 16 of the contraction instead of 8.
//
// A operands read from TMEM hold two binary16 elements per 32-bit column,
// element 2c in the low half of column c.
//
//   dK/dV kernel: one CTA per 128 keys of one (batch, kv head); TMEM lane r is
//     key r.  K hi, V hi in TMEM (head_dim 128) or shared memory (64), K lo,
//     V lo in shared memory.  For each query block (128 queries at head_dim
//     64, 64 at 128) of every query head of the group:
//       S^T  = K Q^T,  dP^T = V dO^T              (B: Q, dO tiles, K-major)
//       P^T pair over S^T, dS^T pair over dP^T    (registers -> TMEM)
//       dV  += P^T dO, dK += dS^T Q               (B: the same tiles, MN-major)
//   dQ kernel: one CTA per 128 queries of one (batch, head), TMEM lane r is
//     query r; Q hi, dO hi in TMEM (head_dim 128) or shared memory (64), Q
//     lo, dO lo in shared memory.  For each key block (128 keys at head_dim
//     64, 64 at 128): S = Q K^T, dP = dO V^T; dS pair over S; dQ += dS K.
//   At head_dim 64 the gradient MMAs take hi times [hi | lo] of their B tiles
//   as one instruction of N = 128 (the lo tile sits one 64-column chunk
//   stride after the hi tile) into accumulators of 128 columns whose halves
//   the epilogue adds.
//
// Warp roles, barriers, the abort protocol and the output epilogue follow
// attention_bwd_tc.cu.  All mbarrier waits are bounded; a timeout raises a
// CTA-wide abort flag, in-flight copies and MMAs are waited for (bounded) and
// TMEM is always released.
#include <cuda_fp16.h>

#include <type_traits>

#include "attention_f16.cuh"

namespace etb {

namespace {

using namespace f16att;

constexpr int kPExp = 14;  // P pairs carry P 2^14

// ---- prepasses ------------------------------------------------------------------

__device__ __forceinline__ float lse2_of(float m, float l) {
  return l > 0.0f ? (m + logf(l)) * kLog2e : INFINITY;
}

// Warps take query rows (b, hq, tq), row = (b*Hq + hq)*Tq + tq, in a
// grid-stride loop; each lane reads VEC consecutive elements per step:
// delta = rowsum(dO (o + o_lo)) (lane partial sums, warp tree), lse2, and
// max |dO| over every row the warp saw into amax[3] (one atomic per warp).
template <int VEC, bool VLOAD>
__global__ void attn16_stats_kernel(AttnParams p, AttnTensor o, const float* __restrict__ o_lo,
                                    AttnTensor dout, const float* __restrict__ row_max,
                                    const float* __restrict__ row_sum, float* __restrict__ delta,
                                    float* __restrict__ lse2, unsigned* amax) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)p.B * p.Hq * p.Tq;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  float m = 0.0f;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int tq = (int)(row % p.Tq);
    const int hq = (int)((row / p.Tq) % p.Hq);
    const int b = (int)(row / ((int64_t)p.Tq * p.Hq));
    const int64_t ooff = b * o.sb + hq * o.sh + (int64_t)tq * o.st;
    const float* orow = o.ptr + ooff;
    const float* lrow = o_lo ? o_lo + ooff : nullptr;
    const float* grow = dout.ptr + b * dout.sb + hq * dout.sh + (int64_t)tq * dout.st;
    float s = 0.0f;
    for (int j = VEC * lane; j < p.Dh; j += 32 * VEC) {
      float g[VEC], x[VEC];
      load_vec<VEC, VLOAD>(grow + j, g);
      load_vec<VEC, VLOAD>(orow + j, x);
      if (lrow) {
        float y[VEC];
        load_vec<VEC, VLOAD>(lrow + j, y);
#pragma unroll
        for (int u = 0; u < VEC; u++) x[u] = x[u] + y[u];
      }
#pragma unroll
      for (int u = 0; u < VEC; u++) {
        s = fmaf(g[u], x[u], s);
        m = fmaxf(m, fabsf(g[u]));
        if (g[u] != g[u]) m = g[u];
      }
    }
    s = warp_sum(s);
    if (lane == 0) {
      delta[row] = s;
      lse2[row] = lse2_of(row_max[row], row_sum[row]);
    }
  }
  amax_record_warp(amax + 3, m);
}

// max |hi + lo| of the workspace's Q, K, V pairs (blockIdx.y = 0, 1, 2) into
// amax[blockIdx.y].
__global__ void attn16_amax_kernel(const float* __restrict__ qh, const float* __restrict__ ql,
                                   int64_t nq4, const float* __restrict__ kh,
                                   const float* __restrict__ kl, const float* __restrict__ vh,
                                   const float* __restrict__ vl, int64_t nk4, unsigned* amax) {
  const int t = blockIdx.y;
  const float4* h = reinterpret_cast<const float4*>(t == 0 ? qh : t == 1 ? kh : vh);
  const float4* l = reinterpret_cast<const float4*>(t == 0 ? ql : t == 1 ? kl : vl);
  const int64_t n4 = t == 0 ? nq4 : nk4;
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(h + i), b = __ldg(l + i);
    m = abs_max4(m, make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w));
  }
  amax_record_warp(amax + t, m);
}

// Binary16 pairs of the workspace's Q, K, V (blockIdx.y = 0, 1, 2): hi + lo of
// the TF32 pair scaled by 2^e.
__global__ void attn16_split_qkv_kernel(const float* __restrict__ qh, const float* __restrict__ ql,
                                        int64_t nq4, const float* __restrict__ kh,
                                        const float* __restrict__ kl, const float* __restrict__ vh,
                                        const float* __restrict__ vl, int64_t nk4,
                                        uint16_t* q16h, uint16_t* q16l, uint16_t* k16h,
                                        uint16_t* k16l, uint16_t* v16h, uint16_t* v16l,
                                        const unsigned* amax) {
  const int t = blockIdx.y;
  const float4* h = reinterpret_cast<const float4*>(t == 0 ? qh : t == 1 ? kh : vh);
  const float4* l = reinterpret_cast<const float4*>(t == 0 ? ql : t == 1 ? kl : vl);
  uint16_t* oh = t == 0 ? q16h : t == 1 ? k16h : v16h;
  uint16_t* ol = t == 0 ? q16l : t == 1 ? k16l : v16l;
  const int64_t n4 = t == 0 ? nq4 : nk4;
  const float s = exp2_int(pair_exponent(__uint_as_float(amax[t])));
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(h + i), b = __ldg(l + i);
    f16_store4(oh, ol, 4 * i, make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w), s);
  }
}

// Binary16 pair of dO, head-major [B, Hq, Tq, Dh], from the strided tensor:
// warps take rows in a grid-stride loop, each lane VEC elements per step.
template <int VEC, bool VLOAD>
__global__ void attn16_split_dout_kernel(AttnParams p, AttnTensor dout, uint16_t* g16h,
                                         uint16_t* g16l, const unsigned* amax) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)p.B * p.Hq * p.Tq;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const float sc = exp2_int(pair_exponent(__uint_as_float(amax[3])));
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int tq = (int)(row % p.Tq);
    const int hq = (int)((row / p.Tq) % p.Hq);
    const int b = (int)(row / ((int64_t)p.Tq * p.Hq));
    const float* grow = dout.ptr + b * dout.sb + hq * dout.sh + (int64_t)tq * dout.st;
    for (int j = VEC * lane; j < p.Dh; j += 32 * VEC) {
      float g[VEC];
      load_vec<VEC, VLOAD>(grow + j, g);
#pragma unroll
      for (int u = 0; u < VEC; u += 2) {
        float hi, lo;
        pair2(g[u] * sc, g[u + 1] * sc, hi, lo);
        *reinterpret_cast<uint32_t*>(g16h + row * p.Dh + j + u) = __float_as_uint(hi);
        *reinterpret_cast<uint32_t*>(g16l + row * p.Dh + j + u) = __float_as_uint(lo);
      }
    }
  }
}

struct Bwd16Args {
  const float *lse2, *delta;
  const unsigned* amax;
  int* error;
  float* chunks;     // dK/dV chunk sums, kBwdChunkFloats per slot
  int* slot_flags;   // 0 free, 1 taken
  int chunk_slots;
  const int* exps;   // non-null: the producers' exponents of Q, K, V, dO
};

// dK and dV accumulate over up to G Tq queries; the tensor pipe's f32
// accumulation truncates, so a CTA whose key tile sees more than
// kChunkQueries queries sums its accumulators in chunks:
// at every chunk boundary the probability warps add the finished chunk into
// the CTA's slot in global memory (f32), and the next chunk restarts the
// TMEM accumulation.  (Measured at T = 16,384: one accumulator per key tile
// left dK / dV 1e-4 from float64, outside the A2 tolerance.)
constexpr int kChunkQueries = 2048;

// A free chunk slot for this CTA (thread 0, after its TMEM allocation):
// bounded scan from a CTA-dependent start; -1 (and the error word) if none
// is free, which cannot happen with one slot-holding CTA per SM.
__device__ __forceinline__ int take_chunk_slot(const Bwd16Args& a) {
  const uint64_t lin = blockIdx.x + (uint64_t)gridDim.x * (blockIdx.y + (uint64_t)gridDim.y * blockIdx.z);
  for (int i = 0; i < 4 * a.chunk_slots; i++) {
    const int s = (int)((lin + (uint64_t)i) % (uint64_t)a.chunk_slots);
    if (atomicCAS(a.slot_flags + s, 0, 1) == 0) return s;
  }
  atomicExch(a.error, 0x6e6d);
  return -1;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}
__device__ __forceinline__ int count_below(const int64_t* a, int n, int64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---- warp roles (as attention_bwd_tc.cu) -----------------------------------------
constexpr int THREADS = 352;
constexpr int SOFT = 256;  // probability threads (warps 0-7)
constexpr int MMA_A = 8, MMA_B = 9, LOADER = 10;

// ---- dK / dV ----------------------------------------------------------------------

constexpr int BK = 128;  // keys per CTA (TMEM lanes)

// v += the 32 columns of this thread's lane at taddr (the second half of a
// concatenated accumulator).
__device__ __forceinline__ void add_acc_half(uint32_t taddr, float (&v)[32]) {
  float w[32];
  tmem_ld32(taddr, w);
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] += w[i];
}

template <int DH>
struct Kv16Layout {
  // queries per block: 128 at head_dim 64 (S^T and dP^T at N = 128, the
  // tensor pipe's full rate; TMEM has the room), 64 at head_dim 128
  static constexpr int BQ = DH == 64 ? 128 : 64;
  static constexpr int QT = BQ * DH * 2;  // [BQ, DH] binary16 tile
  static constexpr int KT = BK * DH * 2;  // [BK, DH] binary16 tile
  // CAT (head_dim 64): dV and dK take P^T / dS^T hi times [dO | Q hi, lo] as
  // one MMA of N = 2 DH (the lo tile sits one 64-column chunk stride after
  // the hi tile), into accumulators of 2 DH columns whose halves the
  // epilogue adds; K hi and V hi then stay in shared memory to leave TMEM
  // the room
  static constexpr bool CAT = DH == 64;
  // K lo, V lo (shared-memory A operands); two stages of the Q pair and of the
  // dO pair (hi, lo), each tile read K-major and MN-major; (CAT) K hi, V hi
  static constexpr int KL = 0, VL = KT, QR = 2 * KT, GR = QR + 4 * QT;
  static constexpr int KHS = GR + 4 * QT, VHS = KHS + KT;
  static constexpr int BARS = CAT ? VHS + KT : GR + 4 * QT;
  static constexpr int SMEM = BARS + 256 + 1024;
  static_assert(QT == (DH / 64) * BQ * 128, "lo tile one chunk stride after the hi tile");
  // otherwise K hi / V hi pass through stage 1 of the Q / dO rings on their
  // way to TMEM
  static_assert(CAT || KT <= 2 * QT, "key tile in one ring stage");
  // the epilogue stages dK, dV rows ([128][DH + 4] f32 each) and two column-sum
  // scratch areas in the freed operand buffers
  static_assert(2 * 128 * (DH + 4) * 4 + 2 * SOFT * 16 <= BARS, "epilogue staging");
  // TMEM: K hi, V hi (two elements per column; not with CAT), dK, dV
  // accumulators (CAT: 2 DH columns each), S^T (then the P^T pair), dP^T
  // (then the dS^T pair)
  static constexpr uint32_t ACC = CAT ? 2 * DH : DH;
  static constexpr uint32_t KH = 0, VH = DH / 2, DK = CAT ? 0 : DH, DV = DK + ACC, ST = DV + ACC;
  static constexpr uint32_t DPT = ST + BQ;
  static constexpr uint32_t COLS = 512;
  static_assert(DPT + BQ <= COLS, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory");
};

template <int DH, bool MASKED, bool THREE>
__global__ void __launch_bounds__(THREADS, 1)
attn_bwd_kv_f16_kernel(const __grid_constant__ CUtensorMap kh_map,
                       const __grid_constant__ CUtensorMap kl_map,
                       const __grid_constant__ CUtensorMap vh_map,
                       const __grid_constant__ CUtensorMap vl_map,
                       const __grid_constant__ CUtensorMap qh_map,
                       const __grid_constant__ CUtensorMap ql_map,
                       const __grid_constant__ CUtensorMap gh_map,
                       const __grid_constant__ CUtensorMap gl_map, AttnParams p, AttnOut dk,
                       AttnOut dv, Bwd16Args a) {
  if constexpr (!MASKED) p.mask = nullptr;
  using L = Kv16Layout<DH>;
  constexpr int BQ = L::BQ;
  constexpr int NQC = BQ / 64;  // 32-query chunks per probability thread
  // a CTA sums dK / dV in f32 chunks of 2,048 queries
  constexpr int kChunkBlocks = kChunkQueries / BQ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(16) float lse_s[2 * BQ], dlt_s[2 * BQ];  // per-block statistics ring
  __shared__ __align__(16) int64_t qp_s[2 * BQ];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  // ring barriers come in pairs (stage 0, stage 1); stage s serves every
  // other block, so block j waits phase (j >> 1) & 1 of stage j & 1.  An
  // EMPTY barrier completes when both chains' MMAs reading the stage are done.
  enum {
    LO_FULL, QF0, QF1, QE0, QE1, GF0, GF1, GE0, GE1, SA_DONE, SB_DONE, P_READY, VA_DONE, KB_DONE,
    D_READY0, D_READY1, ST_FULL0, ST_FULL1, DRAIN_A, DRAIN_B, CHUNK_DONE, NBARS
  };
  const uint32_t bar0 = smem_u32(bars);
  auto B_ = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, khalf = (warp >> 2) & 1;
  const int row = quarter * 32 + lane;
  const int k0 = blockIdx.x * BK, hkv = blockIdx.y, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int tk = k0 + row;
  const bool valid_k = tk < p.Tk;
  const uint32_t base = smem_u32(smem);
  const uint32_t kh_stage = base + (L::CAT ? L::KHS : L::QR + 2 * L::QT);
  const uint32_t vh_stage = base + (L::CAT ? L::VHS : L::GR + 2 * L::QT);
  if (warp == LOADER && lane == 0) {
    // the loader initialises the barriers and issues the key tile at once
    // (its copies overlap the TMEM allocation and the position scan below):
    // K, V lo stay in shared memory; K, V hi pass through stage 1 of the rings
    // on their way to TMEM
    for (int i = 0; i < NBARS; i++) {
      const uint32_t n = (i == P_READY || i == D_READY0 || i == D_READY1 || i == CHUNK_DONE) ? SOFT
                         : (i == ST_FULL0 || i == ST_FULL1)               ? 32
                         : (i >= QE0 && i <= QE1) || (i >= GE0 && i <= GE1) ? 2
                                                                          : 1;
      mbar_init(B_(i), n);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
    mbar_expect_tx(B_(LO_FULL), 4 * L::KT);
    const int r = (int)(((int64_t)b * p.Hkv + hkv) * p.Tk + k0);
#pragma unroll
    for (int c = 0; c < DH / 64; c++) {
      const uint32_t o = (uint32_t)c * BK * 128u;
      tma_load_2d(base + L::KL + o, &kl_map, B_(LO_FULL), 64 * c, r);
      tma_load_2d(base + L::VL + o, &vl_map, B_(LO_FULL), 64 * c, r);
      tma_load_2d(kh_stage + o, &kh_map, B_(LO_FULL), 64 * c, r);
      tma_load_2d(vh_stage + o, &vh_map, B_(LO_FULL), 64 * c, r);
    }
  }
  if (tid == 0) *abort = 0;
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
  const int64_t* qp = p.qpos + (int64_t)b * p.Tq;
  const int q_begin = warp_count(qp, p.Tq, kp[k0], false);  // first query that can see a key
  const int jb = q_begin / BQ, nqb = (p.Tq + BQ - 1) / BQ;
  const int per_head = q_begin < p.Tq ? nqb - jb : 0;
  const int n_it = G * per_head;
  auto q0_of = [&](int it) { return (jb + it % per_head) * BQ; };
  auto hq_of = [&](int it) { return hkv * G + it / per_head; };
  const bool chunked = n_it > kChunkBlocks;
  volatile int* slot_s = reinterpret_cast<volatile int*>(tslot + 2);
  if (tid == 0) {
    *slot_s = chunked ? take_chunk_slot(a) : -1;
    if (chunked && *slot_s < 0) *abort = 1;
  }
  // the hi, lo tiles of block j's pair into stage j & 1 of a ring
  auto load_pair = [&](int ring, int full, const CUtensorMap* hm, const CUtensorMap* lm, int j) {
    const int s = j & 1;
    const uint32_t dst = base + ring + (uint32_t)s * 2u * L::QT;
    const int r = (int)(((int64_t)b * p.Hq + hq_of(j)) * p.Tq + q0_of(j));
    mbar_expect_tx(B_(full + s), 2 * L::QT);
#pragma unroll
    for (int c = 0; c < DH / 64; c++) {
      const uint32_t o = (uint32_t)c * BQ * 128u;
      tma_load_2d(dst + o, hm, B_(full + s), 64 * c, r);
      tma_load_2d(dst + L::QT + o, lm, B_(full + s), 64 * c, r);
    }
  };
  int nq = 0, ng = 0;  // blocks issued per ring (loader lane 0)
  if (warp == LOADER && lane == 0 && n_it > 0) {  // block 0's pairs into stage 0
    load_pair(L::QR, QF0, &qh_map, &ql_map, 0);
    load_pair(L::GR, GF0, &gh_map, &gl_map, 0);
    nq = ng = 1;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // K hi (warps 0-3) and V hi (warps 4-7) rows -> TMEM (CAT: they stay in
  // shared memory)
  if (!L::CAT && warp < 8 && n_it > 0) {
    const bool ok = mbar_wait(B_(LO_FULL), 0u, a.error);
    if (!ok) *abort = 1;
    if (__all_sync(0xffffffffu, ok)) {
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
      tile_row16_to_tmem<DH>(khalf == 0 ? kh_stage : vh_stage, row, trow,
                             khalf == 0 ? L::KH : L::VH);
      tmem_wait_st();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == LOADER) {
    // ---- producer: operand pairs by TMA, per-block statistics by the lanes
    bool ok = true;
    for (int j = 0; ok && j < n_it; j++) {
      const int q0 = q0_of(j), hq = hq_of(j);
      if (lane == 0 && j > 0) {  // block 0's pairs went out before the loop
        const int s = j & 1;
        if (j >= 2) ok = role_wait(B_(QE0 + s), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
        if (ok) { load_pair(L::QR, QF0, &qh_map, &ql_map, j); nq++; }
        if (ok && j >= 2) ok = role_wait(B_(GE0 + s), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
        if (ok) { load_pair(L::GR, GF0, &gh_map, &gl_map, j); ng++; }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // statistics of block j into ring slot j&1, free once block j-2's
      // gradients are done
      if (ok && j >= 2) ok = role_wait(B_(D_READY0 + (j & 1)), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
#pragma unroll
        for (int h = 0; h < BQ / 32; h++) {
          const int q = q0 + 32 * h + lane, si = (j & 1) * BQ + 32 * h + lane;
          const int64_t rr = ((int64_t)b * p.Hq + hq) * p.Tq + q;
          lse_s[si] = q < p.Tq ? a.lse2[rr] : INFINITY;
          dlt_s[si] = q < p.Tq ? a.delta[rr] : 0.0f;
          qp_s[si] = q < p.Tq ? qp[q] : INT64_MAX;  // keeps the block's positions ascending
        }
        mbar_arrive(B_(ST_FULL0 + (j & 1)));
      }
    }
    if (lane == 0) {
      // every copy (the key tile's too) has landed before the CTA releases
      // its memory
      mbar_wait(B_(LO_FULL), 0u, a.error);
      for (int j = nq - 2 < 0 ? 0 : nq - 2; j < nq; j++)
        mbar_wait(B_(QF0 + (j & 1)), (uint32_t)((j >> 1) & 1), a.error);
      for (int j = ng - 2 < 0 ? 0 : ng - 2; j < ng; j++)
        mbar_wait(B_(GF0 + (j & 1)), (uint32_t)((j >> 1) & 1), a.error);
    }
  } else if (warp == MMA_A || warp == MMA_B) {
    // ---- MMA chains.  A: S^T = K Q^T, dV += P^T dO.  B: dP^T = V dO^T, dK += dS^T Q.
    const bool is_a = warp == MMA_A;
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t idesc_s = idesc_f16_m128(BQ, 0);
      constexpr uint32_t idesc_o = idesc_f16_m128(DH, 1);
      constexpr uint32_t idesc_o2 = idesc_f16_m128(2 * DH, 1);   // (CAT) [hi | lo]
      const uint32_t xh = tmem + (is_a ? L::KH : L::VH);          // TMEM A operand (hi)
      const uint32_t xhs = is_a ? kh_stage : vh_stage;            // (CAT) shared-memory hi
      const uint32_t xlo = base + (is_a ? L::KL : L::VL);         // shared-memory A (lo)
      const int kring = is_a ? L::QR : L::GR, mring = is_a ? L::GR : L::QR;
      const uint32_t sd = tmem + (is_a ? L::ST : L::DPT);         // scores, then the pair
      const uint32_t acc_d = tmem + (is_a ? L::DV : L::DK);
      const int kfull = is_a ? QF0 : GF0, kempty = is_a ? QE0 : GE0;
      const int mfull = is_a ? GF0 : QF0, mempty = is_a ? GE0 : QE0;
      const int sdone = is_a ? SA_DONE : SB_DONE, gdone = is_a ? VA_DONE : KB_DONE;
      int s_issued = 0, g_issued = 0;
      bool ok = role_wait(B_(LO_FULL), 0u, a.error, abort);
      for (int j = 0; ok && j < n_it; j++) {
        const int s = j & 1;
        const uint32_t par = (uint32_t)(j & 1), spar = (uint32_t)((j >> 1) & 1);
        ok = role_wait(B_(kfull + s), spar, a.error, abort);
        // the score columns are free once the previous block's gradient MMAs read them
        if (ok && j > 0) ok = role_wait(B_(gdone), (uint32_t)((j - 1) & 1), a.error, abort);
        // dP^T waits for S^T, and S^T of the next block for dP^T of this one
        if (ok && !is_a) ok = role_wait(B_(SA_DONE), par, a.error, abort);
        if (ok && is_a && j > 0) ok = role_wait(B_(SB_DONE), (uint32_t)((j - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kt = base + kring + (uint32_t)s * 2u * L::QT;
#pragma unroll
        for (int k = 0; k < DH / 16; k++) {
          const uint64_t bh = kdesc16<BQ>(kt, k), bl = kdesc16<BQ>(kt + L::QT, k);
          if constexpr (L::CAT) {
            umma_f16(sd, kdesc16<BK>(xhs, k), bh, idesc_s, k > 0 ? 1u : 0u);
            if (THREE) {
              umma_f16(sd, kdesc16<BK>(xhs, k), bl, idesc_s, 1u);
              umma_f16(sd, kdesc16<BK>(xlo, k), bh, idesc_s, 1u);
            }
          } else {
            umma_f16_ts(sd, xh + 8 * k, bh, idesc_s, k > 0 ? 1u : 0u);
            if (THREE) {
              umma_f16_ts(sd, xh + 8 * k, bl, idesc_s, 1u);
              umma_f16(sd, kdesc16<BK>(xlo, k), bh, idesc_s, 1u);
            }
          }
        }
        umma_commit(B_(sdone));
        umma_commit(B_(kempty + s));
        s_issued++;
        ok = role_wait(B_(is_a ? P_READY : D_READY0 + s), is_a ? par : spar, a.error, abort);
        if (ok) ok = role_wait(B_(mfull + s), spar, a.error, abort);
        // a new chunk starts once the probability warps have added the last one
        const bool restart = j % kChunkBlocks == 0;
        if (ok && restart && j > 0)
          ok = role_wait(B_(CHUNK_DONE), (uint32_t)((j / kChunkBlocks - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t mt = base + mring + (uint32_t)s * 2u * L::QT;
#pragma unroll
        for (int k = 0; k < BQ / 16; k++) {
          // queries 16k..16k+15: hi / lo columns of the half that wrote them
          const uint32_t ah = sd + 32u * (uint32_t)(k >> 1) + 8u * (uint32_t)(k & 1);
          const uint64_t bh = mdesc16<BQ>(mt, k), bl = mdesc16<BQ>(mt + L::QT, k);
          if (L::CAT && THREE) {  // hi times [hi | lo], then lo times hi
            umma_f16_ts(acc_d, ah, bh, idesc_o2, (!restart || k > 0) ? 1u : 0u);
            umma_f16_ts(acc_d, ah + 16u, bh, idesc_o, 1u);
          } else {
            umma_f16_ts(acc_d, ah, bh, idesc_o, (!restart || k > 0) ? 1u : 0u);
            if (THREE) {
              umma_f16_ts(acc_d, ah, bl, idesc_o, 1u);
              umma_f16_ts(acc_d, ah + 16u, bh, idesc_o, 1u);
            }
          }
        }
        umma_commit(B_(gdone));
        umma_commit(B_(mempty + s));
        g_issued++;
      }
      // every MMA of this chain (and the barrier arrivals committed after
      // them) completes before TMEM and shared memory are released
      (void)s_issued; (void)g_issued;
      umma_commit(B_(is_a ? DRAIN_A : DRAIN_B));
      mbar_wait(B_(is_a ? DRAIN_A : DRAIN_B), 0u, a.error);
    }
  } else {
    // ---- P^T = 2^(S^T scale log2(e) - lse2), then dS^T = P^T (dP^T - delta)
    const Exps ex = exps_of(a.amax, DH, a.exps);
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int64_t kpos_row = valid_k ? kp[tk] : INT64_MAX;
    const bool keys_full = k0 + BK <= p.Tk;
    const int64_t kpos_last = kp[min(k0 + BK, p.Tk) - 1];
    const float c2 = p.scale * kLog2e * exp2_int(-(ex.q + ex.k));
    const float u_dp = exp2_int(-(ex.v + ex.g));
    const float s_p = exp2_int(kPExp), s_ds = exp2_int(ex.ds);
    // this thread's queries of each block: NQC chunks of 32 from cb; chunk c's
    // P and dS pairs go over its own 32 S^T / dP^T columns (hi, then lo)
    const int cb = 32 * NQC * khalf;
    const int slot = *slot_s;
    // this thread's row of the chunk sums: dK (warps 0-3) or dV (warps 4-7)
    float* crow = slot >= 0 ? a.chunks + (size_t)slot * kBwdChunkFloats +
                                  (size_t)(khalf * 128 + row) * DH
                            : nullptr;
    bool ok = true;
    for (int j = 0; ok && j < n_it; j++) {
      const int s = j & 1;
      const uint32_t par = (uint32_t)(j & 1), spar = (uint32_t)((j >> 1) & 1);
      const int q0 = q0_of(j);
      // mask bytes of this thread's first 32 queries, issued ahead of the
      // waits (later chunks load theirs in the chunk loop); clamped indices
      // stay in bounds
      const int tkc = min(tk, p.Tk - 1);
      auto mask_chunk = [&](int c, uint8_t (&keep)[32]) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int q = min(q0 + cb + 32 * c + i, p.Tq - 1);
          keep[i] = p.mask[((int64_t)b * p.Tq + q) * p.Tk + tkc];
        }
      };
      uint8_t keep[32];
      if (p.mask != nullptr) mask_chunk(0, keep);
      ok = role_wait(B_(ST_FULL0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SA_DONE), par, a.error, abort);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld/st are warp-collective
      if (!ok) break;
      tc_fence_after();
      const bool full_block =
          p.mask == nullptr && keys_full && q0 + BQ <= p.Tq && qp_s[s * BQ] >= kpos_last;
      // queries of the block see this key from the first whose position
      // reaches it, up to the last query of the sequence
      const int first = full_block ? 0 : count_below(qp_s + s * BQ, BQ, kpos_row) - cb;
      const int last = full_block ? 32 * NQC : p.Tq - q0 - cb;
      float pv[32 * NQC];
#pragma unroll
      for (int c = 0; c < NQC; c++) {
        float sv[32], ls[32];
        tmem_ld32(trow + L::ST + cb + 32 * c, sv);
        const float4* l4 = reinterpret_cast<const float4*>(lse_s + s * BQ + cb + 32 * c);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 v = l4[i];
          ls[4 * i] = v.x; ls[4 * i + 1] = v.y; ls[4 * i + 2] = v.z; ls[4 * i + 3] = v.w;
        }
        float* pc = pv + 32 * c;
        if (full_block) {
#pragma unroll
          for (int i = 0; i < 32; i++) pc[i] = ex2(fmaf(sv[i], c2, -ls[i]));
        } else {
          if (c > 0 && p.mask != nullptr) mask_chunk(c, keep);
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int qi = 32 * c + i;
            bool adm = qi >= first && qi < last;
            if (p.mask != nullptr) adm = adm && keep[i] != 0;
            pc[i] = adm ? ex2(fmaf(sv[i], c2, -ls[i])) : 0.0f;
          }
        }
        float chunk[32], hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 32; i++) chunk[i] = pc[i];
        pack_pairs(chunk, s_p, hi, lo);
        tmem_st16(trow + L::ST + cb + 32 * c, hi);
        tmem_st16(trow + L::ST + cb + 32 * c + 16, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(B_(P_READY));
      if (j > 0 && j % kChunkBlocks == 0) {
        // the chunk ending with block j - 1: once this thread's accumulator
        // (dK for warps 0-3, dV for 4-7) has its last MMA of that chunk, add
        // it into the slot; the next chunk's first gradient MMAs wait for
        // every thread (block j's probabilities are already out)
        ok = role_wait(B_(khalf == 0 ? KB_DONE : VA_DONE), (uint32_t)((j - 1) & 1), a.error,
                       abort);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const bool first_chunk = j == kChunkBlocks;
#pragma unroll
        for (int c = 0; c < DH / 32; c++) {
          float v[32];
          tmem_ld32(trow + (khalf == 0 ? L::DK : L::DV) + 32 * c, v);
          if (L::CAT && THREE) add_acc_half(trow + (khalf == 0 ? L::DK : L::DV) + DH + 32 * c, v);
          float4* dst = reinterpret_cast<float4*>(crow + 32 * c);
#pragma unroll
          for (int u = 0; u < 8; u++) {
            float4 x = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
            if (!first_chunk) {
              const float4 y = dst[u];
              x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
            }
            dst[u] = x;
          }
        }
        tc_fence_before();
        mbar_arrive(B_(CHUNK_DONE));
      }
      ok = role_wait(B_(SB_DONE), par, a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < NQC; c++) {
        float dp[32], dl[32];
        tmem_ld32(trow + L::DPT + cb + 32 * c, dp);
        const float4* d4 = reinterpret_cast<const float4*>(dlt_s + s * BQ + cb + 32 * c);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 v = d4[i];
          dl[4 * i] = v.x; dl[4 * i + 1] = v.y; dl[4 * i + 2] = v.z; dl[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < 32; i++) dp[i] = pv[32 * c + i] * (dp[i] * u_dp - dl[i]);
        float hi[16], lo[16];
        pack_pairs(dp, s_ds, hi, lo);
        tmem_st16(trow + L::DPT + cb + 32 * c, hi);
        tmem_st16(trow + L::DPT + cb + 32 * c + 16, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(B_(D_READY0 + s));
    }
    if (ok && n_it > 0) {
      const uint32_t last = (uint32_t)((n_it - 1) & 1);
      ok = role_wait(B_(VA_DONE), last, a.error, abort);
      if (ok) ok = role_wait(B_(KB_DONE), last, a.error, abort);
    }
    ok = __all_sync(0xffffffffu, ok);
    // warps 0-3 stage the dK rows, warps 4-7 the dV rows (accumulators
    // multiplied back to f32 scale), in the freed operand buffers; the
    // gradient scale, the RoPE backward rotation (dK) and the output split are
    // applied while the rows are written out (coalesced)
    const uint32_t stage = base + (uint32_t)(khalf * 128 * (DH + 4) * 4);
    // a tile no query sees stages its zero rows over the key tile's buffers:
    // its copies land first
    if (n_it == 0 && !mbar_wait(B_(LO_FULL), 0u, a.error)) ok = false;
    // head_dim 64: the tile's RoPE table rows into the freed ring (past the
    // staging and column-sum areas), so the dK rotation below reads shared
    // memory
    const uint32_t tab = base + (uint32_t)(2 * 128 * (DH + 4) * 4 + 2 * SOFT * 16);
    static_assert(DH != 64 || 2 * 128 * (DH + 4) * 4 + 2 * SOFT * 16 + 2 * 128 * (DH / 2) * 4 <=
                                  L::BARS, "table copy");
    bool tab_s = false;
    if (DH == 64 && ok)
      tab_s = rope_rows_to_smem(tab, p.k_cos, p.k_sin,
                                (int64_t)(p.k_rope_batched ? b * p.Tk + k0 : k0),
                                min(BK, p.Tk - k0), DH, tid, SOFT);
    if (ok) {
      tc_fence_after();
      const float un = khalf == 0 ? exp2_int(-(ex.ds + ex.q)) : exp2_int(-(kPExp + ex.g));
#pragma unroll
      for (int c = 0; c < DH / 32; c++) {
        float v[32];
        if (n_it > 0) {
          tmem_ld32(trow + (khalf == 0 ? L::DK : L::DV) + 32 * c, v);
          if (L::CAT && THREE) add_acc_half(trow + (khalf == 0 ? L::DK : L::DV) + DH + 32 * c, v);
          if (crow != nullptr) {  // plus the earlier chunks
            const float4* src = reinterpret_cast<const float4*>(crow + 32 * c);
#pragma unroll
            for (int u = 0; u < 8; u++) {
              const float4 y = src[u];
              v[4 * u] += y.x; v[4 * u + 1] += y.y; v[4 * u + 2] += y.z; v[4 * u + 3] += y.w;
            }
          }
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] *= un;
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = 0.0f;
        }
        stage_row32(stage, DH, row, 32 * c, v, 0, 32);
      }
    }
    named_sync(1, SOFT);
    const uint32_t red = base + (uint32_t)(2 * 128 * (DH + 4) * 4);
    float amax_k = 0.0f, amax_v = 0.0f;
    if (ok) {
      const bool split = dk.lo != nullptr && dv.lo != nullptr;
      const int rows = min(BK, p.Tk - k0);
      const int64_t ko = b * dk.sb + hkv * dk.sh + (int64_t)k0 * dk.st;
      const float4 sk = store_rows_split(
          base, DH, rows, dk.ptr, split ? dk.lo : nullptr, ko, dk.st, tid, SOFT,
          [&](int r, int c4, float4& v) {
            if (tab_s) {
              grad_rotate4_smem(v, p.scale, tab, r, c4, DH / 2);
              return;
            }
            const int t = k0 + r;
            const int64_t trw = (int64_t)(p.k_rope_batched ? b * p.Tk + t : t) * (DH / 2);
            grad_rotate4(v, p.scale, p.k_cos, p.k_sin, trw, c4);
          }, dk.sc, amax_k);
      const int64_t vo = b * dv.sb + hkv * dv.sh + (int64_t)k0 * dv.st;
      const float4 sv = store_rows_split(base + (uint32_t)(128 * (DH + 4) * 4), DH, rows,
                                         dv.ptr, split ? dv.lo : nullptr, vo, dv.st, tid,
                                         SOFT, [](int, int, float4&) {}, dv.sc, amax_v);
      colsum_put(red, tid, sk);
      colsum_put(red + SOFT * 16u, tid, sv);
    }
    if (dk.sc.amax != nullptr) amax_record_warp(dk.sc.amax, amax_k);
    if (dv.sc.amax != nullptr) amax_record_warp(dv.sc.amax, amax_v);
    named_sync(1, SOFT);
    if (ok) {
      const int64_t prow = (int64_t)b * ((p.Tk + BK - 1) / BK) + blockIdx.x;
      if (dk.colsum != nullptr)
        colsum_get(red, tid, SOFT, DH, dk.colsum + prow * dk.colsum_ld + hkv * DH);
      if (dv.colsum != nullptr)
        colsum_get(red + SOFT * 16u, tid, SOFT, DH, dv.colsum + prow * dv.colsum_ld + hkv * DH);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::COLS);
  }
  if (tid == 0 && *slot_s >= 0) {  // the slot's sums were read above
    __threadfence();
    atomicExch(a.slot_flags + *slot_s, 0);
  }
}

// ---- dQ ---------------------------------------------------------------------------

constexpr int QM = 128;  // queries per CTA (TMEM lanes)

template <int DH>
struct Q16Layout {
  // keys per block: 128 at head_dim 64 (S and dP at N = 128, the tensor
  // pipe's full rate; TMEM then holds one dP buffer, DP1), 64 at head_dim 128
  static constexpr int KN = DH == 64 ? 128 : 64;
  static constexpr bool DP1 = KN == 128;
  static constexpr int KT = KN * DH * 2;  // [KN, DH] binary16 tile
  static constexpr int RT = QM * DH * 2;  // [QM, DH] binary16 row tile
  // Q lo and dO lo rows (shared-memory A operands); two stages of K hi/lo,
  // V hi/lo (the K tiles read K-major by S and MN-major by dQ)
  static constexpr int QL = 0, GL = RT, STAGE0 = 2 * RT;
  static constexpr int STAGE = 4 * KT;
  static constexpr int KPOS = STAGE0 + 2 * STAGE;  // [2][KN] key positions
  // CATQ (head_dim 64): dQ takes dS hi times [K hi | K lo] as one MMA of
  // N = 2 DH (the lo tile sits one 64-column chunk stride after the hi tile)
  // into an accumulator of 2 DH columns whose halves the epilogue adds; Q hi
  // and dO hi then stay in shared memory to leave TMEM the room
  static constexpr bool CATQ = DH == 64;
  static constexpr int QHS = KPOS + 2 * KN * 8, GHS = QHS + RT;
  static constexpr int BARS = CATQ ? GHS + RT : KPOS + 2 * KN * 8;
  static constexpr int SMEM = BARS + 256 + 1024;
  static_assert(KT == (DH / 64) * KN * 128, "K lo one chunk stride after K hi");
  // otherwise Q hi and dO hi rows pass through stage 1 on their way to TMEM
  static_assert(2 * RT <= STAGE, "row tiles in one stage");
  static_assert(128 * (DH + 4) * 4 + SOFT * 16 <= KPOS, "epilogue staging");
  // TMEM: Q hi, dO hi (two elements per column); two slots of S (the dS pair
  // over S), each with its dP behind it, or (DP1) one dP buffer behind both
  // slots; the dQ accumulator
  static constexpr uint32_t ACC = CATQ ? 2 * DH : DH;  // dQ accumulator columns
  static constexpr uint32_t QH = 0, GH = DH / 2, SL0 = CATQ ? 0 : DH, SLOT = DP1 ? KN : 2 * KN;
  static constexpr uint32_t DPB = SL0 + 2 * SLOT, DQ = DPB + (DP1 ? KN : 0);
  static constexpr uint32_t COLS = 512;
  static_assert(DQ + ACC <= COLS, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory");
};

template <int DH, bool MASKED, bool THREE>
__global__ void __launch_bounds__(THREADS, 1)
attn_bwd_q_f16_kernel(const __grid_constant__ CUtensorMap qh_map,
                      const __grid_constant__ CUtensorMap ql_map,
                      const __grid_constant__ CUtensorMap gh_map,
                      const __grid_constant__ CUtensorMap gl_map,
                      const __grid_constant__ CUtensorMap kh_map,
                      const __grid_constant__ CUtensorMap kl_map,
                      const __grid_constant__ CUtensorMap vh_map,
                      const __grid_constant__ CUtensorMap vl_map, AttnParams p, AttnOut dq,
                      Bwd16Args a) {
  if constexpr (!MASKED) p.mask = nullptr;
  using L = Q16Layout<DH>;
  constexpr int KN = L::KN;
  constexpr int NKC = KN / 64;  // 32-key chunks per probability thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  int64_t* kpos_s = reinterpret_cast<int64_t*>(smem + L::KPOS);  // [2][KN]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  // per-slot barriers come in pairs (slot 0, slot 1); a slot serves every
  // other block, so block j waits phase (j >> 1) & 1 of slot j & 1.  EMPTY
  // completes when dP (chain B) and dQ (chain A) of the stage's block are done.
  // DP_FREE (DP1): the probability threads have block j's dP in registers,
  // so the one dP buffer can take block j + 1's (phase j & 1).
  enum {
    FULL0, FULL1, EMPTY0, EMPTY1, SA0, SA1, SB0, SB1, DS0, DS1, QD0, QD1, KP0, KP1, ROWS_HI,
    ROWS_LO, DRAIN_A, DRAIN_B, DP_FREE, NBARS
  };
  const uint32_t bar0 = smem_u32(bars);
  auto B_ = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, khalf = (warp >> 2) & 1;
  const int row = quarter * 32 + lane;
  const int q0 = blockIdx.x * QM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / (p.Hq / p.Hkv);
  const int tq = q0 + row;
  const bool valid_q = tq < p.Tq;
  const uint32_t base = smem_u32(smem);
  // Q hi, dO hi rows: stage 1 (on their way to TMEM) or (CATQ) their own area
  const uint32_t rows_hi = base + (L::CATQ ? L::QHS : L::STAGE0 + L::STAGE);
  if (tid == 0) {
    for (int i = 0; i < NBARS; i++) {
      const uint32_t n = (i == DS0 || i == DS1 || i == DP_FREE) ? SOFT
                         : (i == KP0 || i == KP1)       ? 32
                         : (i == EMPTY0 || i == EMPTY1) ? 2
                                                        : 1;
      mbar_init(B_(i), n);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
    const int r = (int)(((int64_t)b * p.Hq + hq) * p.Tq + q0);
    mbar_expect_tx(B_(ROWS_LO), 2 * L::RT);
    mbar_expect_tx(B_(ROWS_HI), 2 * L::RT);
#pragma unroll
    for (int c = 0; c < DH / 64; c++) {
      const uint32_t o = (uint32_t)c * QM * 128u;
      tma_load_2d(base + L::QL + o, &ql_map, B_(ROWS_LO), 64 * c, r);
      tma_load_2d(base + L::GL + o, &gl_map, B_(ROWS_LO), 64 * c, r);
      tma_load_2d(rows_hi + o, &qh_map, B_(ROWS_HI), 64 * c, r);
      tma_load_2d(rows_hi + L::RT + o, &gh_map, B_(ROWS_HI), 64 * c, r);
    }
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  int nkb = 0, full_kb = 0;
  {
    const int qlast = min(q0 + QM, p.Tq) - 1;
    const int64_t qmax = p.qpos[(int64_t)b * p.Tq + qlast];
    const int64_t qmin = p.qpos[(int64_t)b * p.Tq + q0];
    const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
    const int seen = warp_count(kp, p.Tk, qmax, true);      // keys some row of the tile sees
    const int seen_all = warp_count(kp, seen, qmin, true);  // keys every row sees
    nkb = (seen + KN - 1) / KN;
    full_kb = (p.mask == nullptr && q0 + QM <= p.Tq) ? seen_all / KN : 0;
  }
  const int64_t kv_row0 = ((int64_t)b * p.Hkv + hkv) * p.Tk;
  auto load_stage = [&](int j) {  // K hi/lo, V hi/lo of block j into stage j & 1
    const uint32_t bar = B_(FULL0 + (j & 1)), dst = base + L::STAGE0 + (j & 1) * L::STAGE;
    const int r = (int)(kv_row0 + (int64_t)j * KN);
    mbar_expect_tx(bar, L::STAGE);
#pragma unroll
    for (int c = 0; c < DH / 64; c++) {
      const uint32_t o = (uint32_t)c * KN * 128u;
      tma_load_2d(dst + o, &kh_map, bar, 64 * c, r);
      tma_load_2d(dst + L::KT + o, &kl_map, bar, 64 * c, r);
      tma_load_2d(dst + 2 * L::KT + o, &vh_map, bar, 64 * c, r);
      tma_load_2d(dst + 3 * L::KT + o, &vl_map, bar, 64 * c, r);
    }
  };
  // block 0 goes out before the set-up barrier (the thread that initialised
  // the barriers issues it)
  if (tid == 0 && nkb > 0) load_stage(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // Q hi and dO hi rows -> TMEM (warps 0-3 Q, 4-7 dO; CATQ: they stay in
  // shared memory)
  if (!L::CATQ && warp < 8) {
    const bool ok = mbar_wait(B_(ROWS_HI), 0u, a.error);
    if (!ok) *abort = 1;
    if (__all_sync(0xffffffffu, ok)) {
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
      tile_row16_to_tmem<DH>(rows_hi + (uint32_t)khalf * L::RT, row, trow,
                             khalf == 0 ? L::QH : L::GH);
      tmem_wait_st();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == LOADER) {
    // ---- producer: stages one block ahead, key positions by the lanes
    int nk = nkb > 0 ? 1 : 0;  // blocks issued (lane 0)
    bool ok = true;
    auto fill_kpos = [&](int j) {
#pragma unroll
      for (int h = 0; h < KN / 32; h++) {
        const int t = j * KN + 32 * h + lane;
        kpos_s[(j & 1) * KN + 32 * h + lane] = t < p.Tk ? p.kpos[(int64_t)b * p.Tk + t] : INT64_MAX;
      }
      mbar_arrive(B_(KP0 + (j & 1)));
    };
    if (nkb > 0) fill_kpos(0);
    for (int j = 0; ok && j + 1 < nkb; j++) {
      const int jn = j + 1;
      // stage jn & 1 is free once dP and dQ of block jn - 2 completed
      if (lane == 0) {
        if (jn >= 2) ok = role_wait(B_(EMPTY0 + (jn & 1)), (uint32_t)(((jn >> 1) - 1) & 1), a.error, abort);
        if (ok) { load_stage(jn); nk++; }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // position slot jn & 1 is free once block jn - 2's dS is written
      if (ok && jn >= 2) ok = role_wait(B_(DS0 + (jn & 1)), (uint32_t)(((jn >> 1) - 1) & 1), a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) fill_kpos(jn);
    }
    if (lane == 0) {  // every copy has landed before the CTA releases its memory
      mbar_wait(B_(ROWS_LO), 0u, a.error);
      if (L::CATQ) mbar_wait(B_(ROWS_HI), 0u, a.error);
      for (int j = nk - 2 < 0 ? 0 : nk - 2; j < nk; j++)
        mbar_wait(B_(FULL0 + (j & 1)), (uint32_t)((j >> 1) & 1), a.error);
    }
  } else if (warp == MMA_A || warp == MMA_B) {
    // ---- MMA chains.  A: S = Q K^T, then dQ += dS K of the previous block.
    // B: dP = dO V^T.
    const bool is_a = warp == MMA_A;
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc_s = idesc_f16_m128(KN, 0);
      constexpr uint32_t idesc_q = idesc_f16_m128(DH, 1);
      constexpr uint32_t idesc_q2 = idesc_f16_m128(2 * DH, 1);  // (CATQ) [K hi | K lo]
      const uint32_t xh = tmem + (is_a ? L::QH : L::GH);
      const uint32_t xhs = rows_hi + (is_a ? 0u : (uint32_t)L::RT);  // (CATQ) shared-memory hi
      const uint32_t xlo = base + (is_a ? L::QL : L::GL);
      const int sdone = is_a ? SA0 : SB0;
      int s_issued = 0, q_issued = 0;
      bool ok = role_wait(B_(ROWS_LO), 0u, a.error, abort);
      if (ok && L::CATQ) ok = role_wait(B_(ROWS_HI), 0u, a.error, abort);
      auto issue_dq = [&](int i) {
        const int s = i & 1;
        ok = role_wait(B_(DS0 + s), (uint32_t)((i >> 1) & 1), a.error, abort);
        if (!ok) return;
        tc_fence_after();
        const uint32_t sd = tmem + L::SL0 + (uint32_t)s * L::SLOT;  // the dS pair
        const uint32_t kt = base + L::STAGE0 + (uint32_t)s * L::STAGE;
#pragma unroll
        for (int k = 0; k < KN / 16; k++) {
          const uint32_t ah = sd + 32u * (uint32_t)(k >> 1) + 8u * (uint32_t)(k & 1);
          const uint64_t bh = mdesc16<KN>(kt, k), bl = mdesc16<KN>(kt + L::KT, k);
          if (L::CATQ && THREE) {  // hi times [hi | lo], then lo times hi
            umma_f16_ts(tmem + L::DQ, ah, bh, idesc_q2, (i > 0 || k > 0) ? 1u : 0u);
            umma_f16_ts(tmem + L::DQ, ah + 16u, bh, idesc_q, 1u);
          } else {
            umma_f16_ts(tmem + L::DQ, ah, bh, idesc_q, (i > 0 || k > 0) ? 1u : 0u);
            if (THREE) {
              umma_f16_ts(tmem + L::DQ, ah, bl, idesc_q, 1u);
              umma_f16_ts(tmem + L::DQ, ah + 16u, bh, idesc_q, 1u);
            }
          }
        }
        umma_commit(B_(QD0 + s));
        umma_commit(B_(EMPTY0 + s));
        q_issued++;
      };
      for (int j = 0; ok && j < nkb; j++) {
        const int s = j & 1;
        ok = role_wait(B_(FULL0 + s), (uint32_t)((j >> 1) & 1), a.error, abort);
        // the slot's columns are free once block j - 2's dS was read (dQ, A)
        // or written (dP columns, B); the one dP buffer (DP1) once block j -
        // 1's dP is in the probability threads' registers
        if (ok && is_a && j >= 2)
          ok = role_wait(B_(QD0 + s), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
        if (ok && !is_a && L::DP1 && j >= 1)
          ok = role_wait(B_(DP_FREE), (uint32_t)((j - 1) & 1), a.error, abort);
        if (ok && !is_a && !L::DP1 && j >= 2)
          ok = role_wait(B_(DS0 + s), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t stg = base + L::STAGE0 + (uint32_t)s * L::STAGE + (is_a ? 0u : 2u * L::KT);
        const uint32_t sd = is_a ? tmem + L::SL0 + (uint32_t)s * L::SLOT
                            : tmem + (L::DP1 ? L::DPB : L::SL0 + (uint32_t)s * L::SLOT + KN);
#pragma unroll
        for (int k = 0; k < DH / 16; k++) {
          const uint64_t bh = kdesc16<KN>(stg, k), bl = kdesc16<KN>(stg + L::KT, k);
          if constexpr (L::CATQ) {
            umma_f16(sd, kdesc16<QM>(xhs, k), bh, idesc_s, k > 0 ? 1u : 0u);
            if (THREE) {
              umma_f16(sd, kdesc16<QM>(xhs, k), bl, idesc_s, 1u);
              umma_f16(sd, kdesc16<QM>(xlo, k), bh, idesc_s, 1u);
            }
          } else {
            umma_f16_ts(sd, xh + 8 * k, bh, idesc_s, k > 0 ? 1u : 0u);
            if (THREE) {
              umma_f16_ts(sd, xh + 8 * k, bl, idesc_s, 1u);
              umma_f16(sd, kdesc16<QM>(xlo, k), bh, idesc_s, 1u);
            }
          }
        }
        umma_commit(B_(sdone + s));
        if (!is_a) umma_commit(B_(EMPTY0 + s));
        s_issued++;
        if (is_a && j >= 1) issue_dq(j - 1);
      }
      if (is_a && ok) issue_dq(nkb - 1);
      // every MMA of this chain (and the barrier arrivals committed after
      // them) completes before TMEM and shared memory are released
      (void)s_issued; (void)q_issued;
      umma_commit(B_(is_a ? DRAIN_A : DRAIN_B));
      mbar_wait(B_(is_a ? DRAIN_A : DRAIN_B), 0u, a.error);
    }
  } else {
    // ---- dS = P (dP - delta), P = 2^(S scale log2(e) - lse2)
    const Exps ex = exps_of(a.amax, DH, a.exps);
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
    const float lse_row = valid_q ? a.lse2[ri] : INFINITY;
    const float dlt_row = valid_q ? a.delta[ri] : 0.0f;
    const int64_t qpos_row = valid_q ? p.qpos[(int64_t)b * p.Tq + tq] : INT64_MIN;
    const float c2 = p.scale * kLog2e * exp2_int(-(ex.q + ex.k));
    const float u_dp = exp2_int(-(ex.v + ex.g));
    const float s_ds = exp2_int(ex.ds);
    // this thread's keys of each block: NKC chunks of 32 from cb; chunk c's
    // dS pair goes over its own 32 S columns (hi, then lo)
    const int cb = 32 * NKC * khalf;
    bool ok = true;
    for (int j = 0; ok && j < nkb; j++) {
      const int s = j & 1;
      const uint32_t spar = (uint32_t)((j >> 1) & 1);
      const bool full_block = j < full_kb;
      ok = role_wait(B_(KP0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SA0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SB0 + s), spar, a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // keys of the block this query sees: those whose position does not exceed its own
      const int seen = full_block ? KN : count_below(kpos_s + s * KN, KN, qpos_row + 1) - cb;
      const uint32_t slot = trow + L::SL0 + (uint32_t)s * L::SLOT;
      const uint32_t dpc = L::DP1 ? trow + L::DPB : slot + KN;
#pragma unroll
      for (int c = 0; c < NKC; c++) {
        uint8_t keep[32];
        if (!full_block && p.mask != nullptr) {  // clamped indices stay in bounds
          const int64_t mrow = ((int64_t)b * p.Tq + min(tq, p.Tq - 1)) * p.Tk;
#pragma unroll
          for (int i = 0; i < 32; i++)
            keep[i] = p.mask[mrow + min(j * KN + cb + 32 * c + i, p.Tk - 1)];
        }
        float sv[32], dp[32];
        tmem_ld32(slot + cb + 32 * c, sv);
        tmem_ld32(dpc + cb + 32 * c, dp);
        if (L::DP1 && c == NKC - 1) {  // the dP buffer is free for block j + 1
          tc_fence_before();
          mbar_arrive(B_(DP_FREE));
        }
#pragma unroll
        for (int i = 0; i < 32; i++) {
          bool adm = full_block;
          if (!full_block) {
            adm = 32 * c + i < seen;
            if (p.mask != nullptr) adm = adm && keep[i] != 0;
          }
          const float pv = adm ? ex2(fmaf(sv[i], c2, -lse_row)) : 0.0f;
          sv[i] = pv * (dp[i] * u_dp - dlt_row);
        }
        float hi[16], lo[16];
        pack_pairs(sv, s_ds, hi, lo);
        tmem_st16(slot + cb + 32 * c, hi);
        tmem_st16(slot + cb + 32 * c + 16, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(B_(DS0 + s));
    }
    if (ok && nkb > 0) {
      const int i = nkb - 1;
      ok = role_wait(B_(QD0 + (i & 1)), (uint32_t)((i >> 1) & 1), a.error, abort);
    }
    ok = __all_sync(0xffffffffu, ok);
    // a tile that sees no key stages its zero rows over the Q / dO lo rows:
    // their copies land first
    if (nkb == 0 && !mbar_wait(B_(ROWS_LO), 0u, a.error)) ok = false;
    // head_dim 64: the tile's RoPE table rows into the freed stages (past the
    // staging and column-sum areas), so the dQ rotation below reads shared
    // memory
    const uint32_t tab = base + (uint32_t)(128 * (DH + 4) * 4 + SOFT * 16);
    static_assert(DH != 64 || 128 * (DH + 4) * 4 + SOFT * 16 + 2 * 128 * (DH / 2) * 4 <= L::KPOS,
                  "table copy");
    bool tab_s = false;
    if (DH == 64 && ok)
      tab_s = rope_rows_to_smem(tab, p.q_cos, p.q_sin,
                                (int64_t)(p.q_rope_batched ? b * p.Tq + q0 : q0),
                                min(QM, p.Tq - q0), DH, tid, SOFT);
    // dQ rows (multiplied back to f32 scale) staged in the freed stages; the
    // gradient scale, the RoPE backward rotation and the output split are
    // applied while the rows are written out (coalesced)
    if (ok) {
      tc_fence_after();
      const float un = exp2_int(-(ex.ds + ex.k));
#pragma unroll
      for (int c = 0; c < DH / 64; c++) {
        const int col = khalf * (DH / 2) + 32 * c;
        float v[32];
        if (nkb > 0) {
          tmem_ld32(trow + L::DQ + col, v);
          if (L::CATQ && THREE) add_acc_half(trow + L::DQ + DH + col, v);
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] *= un;
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = 0.0f;
        }
        stage_row32(base, DH, row, col, v, 0, 32);
      }
    }
    named_sync(1, SOFT);
    const uint32_t red = base + (uint32_t)(128 * (DH + 4) * 4);
    float amax = 0.0f;
    if (ok) {
      const int64_t qo = b * dq.sb + hq * dq.sh + (int64_t)q0 * dq.st;
      const float4 sq = store_rows_split(
          base, DH, min(QM, p.Tq - q0), dq.ptr, dq.lo, qo, dq.st, tid, SOFT,
          [&](int r, int c4, float4& v) {
            if (tab_s) {
              grad_rotate4_smem(v, p.scale, tab, r, c4, DH / 2);
              return;
            }
            const int t = q0 + r;
            const int64_t trw = (int64_t)(p.q_rope_batched ? b * p.Tq + t : t) * (DH / 2);
            grad_rotate4(v, p.scale, p.q_cos, p.q_sin, trw, c4);
          }, dq.sc, amax);
      colsum_put(red, tid, sq);
    }
    if (dq.sc.amax != nullptr) amax_record_warp(dq.sc.amax, amax);
    named_sync(1, SOFT);
    if (ok && dq.colsum != nullptr) {
      const int64_t prow = (int64_t)b * ((p.Tq + QM - 1) / QM) + blockIdx.x;
      colsum_get(red, tid, SOFT, DH, dq.colsum + prow * dq.colsum_ld + hq * DH);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::COLS);
  }
}

template <int DH>
bool launch_bwd_f16(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                    const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                    AttnOut dk, AttnOut dv, cudaStream_t stream) {
  const AttnWs w = attn_ws(p);
  const int64_t qrows = (int64_t)p.B * p.Hq * p.Tq, krows = (int64_t)p.B * p.Hkv * p.Tk;
  if (qrows >= ((int64_t)1 << 31) || krows >= ((int64_t)1 << 31)) return false;
  constexpr auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  auto map16 = [&](CUtensorMap* m, const uint16_t* ptr, int64_t rows, int box_rows) {
    return make_map_box(m, ptr, DH, (uint64_t)rows, DH, 64u, (uint32_t)box_rows, SW, true);
  };
  CUtensorMap kh, kl, vh, vl, qh, ql, gh, gl;                 // dK/dV kernel
  CUtensorMap qh128, ql128, gh128, gl128, kkh, kkl, vkh, vkl;  // dQ kernel
  const bool built = map16(&kh, w.k16h, krows, BK) && map16(&kl, w.k16l, krows, BK) &&
                     map16(&vh, w.v16h, krows, BK) && map16(&vl, w.v16l, krows, BK) &&
                     map16(&qh, w.q16h, qrows, Kv16Layout<DH>::BQ) &&
                     map16(&ql, w.q16l, qrows, Kv16Layout<DH>::BQ) &&
                     map16(&gh, w.g16h, qrows, Kv16Layout<DH>::BQ) &&
                     map16(&gl, w.g16l, qrows, Kv16Layout<DH>::BQ) &&
                     map16(&qh128, w.q16h, qrows, QM) && map16(&ql128, w.q16l, qrows, QM) &&
                     map16(&gh128, w.g16h, qrows, QM) && map16(&gl128, w.g16l, qrows, QM) &&
                     map16(&kkh, w.k16h, krows, Q16Layout<DH>::KN) &&
                     map16(&kkl, w.k16l, krows, Q16Layout<DH>::KN) &&
                     map16(&vkh, w.v16h, krows, Q16Layout<DH>::KN) &&
                     map16(&vkl, w.v16l, krows, Q16Layout<DH>::KN);
  if (!built) return false;
  // Q, K, V pairs: from the 3xTF32 pairs a producer left in the workspace
  // (maxima, then the split), kept from this call's binary16 forward, or
  // prepared from q, k, v here
  if (p.pairs16) {
    // written by the QKV GEMM epilogue
  } else if (p.qkv_ready) {
    const int64_t nq4 = qrows * DH / 4, nk4 = krows * DH / 4;
    const int64_t most = nq4 > nk4 ? nq4 : nk4;
    const int64_t want = (most + 255) / 256, cap = (int64_t)sm_count() * 8;
    const dim3 eg((unsigned)(want < cap ? want : cap), 3);
    cudaMemsetAsync(w.amax16, 0, 3 * sizeof(unsigned), stream);
    attn16_amax_kernel<<<eg, 256, 0, stream>>>(w.qh, w.ql, nq4, w.kh, w.kl, w.vh, w.vl, nk4,
                                               w.amax16);
    attn16_split_qkv_kernel<<<eg, 256, 0, stream>>>(w.qh, w.ql, nq4, w.kh, w.kl, w.vh, w.vl,
                                                    nk4, w.q16h, w.q16l, w.k16h, w.k16l, w.v16h,
                                                    w.v16l, w.amax16);
    count_launch(2);
  } else if (!p.ws_ready) {
    attention_prepare_pairs16(p, stream);
  }
  // row statistics and max |dO|, then dO's pair (with pairs16 the dO GEMM
  // epilogue wrote them)
  if (!p.pairs16) {
    cudaMemsetAsync(w.amax16 + 3, 0, sizeof(unsigned), stream);
    const int64_t want = (qrows + 7) / 8, cap = (int64_t)sm_count() * 16;
    const unsigned rg = (unsigned)(want < cap ? want : cap);
    auto go = [&](auto v, auto vl) {
      constexpr int V = decltype(v)::value;
      constexpr bool VL = decltype(vl)::value;
      attn16_stats_kernel<V, VL><<<rg, 256, 0, stream>>>(p, o, o_lo, dout, row_max, row_sum,
                                                         delta, w.lse2, w.amax16);
      attn16_split_dout_kernel<V, VL><<<rg, 256, 0, stream>>>(p, dout, w.g16h, w.g16l, w.amax16);
    };
    // read width by alignment
    if (rows_vec4(o, o_lo) && rows_vec4(dout, nullptr))
      go(std::integral_constant<int, 4>{}, std::true_type{});
    else if (rows_vec2(o, o_lo) && rows_vec2(dout, nullptr))
      go(std::integral_constant<int, 2>{}, std::true_type{});
    else
      go(std::integral_constant<int, 2>{}, std::false_type{});
    count_launch(2);
  }
  cudaMemsetAsync(w.slot_flags, 0, (size_t)w.chunk_slots * sizeof(int), stream);
  Bwd16Args a{w.lse2, delta, p.pairs16 ? p.pair_amax : w.amax16, device_error_word(), w.chunks,
              w.slot_flags, w.chunk_slots, p.pairs16 ? p.pair_exps : nullptr};
  dim3 g1((p.Tk + BK - 1) / BK, p.Hkv, p.B);
  dim3 g2((p.Tq + QM - 1) / QM, p.Hq, p.B);
  // instances: with / without the mask code, three products / one
  auto go = [&](auto masked, auto three) {
    constexpr bool M = decltype(masked)::value, T3 = decltype(three)::value;
    cudaFuncSetAttribute(attn_bwd_kv_f16_kernel<DH, M, T3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, Kv16Layout<DH>::SMEM);
    cudaFuncSetAttribute(attn_bwd_q_f16_kernel<DH, M, T3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, Q16Layout<DH>::SMEM);
    attn_bwd_kv_f16_kernel<DH, M, T3><<<g1, THREADS, Kv16Layout<DH>::SMEM, stream>>>(
        kh, kl, vh, vl, qh, ql, gh, gl, p, dk, dv, a);
    attn_bwd_q_f16_kernel<DH, M, T3><<<g2, THREADS, Q16Layout<DH>::SMEM, stream>>>(
        qh128, ql128, gh128, gl128, kkh, kkl, vkh, vkl, p, dq, a);
  };
  using Y = std::true_type;
  using N = std::false_type;
  if (p.mask != nullptr) {
    if (p.single) go(Y{}, N{}); else go(Y{}, Y{});
  } else {
    if (p.single) go(N{}, N{}); else go(N{}, Y{});
  }
  count_launch(2);
  return true;
}

}  // namespace

bool attention_backward_f16(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                            const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                            AttnOut dk, AttnOut dv, cudaStream_t stream) {
  if (p.ws == nullptr || encode_fn() == nullptr || p.Tq == 0 || p.Tk == 0) return false;
  // the dO pair comes from dout, or with pairs16 from the dO GEMM epilogue
  if (p.pairs16 ? !p.grad_ready || !(p.ws_ready || p.qkv_ready) || p.pair_exps == nullptr ||
                      p.pair_amax == nullptr
                : p.grad_ready)
    return false;
  if ((reinterpret_cast<uintptr_t>(p.ws) | reinterpret_cast<uintptr_t>(p.ws_grad)) & 15) return false;
  switch (p.Dh) {
    case 64:
      return launch_bwd_f16<64>(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
    case 128:
      return launch_bwd_f16<128>(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
    default:
      return false;
  }
}

}  // namespace etb
