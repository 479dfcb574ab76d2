// A2 causal attention forward on tcgen05 with binary16 operand pairs
// (sm_100a), and the binary16 operand preparation both directions share.
//
// Semantics are those of attention_tc.cu's forward
// (native/a2_attention_provider.c:669-716): O = softmax(s) V over the admitted
// keys, s = scale q.k, the row statistics (maximum of the scaled scores, sum
// of exponentials) returned for the backward.  Operands are binary16 hi / lo
// pairs with one power-of-two exponent per tensor (attention_bwd_f16.cu
// states the scheme): Q, K, V from their maxima, P with 2^7 (the lazy
// rescale below lets P reach 2^8 of the row's stale maximum, and 2^15 stays
// under binary16's 65,504).  Each product is hi hi + hi lo + lo hi (one
// product, hi hi, in the TF32-grade mode).  Against the 3xTF32 forward the
// tiles are half the bytes: at head_dim 128 two K/V stages fit shared memory
// (the 3xTF32 kernel holds one), and at head_dim 64 the key blocks are 128
// wide, so the score MMAs run at N = 128 (the tensor pipe's full rate; N = 64
// instructions take 45-48 cycles for 32 cycles of arithmetic).
//
// One CTA per 128 queries of one (batch, head); TMEM lane = query row.
// Warps 0-7 compute probabilities (two per row: key halves), warp 8 issues
// S = Q K^T, warp 9 O += P V, warp 10 loads K/V stages by TMA.  Q hi lives in
// TMEM (A operand), Q lo in shared memory; two TMEM slots of S (P's pair is
// written over S, each thread over its own columns); O in TMEM with the lazy
// rescale of attention_tc.cu (the stale row maximum stands until a block
// exceeds it by 2^8).  P hi times [V hi | V lo] is one MMA of N = 2 head_dim
// (V lo sits one 64-column chunk stride after V hi), into O's 2 head_dim
// columns, plus P lo times V hi into the first half; the epilogue adds the
// halves.  All mbarrier waits are bounded; a timeout raises a
// CTA-wide abort flag, in-flight copies and MMAs are waited for (bounded) and
// TMEM is always released.
#include <cuda_fp16.h>

#include <type_traits>

#include "attention_f16.cuh"

namespace etb {

namespace {

using namespace f16att;

constexpr int kPExpFwd = 7;         // P pairs carry P 2^7 (P <= 2^8 before normalisation)
constexpr float kRescale = 8.0f;  // log2 of the largest P the stale maximum allows

// ---- operand preparation ---------------------------------------------------------

// max |x| of the raw Q, K, V (blockIdx.y = 0, 1, 2; strided [B, H, T, Dh])
// into amax[blockIdx.y]: warps take rows in a grid-stride loop, each lane
// VEC elements per step, one atomic per warp.  RoPE rotates pairs, so a
// rotated element is at most sqrt(2) max |x|: with 2^e max |x| below 2^15
// the pairs stay under 65,504.
template <int VEC, bool VLOAD>
__global__ void attn16_amax_raw_kernel(AttnParams p, unsigned* amax) {
  const int t = blockIdx.y;
  const AttnTensor& x = t == 0 ? p.q : t == 1 ? p.k : p.v;
  const int H = t == 0 ? p.Hq : p.Hkv, T = t == 0 ? p.Tq : p.Tk;
  const int64_t rows = (int64_t)p.B * H * T;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  float m = 0.0f;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int tt = (int)(row % T);
    const int h = (int)((row / T) % H);
    const int b = (int)(row / ((int64_t)T * H));
    const float* s = x.ptr + b * x.sb + h * x.sh + (int64_t)tt * x.st;
    for (int j = VEC * lane; j < p.Dh; j += 32 * VEC) {
      float v[VEC];
      load_vec<VEC, VLOAD>(s + j, v);
#pragma unroll
      for (int u = 0; u < VEC; u++) {
        m = fmaxf(m, fabsf(v[u]));
        if (v[u] != v[u]) m = v[u];
      }
    }
  }
  amax_record_warp(amax + t, m);
}

// The binary16 pairs of RoPE'd Q, K and plain V (blockIdx.y = 0, 1, 2),
// head-major [B, H, T, Dh]: the rotation in the reference's rounding order
// (attention_tc.cu's prepass), then x 2^e split into hi and lo; warps take
// rows in a grid-stride loop, each lane VEC elements (VEC / 2 pairs) per step.
template <int VEC, bool VLOAD>
__global__ void attn16_split_rope_kernel(AttnParams p, uint16_t* q16h, uint16_t* q16l,
                                         uint16_t* k16h, uint16_t* k16l, uint16_t* v16h,
                                         uint16_t* v16l, const unsigned* amax) {
  const int t = blockIdx.y;
  const AttnTensor& x = t == 0 ? p.q : t == 1 ? p.k : p.v;
  const int H = t == 0 ? p.Hq : p.Hkv, T = t == 0 ? p.Tq : p.Tk;
  const float* ct = t == 0 ? p.q_cos : t == 1 ? p.k_cos : nullptr;
  const float* st = t == 0 ? p.q_sin : t == 1 ? p.k_sin : nullptr;
  const int batched = t == 0 ? p.q_rope_batched : p.k_rope_batched;
  uint16_t* oh = t == 0 ? q16h : t == 1 ? k16h : v16h;
  uint16_t* ol = t == 0 ? q16l : t == 1 ? k16l : v16l;
  const float sc = exp2_int(pair_exponent(__uint_as_float(amax[t])));
  const int half = p.Dh / 2;
  const int64_t rows = (int64_t)p.B * H * T;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int tt = (int)(row % T);
    const int h = (int)((row / T) % H);
    const int b = (int)(row / ((int64_t)T * H));
    const float* s = x.ptr + b * x.sb + h * x.sh + (int64_t)tt * x.st;
    const int64_t trow = (int64_t)(batched ? b * T + tt : tt) * half;
    for (int j = VEC * lane; j < p.Dh; j += 32 * VEC) {
      float v[VEC];
      load_vec<VEC, VLOAD>(s + j, v);
#pragma unroll
      for (int u = 0; u < VEC; u += 2) {
        float x0 = v[u], x1 = v[u + 1];
        if (ct != nullptr) {
          const int64_t ti = trow + (j + u) / 2;
          const float c = ct[ti], sn = st[ti];
          const float aa = rn_mul(x0, c), bb = rn_mul(x1, sn), cc = rn_mul(x0, sn),
                      dd = rn_mul(x1, c);
          x0 = rn_sub(aa, bb);
          x1 = rn_add(cc, dd);
        }
        float hi, lo;
        pair2(x0 * sc, x1 * sc, hi, lo);
        const int64_t o = row * p.Dh + j + u;
        *reinterpret_cast<uint32_t*>(oh + o) = __float_as_uint(hi);
        *reinterpret_cast<uint32_t*>(ol + o) = __float_as_uint(lo);
      }
    }
  }
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
// a / b from rb = RN(1 / b), corrected once with the exact remainder
// (Markstein's refinement, as attention_tc.cu's epilogue divides).
__device__ __forceinline__ float div_by(float a, float b, float rb) {
  const float q = __fmul_rn(a, rb);
  const float r = __fmaf_rn(-q, b, a);
  return __fmaf_rn(r, rb, q);
}

// ---- forward kernel ----------------------------------------------------------------

constexpr int QM = 128;  // query rows per CTA
constexpr int THREADS = 352;
constexpr int SOFT = 256;  // probability threads (warps 0-7)
constexpr int MMA_S = 8, MMA_O = 9, LOADER = 10;

template <int DH>
struct Fwd16Layout {
  static constexpr int KN = DH == 128 ? 64 : 128;  // keys per block
  static constexpr int NKH = KN / 2;                // keys per probability thread
  static constexpr int KT = KN * DH * 2;            // one binary16 [KN, DH] tile
  static constexpr int STAGE = 4 * KT;              // K hi, K lo, V hi, V lo
  static constexpr int RT = QM * DH * 2;            // one binary16 [128, DH] row tile
  static constexpr int QLO = 2 * STAGE;             // Q lo rows (A operand of the lo pass)
  static constexpr int BARS = QLO + RT;
  static constexpr int SMEM = BARS + 256 + 1024;
  static_assert(RT <= STAGE, "Q hi rows pass through stage 1");
  static_assert(QM * (DH + 4) * 4 <= 2 * STAGE, "output staging");
  // TMEM: Q hi (two elements per column), two S slots (the P pair over S), O
  // (f32-grade: 2 DH columns, P hi V hi + P lo V hi in the first DH and P hi
  // V lo in the second, added in the epilogue)
  static constexpr uint32_t QH = 0, S0 = DH / 2, O = S0 + 2 * KN;
  static constexpr uint32_t COLS = 512;
  static_assert(O + 2 * DH <= COLS, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory");
};

struct Fwd16Args {
  const unsigned* amax;  // [0..2] max |x| of Q, K, V
  int* error;
  const int* exps;       // non-null: the producers' exponents of Q, K, V
};

template <int DH, bool MASKED, bool THREE>
__global__ void __launch_bounds__(THREADS, 1)
attn_fwd_f16_kernel(const __grid_constant__ CUtensorMap qh_map,
                    const __grid_constant__ CUtensorMap ql_map,
                    const __grid_constant__ CUtensorMap kh_map,
                    const __grid_constant__ CUtensorMap kl_map,
                    const __grid_constant__ CUtensorMap vh_map,
                    const __grid_constant__ CUtensorMap vl_map, AttnParams p, AttnOut o,
                    float* __restrict__ row_max, float* __restrict__ row_sum, Fwd16Args a) {
  if constexpr (!MASKED) p.mask = nullptr;
  using L = Fwd16Layout<DH>;
  constexpr int KN = L::KN, NKH = L::NKH, NCH = NKH / 32;  // 32-key chunks per thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ int64_t kpos_s[2 * KN];     // key positions of the block, ring of 2
  __shared__ float xmax[2 * 2 * QM];     // [block parity][half][row] maxima / exp-sums
  __shared__ float lrow_s[QM], rrow_s[QM];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  // per-slot / per-stage barriers come in pairs (0, 1): block j uses stage and
  // slot j & 1 and waits phase (j >> 1) & 1
  enum {
    FULL0, FULL1, EMPTY0, EMPTY1, SFULL0, SFULL1, PVD0, PVD1, PREADY0, PREADY1, KP0, KP1,
    ROWS_HI, ROWS_LO, PAIR0, PAIR1, PAIR2, PAIR3, DRAIN_S, DRAIN_O, NBARS
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
  const uint32_t rows_hi = base + L::STAGE;  // stage 1 until block 1 arrives
  if (tid == 0) {
    for (int i = 0; i < NBARS; i++) {
      const uint32_t n = (i == PREADY0 || i == PREADY1)           ? SOFT
                         : (i == KP0 || i == KP1)                 ? 32
                         : (i >= PAIR0 && i <= PAIR3)             ? 64
                                                                  : 1;
      mbar_init(B_(i), n);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
    const int r = (int)(((int64_t)b * p.Hq + hq) * p.Tq + q0);
    mbar_expect_tx(B_(ROWS_LO), L::RT);
    mbar_expect_tx(B_(ROWS_HI), L::RT);
#pragma unroll
    for (int c = 0; c < DH / 64; c++) {
      const uint32_t off = (uint32_t)c * QM * 128u;
      tma_load_2d(base + L::QLO + off, &ql_map, B_(ROWS_LO), 64 * c, r);
      tma_load_2d(rows_hi + off, &qh_map, B_(ROWS_HI), 64 * c, r);
    }
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  int nkb = 0, full_kb = 0;
  {
    const int qlast = min(q0 + QM, p.Tq) - 1;
    const int64_t qmax = p.qpos[(int64_t)b * p.Tq + qlast];
    const int64_t qmin = p.qpos[(int64_t)b * p.Tq + q0];
    const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
    const int seen = warp_count(kp, p.Tk, qmax, true);
    const int seen_all = warp_count(kp, seen, qmin, true);
    nkb = (seen + KN - 1) / KN;
    full_kb = (p.mask == nullptr && q0 + QM <= p.Tq) ? seen_all / KN : 0;
  }
  const int64_t kv_row0 = ((int64_t)b * p.Hkv + hkv) * p.Tk;
  auto load_stage = [&](int j) {  // K hi/lo, V hi/lo of block j into stage j & 1
    const uint32_t bar = B_(FULL0 + (j & 1)), dst = base + (uint32_t)(j & 1) * L::STAGE;
    const int r = (int)(kv_row0 + (int64_t)j * KN);
    mbar_expect_tx(bar, L::STAGE);
#pragma unroll
    for (int c = 0; c < DH / 64; c++) {
      const uint32_t off = (uint32_t)c * KN * 128u;
      tma_load_2d(dst + off, &kh_map, bar, 64 * c, r);
      tma_load_2d(dst + L::KT + off, &kl_map, bar, 64 * c, r);
      tma_load_2d(dst + 2 * L::KT + off, &vh_map, bar, 64 * c, r);
      tma_load_2d(dst + 3 * L::KT + off, &vl_map, bar, 64 * c, r);
    }
  };
  // block 0 goes out before the set-up barrier (the thread that initialised
  // the barriers issues it)
  if (tid == 0 && nkb > 0) load_stage(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
  // Q hi rows -> TMEM (warps 0-3; DH/2 columns)
  if (warp < 4) {
    const bool ok = mbar_wait(B_(ROWS_HI), 0u, a.error);
    if (!ok) *abort = 1;
    if (__all_sync(0xffffffffu, ok)) {
      tile_row16_to_tmem<DH>(rows_hi, row, trow, L::QH);
      tmem_wait_st();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == LOADER) {
    // ---- producer: stages one block ahead, key positions by the lanes
    int nk = nkb > 0 ? 1 : 0;
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
      if (lane == 0) {  // stage jn & 1 is free once the P V of block jn - 2 completed
        if (jn >= 2) ok = role_wait(B_(EMPTY0 + (jn & 1)), (uint32_t)(((jn >> 1) - 1) & 1), a.error, abort);
        if (ok) { load_stage(jn); nk++; }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // position slot jn & 1 is free once block jn - 2's probabilities are out
      if (ok && jn >= 2) ok = role_wait(B_(PREADY0 + (jn & 1)), (uint32_t)(((jn >> 1) - 1) & 1), a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) fill_kpos(jn);
    }
    if (lane == 0) {  // every copy has landed before the CTA releases its memory
      mbar_wait(B_(ROWS_LO), 0u, a.error);
      for (int j = nk - 2 < 0 ? 0 : nk - 2; j < nk; j++)
        mbar_wait(B_(FULL0 + (j & 1)), (uint32_t)((j >> 1) & 1), a.error);
    }
  } else if (warp == MMA_S) {
    // ---- S = Q K^T into slot j & 1
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc = idesc_f16_m128(KN, 0);
      const uint32_t qlo = base + L::QLO;
      bool ok = role_wait(B_(ROWS_LO), 0u, a.error, abort);
      for (int j = 0; ok && j < nkb; j++) {
        const int s = j & 1;
        ok = role_wait(B_(FULL0 + s), (uint32_t)((j >> 1) & 1), a.error, abort);
        // the slot holds P of block j - 2 until its P V completes
        if (ok && j >= 2) ok = role_wait(B_(PVD0 + s), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kt = base + (uint32_t)s * L::STAGE;
        const uint32_t d = tmem + L::S0 + (uint32_t)s * KN;
#pragma unroll
        for (int k = 0; k < DH / 16; k++) {
          const uint64_t bh = kdesc16<KN>(kt, k), bl = kdesc16<KN>(kt + L::KT, k);
          umma_f16_ts(d, tmem + L::QH + 8 * k, bh, idesc, k > 0 ? 1u : 0u);
          if (THREE) {
            umma_f16_ts(d, tmem + L::QH + 8 * k, bl, idesc, 1u);
            umma_f16(d, kdesc16<QM>(qlo, k), bh, idesc, 1u);
          }
        }
        umma_commit(B_(SFULL0 + s));
      }
      umma_commit(B_(DRAIN_S));
      mbar_wait(B_(DRAIN_S), 0u, a.error);
    }
  } else if (warp == MMA_O) {
    // ---- O += P V
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc = idesc_f16_m128(DH, 1);
      // V hi and V lo sit one 64-column chunk stride apart in the stage, so one
      // MN-major descriptor of N = 2 DH covers [V hi | V lo]: P hi times both
      // in one instruction (the pipe's full rate at N = 128)
      constexpr uint32_t idesc2 = idesc_f16_m128(2 * DH, 1);
      static_assert(L::KT == (DH / 64) * KN * 128, "V lo one chunk stride after V hi");
      bool ok = true;
      for (int j = 0; ok && j < nkb; j++) {
        const int s = j & 1;
        ok = role_wait(B_(PREADY0 + s), (uint32_t)((j >> 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vt = base + (uint32_t)s * L::STAGE + 2u * L::KT;
        const uint32_t sd = tmem + L::S0 + (uint32_t)s * KN;
#pragma unroll
        for (int k = 0; k < KN / 16; k++) {
          // keys 16k..16k+15: the hi / lo columns of the half that wrote them
          const int h = k / (NKH / 16), kk = k % (NKH / 16);
          const uint32_t ah = sd + (uint32_t)(NKH * h + 8 * kk);
          const uint64_t bh = mdesc16<KN>(vt, k);
          if (THREE) {
            umma_f16_ts(tmem + L::O, ah, bh, idesc2, (j > 0 || k > 0) ? 1u : 0u);
            umma_f16_ts(tmem + L::O, ah + (uint32_t)(NKH / 2), bh, idesc, 1u);
          } else {
            umma_f16_ts(tmem + L::O, ah, bh, idesc, (j > 0 || k > 0) ? 1u : 0u);
          }
        }
        umma_commit(B_(PVD0 + s));
        umma_commit(B_(EMPTY0 + s));
      }
      umma_commit(B_(DRAIN_O));
      mbar_wait(B_(DRAIN_O), 0u, a.error);
    }
  } else {
    // ---- probabilities: this thread's NKH keys of each block, row shared with warp w ^ 4
    const Exps ex = exps_of(a.amax, DH, a.exps);
    const float c2 = p.scale * kLog2e * exp2_int(-(ex.q + ex.k));  // base-2 score scale
    const float s_p = exp2_int(kPExpFwd);
    const int cb = NKH * khalf;
    const int64_t qpos_row = valid_q ? p.qpos[(int64_t)b * p.Tq + tq] : INT64_MIN;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; ok && j < nkb; j++) {
      const int s = j & 1;
      const uint32_t spar = (uint32_t)((j >> 1) & 1);
      const bool full_block = j < full_kb;
      ok = role_wait(B_(KP0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SFULL0 + s), spar, a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t slot = trow + L::S0 + (uint32_t)s * KN;
      float sv[NKH];
      float bmax = -INFINITY;
      const int seen = full_block ? KN : count_below(kpos_s + s * KN, KN, qpos_row + 1) - cb;
      const int64_t mrow = ((int64_t)b * p.Tq + min(tq, p.Tq - 1)) * p.Tk;
#pragma unroll
      for (int c = 0; c < NCH; c++) {
        float v[32];
        tmem_ld32(slot + cb + 32 * c, v);
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int kk = 32 * c + i;
          bool adm = full_block || kk < seen;
          if (!full_block && p.mask != nullptr)
            adm = adm && p.mask[mrow + min(j * KN + cb + kk, p.Tk - 1)] != 0;
          sv[kk] = adm ? v[i] * c2 : -INFINITY;
          bmax = fmaxf(bmax, sv[kk]);
        }
      }
      // warps w and w+4 hold the two halves of these rows: exchange maxima
      float* xm = xmax + (j & 1) * 2 * QM;
      xm[khalf * QM + row] = bmax;
      mbar_arrive(B_(PAIR0 + quarter));
      ok = __all_sync(0xffffffffu, role_wait(B_(PAIR0 + quarter), (uint32_t)(j & 1), a.error, abort));
      if (!ok) break;
      bmax = fmaxf(bmax, xm[(1 - khalf) * QM + row]);
      // a stale maximum stands until this block exceeds it by more than 2^kRescale
      float factor = 1.0f;
      const bool jump = bmax > m_used + kRescale;  // false for -inf blocks
      if (jump) {
        factor = m_used == -INFINITY ? 0.0f : ex2(m_used - bmax);
        l *= factor;
        m_used = bmax;
      }
      if (__any_sync(0xffffffffu, jump && factor != 0.0f)) {
        // O already holds earlier blocks: wait for the last P V, rescale this half
        bool w = true;
        if (j > 0) w = role_wait(B_(PVD0 + ((j - 1) & 1)), (uint32_t)(((j - 1) >> 1) & 1), a.error, abort);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        tc_fence_after();
        constexpr int OC = THREE ? 2 * DH : DH;  // O's columns
#pragma unroll
        for (int c = 0; c < OC / 64; c++) {
          const uint32_t col = L::O + (uint32_t)(khalf * (OC / 2) + 32 * c);
          float ov[32];
          tmem_ld32(trow + col, ov);
#pragma unroll
          for (int i = 0; i < 32; i++) ov[i] *= factor;
          tmem_st32(trow + col, ov);
        }
      }
      // P pairs: hi of this thread's NKH keys in its first NKH/2 columns, lo
      // in the next NKH/2 (its S columns, all read above)
#pragma unroll
      for (int c = 0; c < NCH; c++) {
        float pv[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float x = sv[32 * c + i];
          pv[i] = (x == -INFINITY) ? 0.0f : ex2(x - m_used);
          l += pv[i];
        }
        float hi[16], lo[16];
        pack_pairs(pv, s_p, hi, lo);
        tmem_st16(slot + cb + 16 * c, hi);
        tmem_st16(slot + cb + NKH / 2 + 16 * c, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(B_(PREADY0 + s));
    }
    if (ok && nkb > 0) {
      const int jl = nkb - 1;
      ok = role_wait(B_(PVD0 + (jl & 1)), (uint32_t)((jl >> 1) & 1), a.error, abort);
    }
    ok = __all_sync(0xffffffffu, ok);
    // full exp-sum of the row from the two halves (one more exchange)
    float* xl = xmax + (nkb & 1) * 2 * QM;
    xl[khalf * QM + row] = l;
    mbar_arrive(B_(PAIR0 + quarter));
    if (ok) ok = __all_sync(0xffffffffu, role_wait(B_(PAIR0 + quarter), (uint32_t)(nkb & 1), a.error, abort));
    const float lsum = l + xl[(1 - khalf) * QM + row];
    const bool empty = lsum == 0.0f;
    if (ok && valid_q && khalf == 0) {
      const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
      row_max[ri] = empty ? 0.0f : m_used * kLn2;
      row_sum[ri] = empty ? 0.0f : lsum;
    }
    if (khalf == 0) {
      lrow_s[row] = (empty || nkb == 0) ? 0.0f : lsum;
      rrow_s[row] = (empty || nkb == 0) ? 0.0f : rn_div(1.0f, lsum);
    }
    // raw O rows (back to f32 scale) staged in the freed stages; o = O / l and
    // the output format are formed while the rows are written out (coalesced)
    const uint32_t stage = base;
    if (ok) {
      tc_fence_after();
      const float un = exp2_int(-(kPExpFwd + ex.v));
#pragma unroll
      for (int c = 0; c < DH / 64; c++) {
        const int col = khalf * (DH / 2) + 32 * c;
        float ov[32];
        if (nkb > 0) {
          tmem_ld32(trow + L::O + col, ov);
          if (THREE) {  // plus the P hi V lo half
            float o2[32];
            tmem_ld32(trow + L::O + DH + col, o2);
#pragma unroll
            for (int i = 0; i < 32; i++) ov[i] += o2[i];
          }
#pragma unroll
          for (int i = 0; i < 32; i++) ov[i] *= un;
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) ov[i] = 0.0f;
        }
        stage_row32(stage, DH, row, col, ov, 0, 32);
      }
    }
    named_sync(1, SOFT);
    float amax = 0.0f;
    if (ok) {
      const int64_t oo = b * o.sb + hq * o.sh + (int64_t)q0 * o.st;
      store_rows_split(stage, DH, min(QM, p.Tq - q0), o.ptr, o.lo, oo, o.st, tid, SOFT,
                       [&](int r, int, float4& v) {
                         const float lr = lrow_s[r], rl = rrow_s[r];
                         if (lr == 0.0f) {
                           v = make_float4(0.f, 0.f, 0.f, 0.f);
                         } else {
                           v.x = div_by(v.x, lr, rl); v.y = div_by(v.y, lr, rl);
                           v.z = div_by(v.z, lr, rl); v.w = div_by(v.w, lr, rl);
                         }
                       }, o.sc, amax);
    }
    if (o.sc.amax != nullptr) amax_record_warp(o.sc.amax, amax);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::COLS);
  }
}

template <int DH>
bool launch_fwd_f16(const AttnParams& p, AttnOut o, float* m, float* l, cudaStream_t stream) {
  using L = Fwd16Layout<DH>;
  const AttnWs w = attn_ws(p);
  const int64_t qrows = (int64_t)p.B * p.Hq * p.Tq, krows = (int64_t)p.B * p.Hkv * p.Tk;
  if (qrows >= ((int64_t)1 << 31) || krows >= ((int64_t)1 << 31)) return false;
  constexpr auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  auto map16 = [&](CUtensorMap* mp, const uint16_t* ptr, int64_t rows, int box_rows) {
    return make_map_box(mp, ptr, DH, (uint64_t)rows, DH, 64u, (uint32_t)box_rows, SW, true);
  };
  CUtensorMap qh, ql, kh, kl, vh, vl;
  if (!map16(&qh, w.q16h, qrows, QM) || !map16(&ql, w.q16l, qrows, QM) ||
      !map16(&kh, w.k16h, krows, L::KN) || !map16(&kl, w.k16l, krows, L::KN) ||
      !map16(&vh, w.v16h, krows, L::KN) || !map16(&vl, w.v16l, krows, L::KN))
    return false;
  // the pairs: from a producer (pairs16), else prepared here from q, k, v
  if (!p.pairs16) attention_prepare_pairs16(p, stream);
  Fwd16Args a{p.pairs16 ? p.pair_amax : w.amax16, device_error_word(),
              p.pairs16 ? p.pair_exps : nullptr};
  dim3 grid((p.Tq + QM - 1) / QM, p.Hq, p.B);
  auto go = [&](auto masked, auto three) {
    constexpr bool M = decltype(masked)::value, T3 = decltype(three)::value;
    cudaFuncSetAttribute(attn_fwd_f16_kernel<DH, M, T3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    attn_fwd_f16_kernel<DH, M, T3><<<grid, THREADS, L::SMEM, stream>>>(qh, ql, kh, kl, vh, vl, p,
                                                                       o, m, l, a);
  };
  using Y = std::true_type;
  using N = std::false_type;
  if (p.mask != nullptr) {
    if (p.single) go(Y{}, N{}); else go(Y{}, Y{});
  } else {
    if (p.single) go(N{}, N{}); else go(N{}, Y{});
  }
  count_launch();
  return true;
}

}  // namespace

bool attention_uses_pairs16(const AttnParams& p) {
  // head_dim 64: from 768^2 the binary16 forward + backward measured faster
  // than 3xTF32 (9 % at 768^2, 2 % at 512^2: the backward's 128-query and
  // 128-key blocks; the forward alone wins only from 4,096^2), below it the
  // preparation passes weigh more
  const bool long_seq = (int64_t)p.Tq * p.Tk >= (int64_t)768 * 768;
  return p.Dh == 128 || (p.Dh == 64 && (p.bwd_pairs16 || long_seq));
}

void attention_prepare_pairs16(const AttnParams& p, cudaStream_t stream) {
  const AttnWs w = attn_ws(p);
  cudaMemsetAsync(w.amax16, 0, 3 * sizeof(unsigned), stream);
  const int64_t most = (int64_t)p.B * (p.Hq > p.Hkv ? p.Hq : p.Hkv) * (p.Tq > p.Tk ? p.Tq : p.Tk);
  const int64_t want = (most + 7) / 8, cap = (int64_t)sm_count() * 16;
  const dim3 g((unsigned)(want < cap ? want : cap), 3);
  // read width by alignment (a pair's two floats are always adjacent)
  const int vec = rows_vec4(p.q, nullptr) && rows_vec4(p.k, nullptr) && rows_vec4(p.v, nullptr) ? 4
                  : rows_vec2(p.q, nullptr) && rows_vec2(p.k, nullptr) && rows_vec2(p.v, nullptr) ? 2
                                                                                                  : 0;
  auto go = [&](auto v, auto vl) {
    constexpr int V = decltype(v)::value;
    constexpr bool VL = decltype(vl)::value;
    attn16_amax_raw_kernel<V, VL><<<g, 256, 0, stream>>>(p, w.amax16);
    attn16_split_rope_kernel<V, VL><<<g, 256, 0, stream>>>(p, w.q16h, w.q16l, w.k16h, w.k16l,
                                                           w.v16h, w.v16l, w.amax16);
  };
  if (vec == 4) go(std::integral_constant<int, 4>{}, std::true_type{});
  else if (vec == 2) go(std::integral_constant<int, 2>{}, std::true_type{});
  else go(std::integral_constant<int, 2>{}, std::false_type{});
  count_launch(2);
}

bool attention_forward_f16(const AttnParams& p, AttnOut o, float* row_max, float* row_sum,
                           cudaStream_t stream) {
  if (p.ws == nullptr || encode_fn() == nullptr || p.Tq == 0 || p.Tk == 0) return false;
  if ((reinterpret_cast<uintptr_t>(p.ws) | reinterpret_cast<uintptr_t>(p.ws_grad)) & 15) return false;
  if (p.pairs16 && (!p.qkv_ready || p.pair_exps == nullptr || p.pair_amax == nullptr)) return false;
  switch (p.Dh) {
    case 64: return launch_fwd_f16<64>(p, o, row_max, row_sum, stream);
    case 128: return launch_fwd_f16<128>(p, o, row_max, row_sum, stream);
    default: return false;
  }
}

}  // namespace etb
