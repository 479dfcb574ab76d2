// A2 causal attention forward on tcgen05 tensor cores (sm_100a, 3xTF32).
//
// Semantics are those of attention.cu (native/a2_attention_provider.c:
// 221-318, 669-716): s = (q . k) / sqrt(Dh) over admitted keys, o = softmax(s)
// v, +0 for a row with no admitted key; the row max m (natural-log domain)
// and the exp-sum l are kept for the backward pass.
//
// Operand preparation (attn_prepare): one bandwidth pass applies RoPE to Q
// and K in registers (bit-identical rotation, host libm tables) and splits
// Q, K, V into tf32-exact hi and residual lo tensors, head-major
// [B, H, T, Dh], so every tile below is a plain TMA box.
//
// Main kernel: one CTA owns 128 query rows of one (batch, head); TMEM lane r
// is query row r.  Warps 0-7 run the softmax (warp w: rows 32*(w%4).., key
// columns 32*(w/4).. of each 64-key block; the two threads of a row exchange
// their block maxima through shared memory); warp 8 issues S = Q K^T, warp 9
// issues O += P V (one thread each), warp 10 loads K/V tiles by TMA.
//   Q hi/lo  TMA -> shared -> TMEM (A operand of every S MMA)
//   K, V     TMA (128-byte swizzle; K 16-byte atoms, V 32-byte atoms),
//            hi and lo tiles, 3 stages (1 for Dh 128)
//   S        kind::tf32 MMAs with A from TMEM, 3 passes; two S slots for
//            Dh <= 64, so S of block j+1 runs during the softmax of block j
//   softmax  base-2 online softmax; P hi/lo -> TMEM (P hi over S)
//   O       += P V, A = P from TMEM, B = V (MN-major), 3 passes
// The softmax keeps a stale row maximum until a block's maximum exceeds it
// by more than 2^8: P = 2^(s - m_used) then stays below 256 and O, l share
// the same scale, so the O rows in TMEM are rescaled (after the previous
// P V completes) only on those rare jumps.  All mbarrier waits are bounded;
// a timeout raises a CTA-wide abort flag, in-flight copies and MMAs are
// waited for (bounded) and TMEM is always released.
#include <type_traits>

#include "attention_tc.cuh"

namespace etb {

namespace {

constexpr int QM = 128;  // query rows per CTA
constexpr int KN = 64;   // keys per block
constexpr int THREADS = 352;
constexpr int SOFT = 256;  // softmax threads (warps 0-7)
constexpr int MMA_S = 8, MMA_O = 9, LOADER = 10;
constexpr float kRescale = 8.0f;  // log2 of the largest P the stale maximum allows

template <int DH>
struct FwdLayout {
  static constexpr int NSLOT = DH <= 64 ? 2 : 1;   // S / P lo slots in TMEM
  static constexpr int NSTAGE = DH <= 64 ? 3 : 1;  // K/V stages in shared memory
  static constexpr int KT = KN * DH * 4;           // one [KN, DH] tile
  static constexpr int STAGE = 4 * KT;             // K hi, K lo (K-major), V hi, V lo (MN-major)
  static constexpr int RT = QM * DH * 4;           // one [128, DH] row tile
  // the last stage also carries the Q row tiles (before the loop; with one
  // stage nothing is loaded meanwhile) and stage 0 the output rows (after it)
  static constexpr int QROWS = NSTAGE >= 2 ? (NSTAGE - 1) * STAGE : 0;
  static constexpr int PRELOAD = NSTAGE >= 2 ? NSTAGE - 1 : 0;  // blocks loaded meanwhile
  static_assert(NSTAGE < 2 || 2 * RT <= STAGE, "Q rows in one stage");
  static constexpr int SMEM_BUF =
      NSTAGE * STAGE >= QROWS + 2 * RT ? NSTAGE * STAGE : QROWS + 2 * RT;
  static_assert(QM * (DH + 4) * 4 <= SMEM_BUF, "output stage");
  static constexpr int BARS = SMEM_BUF;
  static constexpr int SMEM = BARS + 256 + 1024;
  static constexpr uint32_t QH = 0, QL = DH, S0 = 2 * DH, PL0 = S0 + NSLOT * KN,
                            O = PL0 + NSLOT * KN;
  static constexpr uint32_t COLS = (O + DH) <= 256 ? 256 : 512;
  static_assert(O + DH <= 512, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory");
};

struct TcFwdArgs {
  int* error;
};

// ---- operand preparation -------------------------------------------------------

// src element (b, h, t, j) -> hi/lo at ((b*H + h)*T + t)*Dh + j, with RoPE on
// pairs (j, j+1) when a table is given (table row b*T + t or t).
__global__ void attn_prepare_kernel(AttnTensor src, int B, int H, int T, int Dh,
                                    const float* __restrict__ ct, const float* __restrict__ st,
                                    int batched, float* __restrict__ hi, float* __restrict__ lo) {
  const int half = Dh >> 1;
  const int64_t total = (int64_t)B * H * T * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int pr = (int)(i % half);
    const int64_t row = i / half;  // (b*H + h)*T + t
    const int t = (int)(row % T);
    const int h = (int)((row / T) % H);
    const int b = (int)(row / ((int64_t)T * H));
    const float* s = src.ptr + b * src.sb + h * src.sh + (int64_t)t * src.st + 2 * pr;
    float x0 = s[0], x1 = s[1];
    if (ct != nullptr) {
      const int64_t ti = (int64_t)(batched ? b * T + t : t) * half + pr;
      const float c = ct[ti], sn = st[ti];
      const float aa = rn_mul(x0, c), bb = rn_mul(x1, sn), cc = rn_mul(x0, sn), dd = rn_mul(x1, c);
      x0 = rn_sub(aa, bb);
      x1 = rn_add(cc, dd);
    }
    const float h0 = tf32_hi(x0), h1 = tf32_hi(x1);
    const int64_t o = row * Dh + 2 * pr;
    *reinterpret_cast<float2*>(hi + o) = make_float2(h0, h1);
    *reinterpret_cast<float2*>(lo + o) = make_float2(x0 - h0, x1 - h1);
  }
}

// a / b from rb = RN(1 / b): the quotient q = RN(a rb) corrected once with
// the exact remainder a - q b (one FMA) -- Markstein's division refinement
// (P. Markstein, IA-64 and Elementary Functions, 2000), which rounds correctly
// except in rare boundary cases (then within one unit in the last place).
__device__ __forceinline__ float div_by(float a, float b, float rb) {
  const float q = __fmul_rn(a, rb);
  const float r = __fmaf_rn(-q, b, a);
  return __fmaf_rn(r, rb, q);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// Number of entries of the ascending array a[0..n) that are below x.
__device__ __forceinline__ int count_below(const int64_t* a, int n, int64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---- forward kernel --------------------------------------------------------------

// MASKED: the instance for calls with a boolean mask; the other one drops the
// mask code (smaller unrolled loops).
template <int DH, bool MASKED, bool THREE>
__global__ void __launch_bounds__(THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap qh_map, const __grid_constant__ CUtensorMap ql_map,
                   const __grid_constant__ CUtensorMap kh_map, const __grid_constant__ CUtensorMap kl_map,
                   const __grid_constant__ CUtensorMap vh_map, const __grid_constant__ CUtensorMap vl_map,
                   AttnParams p, AttnOut o, float* __restrict__ row_max,
                   float* __restrict__ row_sum, TcFwdArgs a) {
  if constexpr (!MASKED) p.mask = nullptr;
  using L = FwdLayout<DH>;
  constexpr int NSL = L::NSLOT, NST = L::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ int64_t kpos_s[2 * KN];     // key positions of the block, ring of 2
  __shared__ float xmax[2 * 2 * QM];     // [block parity][half][row] maxima / exp-sums
  __shared__ float lrow_s[QM], rrow_s[QM];  // row exp-sums and their reciprocals (output pass)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  // barrier slots: full[NST] | empty[NST] | s_full[NSL] | pv_done[NSL] | p_ready[2] |
  // kp_full[2] | rows | pair[4] (the two softmax warps of a lane quarter)
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t FULL = bar0, EMPTY = FULL + 8 * NST, SFULL = EMPTY + 8 * NST,
                 PVD = SFULL + 8 * NSL, PREADY = PVD + 8 * NSL, KPFULL = PREADY + 16,
                 ROWS = KPFULL + 16, PAIR = ROWS + 8;
  constexpr int NBARS = 2 * NST + 2 * NSL + 9;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, khalf = (warp >> 2) & 1;
  const int row = quarter * 32 + lane;  // query row in the tile == TMEM lane
  const int q0 = blockIdx.x * QM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / (p.Hq / p.Hkv);
  const int tq = q0 + row;
  const bool valid_q = tq < p.Tq;
  if (tid == 0) {
    for (int i = 0; i < NBARS; i++) {
      const uint32_t bar = bar0 + 8 * i;
      const bool soft = bar == PREADY || bar == PREADY + 8;
      const bool kp = bar == KPFULL || bar == KPFULL + 8;
      const bool pair = bar >= PAIR;
      mbar_init(bar, soft ? SOFT : kp ? 32 : pair ? 64 : 1);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
    // Q hi/lo rows pass through the last K/V stage (the first ones receive
    // key blocks meanwhile) on their way to TMEM
    mbar_expect_tx(ROWS, 2 * L::RT);
    const int r = (int)(((int64_t)b * p.Hq + hq) * p.Tq + q0);
    const uint32_t qs = smem_u32(smem) + L::QROWS;
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t off = (uint32_t)c * QM * 128u;
      tma_load_2d(qs + off, &qh_map, ROWS, 32 * c, r);
      tma_load_2d(qs + L::RT + off, &ql_map, ROWS, 32 * c, r);
    }
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  // key blocks that can hold an admitted key, and the number of leading
  // blocks visible to every row of the tile (positions strictly increase)
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
  const uint32_t base = smem_u32(smem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
  const int64_t kv_row0 = ((int64_t)b * p.Hkv + hkv) * p.Tk;
  // ---- loader (warp LOADER): K/V stages by TMA, key positions by the lanes;
  // the blocks whose stages the Q rows leave free are issued while the
  // softmax warps move Q into TMEM
  int loads = 0;
  bool lok = true;
  auto load_block = [&](int j) {
    const int st = j % NST;
    bool ok = true;
    if (lane == 0) {
      if (j >= NST) ok = role_wait(EMPTY + 8 * st, (uint32_t)((j / NST - 1) & 1), a.error, abort);
      if (ok) {
        const uint32_t bar = FULL + 8 * st, dst = base + st * L::STAGE;
        const int r = (int)(kv_row0 + (int64_t)j * KN);
        mbar_expect_tx(bar, L::STAGE);
#pragma unroll
        for (int c = 0; c < DH / 32; c++) {
          const uint32_t off = (uint32_t)c * KN * 128u;
          tma_load_2d(dst + off, &kh_map, bar, 32 * c, r);
          tma_load_2d(dst + L::KT + off, &kl_map, bar, 32 * c, r);
          tma_load_2d(dst + 2 * L::KT + off, &vh_map, bar, 32 * c, r);
          tma_load_2d(dst + 3 * L::KT + off, &vl_map, bar, 32 * c, r);
        }
        loads++;
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok && j >= 2) ok = role_wait(PREADY + 8 * (j & 1), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
#pragma unroll
      for (int h = 0; h < KN / 32; h++) {
        const int t = j * KN + 32 * h + lane;
        kpos_s[(j & 1) * KN + 32 * h + lane] = t < p.Tk ? p.kpos[(int64_t)b * p.Tk + t] : INT64_MAX;
      }
      mbar_arrive(KPFULL + 8 * (j & 1));
    }
    lok = ok;
  };
  const int pre = min(L::PRELOAD, nkb);
  if (warp == LOADER) {
    for (int j = 0; lok && j < pre; j++) load_block(j);
  } else if (warp < 8) {
    const bool ok = mbar_wait(ROWS, 0u, a.error);
    if (!ok) *abort = 1;
    if (__all_sync(0xffffffffu, ok)) {
      tile_row_to_tmem<DH>(base + L::QROWS + (uint32_t)khalf * L::RT, row, trow,
                           khalf == 0 ? L::QH : L::QL);
      tmem_wait_st();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == LOADER) {
    for (int j = pre; lok && j < nkb; j++) load_block(j);
    if (lane == 0) {  // every copy has landed before the CTA releases its memory
      for (int j = loads - NST < 0 ? 0 : loads - NST; j < loads; j++)
        mbar_wait(FULL + 8 * (j % NST), (uint32_t)((j / NST) & 1), a.error);
    }
  } else if (warp == MMA_S) {
    // ---- S = Q K^T (3 passes) into slot j % NSLOT
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc = idesc_tf32_m128(KN, 0);
      int issued = 0;
      bool ok = true;
      for (int j = 0; ok && j < nkb; j++) {
        const int sl = j % NSL, st = j % NST;
        ok = role_wait(FULL + 8 * st, (uint32_t)((j / NST) & 1), a.error, abort);
        // the slot holds P of block j - NSLOT until its P V completes
        if (ok && j >= NSL) ok = role_wait(PVD + 8 * sl, (uint32_t)((j / NSL - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t stg = base + st * L::STAGE;
        const uint64_t kh = kmajor_desc(stg, KN, 0), kl = kmajor_desc(stg + L::KT, KN, 0);
        const uint32_t d = tmem + L::S0 + sl * KN;
#pragma unroll
        for (int k = 0; k < DH / 8; k++) {
          const uint32_t acc = k > 0 ? 1u : 0u;
          umma_tf32_ts(d, tmem + L::QH + 8 * k, kslice<KN>(kh, k), idesc, acc);
          if (THREE) {
            umma_tf32_ts(d, tmem + L::QH + 8 * k, kslice<KN>(kl, k), idesc, 1u);
            umma_tf32_ts(d, tmem + L::QL + 8 * k, kslice<KN>(kh, k), idesc, 1u);
          }
        }
        umma_commit(SFULL + 8 * sl);
        issued++;
      }
      if (issued > 0)  // committed MMAs finish before TMEM is released
        mbar_wait(SFULL + 8 * ((issued - 1) % NSL), (uint32_t)(((issued - 1) / NSL) & 1), a.error);
    }
  } else if (warp == MMA_O) {
    // ---- O += P V (3 passes)
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc = idesc_tf32_m128(DH, 1);
      int issued = 0;
      bool ok = true;
      for (int j = 0; ok && j < nkb; j++) {
        const int sl = j % NSL, st = j % NST;
        ok = role_wait(PREADY + 8 * (j & 1), (uint32_t)((j >> 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t stg = base + st * L::STAGE;
        const uint64_t vh = mnmajor_desc(stg + 2 * L::KT, KN, 0),
                       vl = mnmajor_desc(stg + 3 * L::KT, KN, 0);
        const uint32_t ph = tmem + L::S0 + sl * KN, pl = tmem + L::PL0 + sl * KN;
#pragma unroll
        for (int k = 0; k < KN / 8; k++) {
          const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
          umma_tf32_ts(tmem + L::O, ph + 8 * k, mslice(vh, k), idesc, acc);
          if (THREE) {
            umma_tf32_ts(tmem + L::O, ph + 8 * k, mslice(vl, k), idesc, 1u);
            umma_tf32_ts(tmem + L::O, pl + 8 * k, mslice(vh, k), idesc, 1u);
          }
        }
        umma_commit(PVD + 8 * sl);
        umma_commit(EMPTY + 8 * st);
        issued++;
      }
      if (issued > 0) {  // committed MMAs finish before TMEM and shared memory are released
        const int jl = issued - 1;
        mbar_wait(PVD + 8 * (jl % NSL), (uint32_t)((jl / NSL) & 1), a.error);
        mbar_wait(EMPTY + 8 * (jl % NST), (uint32_t)((jl / NST) & 1), a.error);
      }
    }
  } else {
    // ---- softmax: this thread's 32 keys of each block, row shared with warp w^4
    const float c2 = p.scale * kLog2e;  // base-2 score scale
    const int cb = 32 * khalf;
    const int64_t qpos_row = valid_q ? p.qpos[(int64_t)b * p.Tq + tq] : INT64_MIN;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; ok && j < nkb; j++) {
      const int sl = j % NSL;
      const bool full_block = j < full_kb;
      uint8_t keep[32];
      if (!full_block && p.mask != nullptr) {  // clamped indices stay in bounds
        const int64_t mrow = ((int64_t)b * p.Tq + min(tq, p.Tq - 1)) * p.Tk;
#pragma unroll
        for (int i = 0; i < 32; i++) keep[i] = p.mask[mrow + min(j * KN + cb + i, p.Tk - 1)];
      }
      ok = role_wait(KPFULL + 8 * (j & 1), (uint32_t)((j >> 1) & 1), a.error, abort);
      if (ok) ok = role_wait(SFULL + 8 * sl, (uint32_t)((j / NSL) & 1), a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float s[32];
      tmem_ld32(trow + L::S0 + sl * KN + cb, s);
      float bmax = -INFINITY;
      if (full_block) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          s[i] *= c2;
          bmax = fmaxf(bmax, s[i]);
        }
      } else {
        // keys of the block this row sees: those whose position does not exceed its own
        const int seen = count_below(kpos_s + (j & 1) * KN, KN, qpos_row + 1) - cb;
#pragma unroll
        for (int i = 0; i < 32; i++) {
          bool adm = i < seen;
          if (p.mask != nullptr) adm = adm && keep[i] != 0;
          s[i] = adm ? s[i] * c2 : -INFINITY;
          bmax = fmaxf(bmax, s[i]);
        }
      }
      // warps w and w+4 hold the two halves of these rows: exchange maxima
      // (a slot per block parity; a slot is rewritten only after the partner
      // has passed the next exchange, so after it read this one)
      float* xm = xmax + (j & 1) * 2 * QM;
      xm[khalf * QM + row] = bmax;
      mbar_arrive(PAIR + 8 * quarter);
      ok = __all_sync(0xffffffffu, role_wait(PAIR + 8 * quarter, (uint32_t)(j & 1), a.error, abort));
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
        if (j > 0)
          w = role_wait(PVD + 8 * ((j - 1) % NSL), (uint32_t)(((j - 1) / NSL) & 1), a.error, abort);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < (DH >= 64 ? DH / 64 : 1); c++) {
          const uint32_t col = L::O + (DH >= 64 ? (uint32_t)(khalf * (DH / 2) + 32 * c) : 0u);
          if (DH >= 64 || khalf == 0) {
            float ov[32];
            tmem_ld32(trow + col, ov);
#pragma unroll
            for (int i = 0; i < 32; i++) ov[i] *= factor;
            tmem_st32(trow + col, ov);
          }
        }
      }
      float ph[32], pl[32];
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const float pv = (s[i] == -INFINITY) ? 0.0f : ex2(s[i] - m_used);
        l += pv;
        ph[i] = tf32_round(pv);
        pl[i] = pv - ph[i];
      }
      tmem_st32(trow + L::S0 + sl * KN + cb, ph);
      tmem_st32(trow + L::PL0 + sl * KN + cb, pl);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(PREADY + 8 * (j & 1));
    }
    if (ok && nkb > 0)
      ok = role_wait(PVD + 8 * ((nkb - 1) % NSL), (uint32_t)(((nkb - 1) / NSL) & 1), a.error, abort);
    ok = __all_sync(0xffffffffu, ok);
    // full exp-sum of the row from the two halves (one more exchange)
    float* xl = xmax + (nkb & 1) * 2 * QM;
    xl[khalf * QM + row] = l;
    mbar_arrive(PAIR + 8 * quarter);
    if (ok) ok = __all_sync(0xffffffffu, role_wait(PAIR + 8 * quarter, (uint32_t)(nkb & 1), a.error, abort));
    const float lsum = l + xl[(1 - khalf) * QM + row];
    const bool empty = lsum == 0.0f;
    if (ok && valid_q && khalf == 0) {
      const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
      row_max[ri] = empty ? 0.0f : m_used * kLn2;
      row_sum[ri] = empty ? 0.0f : lsum;
    }
    // the raw O rows are staged in the free stages with their exp-sums (0 for
    // a row without admitted keys); o = O / l, split into the TF32 hi part
    // (o) and the residual (o.lo) when o.lo is set, is formed while the rows
    // are written out (coalesced)
    if (khalf == 0) {
      lrow_s[row] = (empty || nkb == 0) ? 0.0f : lsum;
      rrow_s[row] = (empty || nkb == 0) ? 0.0f : rn_div(1.0f, lsum);
    }
    const uint32_t stage = base;
    if (ok) {
      tc_fence_after();
      if constexpr (DH >= 64) {
#pragma unroll
        for (int c = 0; c < DH / 64; c++) {
          const int col = khalf * (DH / 2) + 32 * c;
          float ov[32];
          if (nkb > 0) {
            tmem_ld32(trow + L::O + col, ov);
          } else {
#pragma unroll
            for (int i = 0; i < 32; i++) ov[i] = 0.0f;
          }
          stage_row32(stage, DH, row, col, ov, 0, 32);
        }
      } else {
        float ov[32];
        if (nkb > 0) {
          tmem_ld32(trow + L::O, ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) ov[i] = 0.0f;
        }
        if (khalf == 0) stage_row32(stage, DH, row, 0, ov, 0, 16);
        else stage_row32(stage, DH, row, 16, ov, 16, 16);
      }
    }
    named_sync(1, SOFT);
    float amax = 0.0f;
    if (ok) {
      const int64_t oo = b * o.sb + hq * o.sh + (int64_t)q0 * o.st;
      store_rows_split(stage, DH, min(QM, p.Tq - q0), o.ptr, o.lo, oo, o.st, tid, SOFT,
                       [&](int r, int, float4& v) {
                         const float l = lrow_s[r], rl = rrow_s[r];
                         if (l == 0.0f) {
                           v = make_float4(0.f, 0.f, 0.f, 0.f);
                         } else {
                           v.x = div_by(v.x, l, rl); v.y = div_by(v.y, l, rl);
                           v.z = div_by(v.z, l, rl); v.w = div_by(v.w, l, rl);
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
bool launch_fwd_tc(const AttnParams& p, AttnOut o, float* m, float* l, cudaStream_t stream) {
  using L = FwdLayout<DH>;
  const AttnWs w = attn_ws(p);
  const int64_t qrows = (int64_t)p.B * p.Hq * p.Tq, krows = (int64_t)p.B * p.Hkv * p.Tk;
  if (qrows >= ((int64_t)1 << 31) || krows >= ((int64_t)1 << 31)) return false;
  constexpr auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  constexpr auto SW32 = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
  if (!make_map(&mqh, w.qh, DH, qrows, DH, QM, SW) || !make_map(&mql, w.ql, DH, qrows, DH, QM, SW) ||
      !make_map(&mkh, w.kh, DH, krows, DH, KN, SW) || !make_map(&mkl, w.kl, DH, krows, DH, KN, SW) ||
      !make_map(&mvh, w.vh, DH, krows, DH, KN, SW32) || !make_map(&mvl, w.vl, DH, krows, DH, KN, SW32))
    return false;
  if (!p.qkv_ready) attention_prepare_qkv(p, w, stream);
  TcFwdArgs a{device_error_word()};
  dim3 grid((p.Tq + QM - 1) / QM, p.Hq, p.B);
  // instances: with / without the mask code, three products / one
  auto go = [&](auto masked, auto three) {
    constexpr bool M = decltype(masked)::value, T3 = decltype(three)::value;
    cudaFuncSetAttribute(attn_fwd_tc_kernel<DH, M, T3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    attn_fwd_tc_kernel<DH, M, T3><<<grid, THREADS, L::SMEM, stream>>>(mqh, mql, mkh, mkl, mvh, mvl,
                                                                      p, o, m, l, a);
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

void attention_prepare_qkv(const AttnParams& p, const AttnWs& w, cudaStream_t stream) {
  const int threads = 256;
  auto prep = [&](const AttnTensor& t, int H, int T, const float* ct, const float* st, int bat,
                  float* hi, float* lo) {
    const int64_t pairs = (int64_t)p.B * H * T * (p.Dh / 2);
    const int64_t want = (pairs + threads - 1) / threads;
    const int grid = (int)(want < (int64_t)sm_count() * 32 ? want : (int64_t)sm_count() * 32);
    if (grid > 0)
      attn_prepare_kernel<<<grid, threads, 0, stream>>>(t, p.B, H, T, p.Dh, ct, st, bat, hi, lo);
  };
  prep(p.q, p.Hq, p.Tq, p.q_cos, p.q_sin, p.q_rope_batched, w.qh, w.ql);
  prep(p.k, p.Hkv, p.Tk, p.k_cos, p.k_sin, p.k_rope_batched, w.kh, w.kl);
  prep(p.v, p.Hkv, p.Tk, nullptr, nullptr, 0, w.vh, w.vl);
  count_launch(3);
}

bool attention_qkv_prep(const AttnParams& p, QkvPrep* out) {
  if (p.ws == nullptr || (reinterpret_cast<uintptr_t>(p.ws) & 15)) return false;
  if (p.Dh != 32 && p.Dh != 64 && p.Dh != 128) return false;
  if (p.Tq != p.Tk) return false;  // one qkv matrix holds every operand
  if (p.pairs16 && (p.Dh == 32 || p.pair_exps == nullptr)) return false;
  const AttnWs w = attn_ws(p);
  QkvPrep q{};
  q.T = p.Tq; q.Hq = p.Hq; q.Hkv = p.Hkv; q.Dh = p.Dh;
  q.q_cos = p.q_cos; q.q_sin = p.q_sin; q.k_cos = p.k_cos; q.k_sin = p.k_sin;
  q.q_rope_batched = p.q_rope_batched; q.k_rope_batched = p.k_rope_batched;
  q.qh = w.qh; q.ql = w.ql; q.kh = w.kh; q.kl = w.kl; q.vh = w.vh; q.vl = w.vl;
  if (p.pairs16) {
    q.q16h = w.q16h; q.q16l = w.q16l; q.k16h = w.k16h; q.k16l = w.k16l;
    q.v16h = w.v16h; q.v16l = w.v16l;
    q.exps = p.pair_exps;
  }
  q.amax = p.pair_amax;
  *out = q;
  return true;
}

void attention_prepare_from_qkv(const float* qkv, int64_t ld, int rows, const QkvPrep& q,
                                cudaStream_t stream) {
  const int B = rows / q.T;
  AttnParams p{};
  p.B = B; p.Hq = q.Hq; p.Hkv = q.Hkv; p.Tq = q.T; p.Tk = q.T; p.Dh = q.Dh;
  const int64_t sb = (int64_t)q.T * ld;
  p.q = AttnTensor{qkv, sb, q.Dh, ld};
  p.k = AttnTensor{qkv + (int64_t)q.Hq * q.Dh, sb, q.Dh, ld};
  p.v = AttnTensor{qkv + (int64_t)(q.Hq + q.Hkv) * q.Dh, sb, q.Dh, ld};
  p.q_cos = q.q_cos; p.q_sin = q.q_sin; p.k_cos = q.k_cos; p.k_sin = q.k_sin;
  p.q_rope_batched = q.q_rope_batched; p.k_rope_batched = q.k_rope_batched;
  AttnWs w{};
  w.qh = q.qh; w.ql = q.ql; w.kh = q.kh; w.kl = q.kl; w.vh = q.vh; w.vl = q.vl;
  attention_prepare_qkv(p, w, stream);
}

size_t attention_qkv_workspace_floats(const AttnParams& p) {
  const size_t nq = (size_t)p.B * p.Hq * p.Tq * p.Dh, nk = (size_t)p.B * p.Hkv * p.Tk * p.Dh;
  return 2 * nq + 4 * nk;
}
size_t attention_grad_workspace_floats(const AttnParams& p) {
  const size_t nq = (size_t)p.B * p.Hq * p.Tq * p.Dh, rows = (size_t)p.B * p.Hq * p.Tq;
  const size_t nk = (size_t)p.B * p.Hkv * p.Tk * p.Dh;
  // dO pair, lse2, then the binary16 K and V pairs, the operand maxima, the
  // chunk slots' flags and the chunk sums
  const size_t slots = (size_t)attn_chunk_slots();
  return 2 * nq + ((rows + 63) & ~(size_t)63) + 2 * nk + 64 + ((slots + 63) & ~(size_t)63) +
         slots * (size_t)kBwdChunkFloats;
}
size_t attention_workspace_floats(const AttnParams& p) {
  return attention_qkv_workspace_floats(p) + attention_grad_workspace_floats(p);
}

bool attention_forward_tc(const AttnParams& p, AttnOut o, float* row_max, float* row_sum,
                          cudaStream_t stream) {
  if (p.ws == nullptr || encode_fn() == nullptr) return false;
  if (reinterpret_cast<uintptr_t>(p.ws) & 15) return false;
  // binary16 pairs where the backward takes them too (it then reuses the
  // pairs), unless a producer already wrote the 3xTF32 operands; a
  // producer's binary16 pairs always go to the binary16 kernel
  if (p.pairs16 || (!p.qkv_ready && attention_uses_pairs16(p)))
    return attention_forward_f16(p, o, row_max, row_sum, stream);
  switch (p.Dh) {
    case 32: return launch_fwd_tc<32>(p, o, row_max, row_sum, stream);
    case 64: return launch_fwd_tc<64>(p, o, row_max, row_sum, stream);
    case 128: return launch_fwd_tc<128>(p, o, row_max, row_sum, stream);
    default: return false;
  }
}

}  // namespace etb
