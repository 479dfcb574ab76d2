// A2 causal attention backward on tcgen05 tensor cores (sm_100a, 3xTF32).
//
// Semantics are those of the SIMT backward in attention.cu
// (native/a2_attention_provider.c:416-666): with P = softmax(S) recomputed
// from the forward statistics, dV = P^T dO, dP = dO V^T,
// dS = P (dP - delta) with delta = rowsum(dO * O), dQ = scale dS K,
// dK = scale dS^T Q, then the RoPE backward rotation on dQ and dK.  Two
// kernels keep every sum in a fixed order (no atomics):
//
//   dK/dV kernel: one CTA per 128 keys of one (batch, kv head); TMEM lane r is
//     key r.  K hi and V hi sit in TMEM (A operands), K lo / V lo in shared
//     memory.  For each 64-query block of every query head of the group:
//       S^T  = K Q^T,  dP^T = V dO^T     (B = Q, dO K-major)
//       P^T, dS^T in registers -> TMEM hi/lo (P^T hi over S^T, dS^T hi over dP^T)
//       dV  += P^T dO, dK += dS^T Q     (B = dO, Q MN-major)
//   dQ kernel: one CTA per 128 queries of one (batch, head), TMEM lane r is
//     query r; Q and dO hi/lo in TMEM.  For each 64-key block:
//       S = Q K^T, dP = dO V^T (B = K, V K-major); dS -> TMEM hi/lo;
//       dQ += dS K (B = K MN-major)
//   Each kernel issues its MMAs from two threads in two warps, one chain per
//   accumulator pair (a single issuing thread tops out near one N = 64 MMA
//   per 46 cycles, two keep the tensor core busy); while one chain waits for
//   the probabilities of a block the other chain's MMAs run.
//
// A prepass writes the RoPE'd, TF32-split head-major Q/K/V (shared with the
// forward) and a second one dO hi/lo, delta and the base-2 log-sum-exp of
// every query row, so P = 2^(s scale log2(e) - lse2).  All mbarrier waits
// are bounded; a timeout raises a CTA-wide abort flag, in-flight copies and
// MMAs are waited for (bounded) and TMEM is always released.
#include <type_traits>

#include "attention_tc.cuh"

namespace etb {

namespace {

// ---- prepass -----------------------------------------------------------------------

// Base-2 log-sum-exp of a query row from the forward's statistics (+inf for
// a row with no admitted key, so every P of it is 0).
__device__ __forceinline__ float lse2_of(float m, float l) {
  return l > 0.0f ? (m + logf(l)) * kLog2e : INFINITY;
}

// One warp per query row (b, hq, tq), row = (b*Hq + hq)*Tq + tq: delta in the
// SIMT kernel's order (lane-strided fma, warp tree), lse2, dO hi/lo.
__global__ void attn_bwd_prepare_kernel(AttnParams p, AttnTensor o, const float* __restrict__ o_lo,
                                        AttnTensor dout, const float* __restrict__ row_max,
                                        const float* __restrict__ row_sum,
                                        float* __restrict__ delta, float* __restrict__ lse2,
                                        float* __restrict__ doh, float* __restrict__ dol) {
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
  for (int j = lane; j < p.Dh; j += 32) {
    const float g = grow[j];
    s = fmaf(g, lrow ? orow[j] + lrow[j] : orow[j], s);
    const float h = tf32_hi(g);
    doh[row * p.Dh + j] = h;
    dol[row * p.Dh + j] = g - h;
  }
  s = warp_sum(s);
  if (lane == 0) {
    delta[row] = s;
    lse2[row] = lse2_of(row_max[row], row_sum[row]);
  }
}

struct TcBwdArgs {
  const float *kh, *vh;     // head-major K, V hi (dK/dV kernel)
  const float *qh, *ql;     // head-major Q hi/lo (dQ kernel)
  const float *doh, *dol;   // head-major dO hi/lo (dQ kernel)
  const float *lse2, *delta;
  int* error;
  float* chunks;     // dK/dV chunk sums, kBwdChunkFloats per slot
  int* slot_flags;   // 0 free, 1 taken
  int chunk_slots;
};

// dK and dV accumulate over up to G Tq queries; the tensor pipe's f32
// accumulation truncates, so a CTA whose key tile sees more than
// kChunkBlocks query blocks (1,024 queries: 3xTF32 issues twice the MMAs per
// query of the binary16 kernels) sums its accumulators in chunks: at every
// chunk boundary the probability warps add the finished chunk into the CTA's
// slot in global memory (f32), and the next chunk restarts the TMEM
// accumulation.
constexpr int kChunkBlocks = 16;

// A free chunk slot for this CTA (thread 0, after its TMEM allocation):
// bounded scan from a CTA-dependent start; -1 (and the error word) if none
// is free, which cannot happen with one slot-holding CTA per SM.
__device__ __forceinline__ int take_chunk_slot(const TcBwdArgs& a) {
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

// Number of entries of the ascending array a[0..n) that are below x.
__device__ __forceinline__ int count_below(const int64_t* a, int n, int64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---- warp roles ----------------------------------------------------------------------------
//
// Warps 0-7 compute probabilities (TMEM lane quarter w%4, column half w/4 of
// every block); warps 8 and 9 each issue one chain of tcgen05 MMAs from one
// thread (a single issuing thread cannot keep the tensor core busy with
// N = 64 tiles, two can); warp 10 loads operand tiles by TMA and stages
// per-block row data.  Hand-offs are mbarriers, and every wait is at most one
// phase behind its barrier.

constexpr int THREADS = 352;
constexpr int SOFT = 256;  // probability threads (warps 0-7)
constexpr int MMA_A = 8, MMA_B = 9, LOADER = 10;

// ---- dK / dV ---------------------------------------------------------------------------

constexpr int BK = 128;  // keys per CTA (TMEM lanes)
constexpr int BQ = 64;   // queries per block

template <int DH>
struct KvLayout {
  static constexpr int QT = BQ * DH * 4;  // [BQ, DH] tile: DH/32 chunks of BQ rows x 128 B
  static constexpr int KT = BK * DH * 4;  // [BK, DH] tile
  // K lo, V lo (shared-memory A operands), then hi+lo pairs of Q and dO,
  // K-major (B of S^T, dP^T) and MN-major (B of dK, dV)
  static constexpr int KL = 0, VL = KT, QK = 2 * KT, GK = QK + 2 * QT, GM = GK + 2 * QT,
                       QM = GM + 2 * QT;
  static constexpr int BARS = QM + 2 * QT;
  static constexpr int SMEM = BARS + 256 + 1024;
  // TMEM: K hi, V hi (A operands), dK, dV accumulators, S^T, dP^T, P^T lo,
  // dS^T lo (P^T hi over S^T, dS^T hi over dP^T)
  static constexpr uint32_t KH = 0, VH = DH, DK = 2 * DH, DV = 3 * DH, ST = 4 * DH,
                            DPT = ST + BQ, PL = ST + 2 * BQ, DSL = ST + 3 * BQ;
  static constexpr uint32_t COLS = 512;
  static_assert(DSL + BQ <= COLS, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory");
};

// MASKED: the instance for calls with a boolean mask; the other one drops the
// mask code (smaller unrolled loops).
template <int DH, bool MASKED, bool THREE>
__global__ void __launch_bounds__(THREADS, 1)
attn_bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap kh_map,
                      const __grid_constant__ CUtensorMap vh_map,
                      const __grid_constant__ CUtensorMap kl_map,
                      const __grid_constant__ CUtensorMap vl_map,
                      const __grid_constant__ CUtensorMap qkh_map,
                      const __grid_constant__ CUtensorMap qkl_map,
                      const __grid_constant__ CUtensorMap gkh_map,
                      const __grid_constant__ CUtensorMap gkl_map,
                      const __grid_constant__ CUtensorMap qmh_map,
                      const __grid_constant__ CUtensorMap qml_map,
                      const __grid_constant__ CUtensorMap gmh_map,
                      const __grid_constant__ CUtensorMap gml_map, AttnParams p, AttnOut dk,
                      AttnOut dv, TcBwdArgs a) {
  if constexpr (!MASKED) p.mask = nullptr;
  using L = KvLayout<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(16) float lse_s[2 * BQ], dlt_s[2 * BQ];  // per-block statistics ring
  __shared__ __align__(16) int64_t qp_s[2 * BQ];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  enum {
    LO_FULL, QK_FULL, QK_EMPTY, GK_FULL, GK_EMPTY, GM_FULL, GM_EMPTY, QM_FULL, QM_EMPTY,
    SA_DONE, SB_DONE, P_READY, VA_DONE, KB_DONE, D_READY0, D_READY1, ST_FULL0, ST_FULL1,
    CHUNK_DONE, NBARS
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
  if (tid == 0) {
    for (int i = 0; i < NBARS; i++) {
      const uint32_t n = (i == P_READY || i == D_READY0 || i == D_READY1 || i == CHUNK_DONE) ? SOFT
                         : (i == ST_FULL0 || i == ST_FULL1)               ? 32
                                                                          : 1;
      mbar_init(B_(i), n);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  // query blocks that can see a key of this tile: from the first query whose
  // position reaches the first key's, for every query head of the group
  const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
  const int64_t* qp = p.qpos + (int64_t)b * p.Tq;
  const uint32_t base = smem_u32(smem);
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
  if (tid == 0 && n_it > 0) {
    // the key tile: K, V lo stay in shared memory as A operands; K, V hi pass
    // through the MN-major Q/dO buffers (needed last by the first block) on
    // their way to TMEM
    mbar_expect_tx(B_(LO_FULL), 4 * L::KT);
    const int r = (int)(((int64_t)b * p.Hkv + hkv) * p.Tk + k0);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * BK * 128u;
      tma_load_2d(base + L::KL + o, &kl_map, B_(LO_FULL), 32 * c, r);
      tma_load_2d(base + L::VL + o, &vl_map, B_(LO_FULL), 32 * c, r);
      tma_load_2d(base + L::GM + o, &kh_map, B_(LO_FULL), 32 * c, r);
      tma_load_2d(base + L::QM + o, &vh_map, B_(LO_FULL), 32 * c, r);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  auto load_pair = [&](int full, const CUtensorMap* hm, const CUtensorMap* lm, int off, int r) {
    mbar_expect_tx(B_(full), 2 * L::QT);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * BQ * 128u;
      tma_load_2d(base + off + o, hm, B_(full), 32 * c, r);
      tma_load_2d(base + off + L::QT + o, lm, B_(full), 32 * c, r);
    }
  };
  auto pair_row = [&](int j) { return (int)(((int64_t)b * p.Hq + hq_of(j)) * p.Tq + q0_of(j)); };
  int nqk = 0, ngk = 0, ngm = 0, nqm = 0;  // pairs issued per buffer (loader lane 0)
  // K hi (warps 0-3) and V hi (warps 4-7) rows -> TMEM, while the loader
  // issues the first block's K-major Q and dO pairs
  if (warp < 8 && n_it > 0) {
    const bool ok = mbar_wait(B_(LO_FULL), 0u, a.error);
    if (!ok) *abort = 1;
    if (__all_sync(0xffffffffu, ok)) {
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
      tile_row_to_tmem<DH>(base + (khalf == 0 ? L::GM : L::QM), row, trow,
                           khalf == 0 ? L::KH : L::VH);
      tmem_wait_st();
    }
  } else if (warp == LOADER && lane == 0 && n_it > 0) {
    load_pair(QK_FULL, &qkh_map, &qkl_map, L::QK, pair_row(0));
    load_pair(GK_FULL, &gkh_map, &gkl_map, L::GK, pair_row(0));
    nqk = ngk = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == LOADER) {
    // ---- producer: operand pairs by TMA, per-block statistics by the lanes
    bool ok = true;
    for (int j = 0; ok && j < n_it; j++) {
      const int q0 = q0_of(j), hq = hq_of(j);
      const int r = pair_row(j);
      const uint32_t prev = (uint32_t)((j - 1) & 1);
      if (lane == 0 && j > 0) {  // block 0's pairs went out with the key tile
        ok = role_wait(B_(QK_EMPTY), prev, a.error, abort);
        if (ok) { load_pair(QK_FULL, &qkh_map, &qkl_map, L::QK, r); nqk++; }
        if (ok) ok = role_wait(B_(GK_EMPTY), prev, a.error, abort);
        if (ok) { load_pair(GK_FULL, &gkh_map, &gkl_map, L::GK, r); ngk++; }
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
      if (ok && lane == 0) {
        if (j > 0) ok = role_wait(B_(GM_EMPTY), prev, a.error, abort);
        if (ok) { load_pair(GM_FULL, &gmh_map, &gml_map, L::GM, r); ngm++; }
        if (ok && j > 0) ok = role_wait(B_(QM_EMPTY), prev, a.error, abort);
        if (ok) { load_pair(QM_FULL, &qmh_map, &qml_map, L::QM, r); nqm++; }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0 && n_it > 0) {
      // every copy has landed before the CTA releases its memory (on the
      // normal path these phases completed long ago)
      mbar_wait(B_(LO_FULL), 0u, a.error);
      if (nqk > 0) mbar_wait(B_(QK_FULL), (uint32_t)((nqk - 1) & 1), a.error);
      if (ngk > 0) mbar_wait(B_(GK_FULL), (uint32_t)((ngk - 1) & 1), a.error);
      if (ngm > 0) mbar_wait(B_(GM_FULL), (uint32_t)((ngm - 1) & 1), a.error);
      if (nqm > 0) mbar_wait(B_(QM_FULL), (uint32_t)((nqm - 1) & 1), a.error);
    }
  } else if (warp == MMA_A || warp == MMA_B) {
    // ---- MMA chains.  A: S^T = K Q^T, dV += P^T dO.  B: dP^T = V dO^T, dK += dS^T Q.
    const bool is_a = warp == MMA_A;
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t idesc_s = idesc_tf32_m128(BQ, 0);
      constexpr uint32_t idesc_o = idesc_tf32_m128(DH, 1);
      const uint32_t xh = is_a ? L::KH : L::VH;                 // TMEM A operand (hi)
      const uint64_t xlo = kmajor_desc(base + (is_a ? L::KL : L::VL), BK, 0);
      const uint64_t bk_h = kmajor_desc(base + (is_a ? L::QK : L::GK), BQ, 0);
      const uint64_t bk_l = kmajor_desc(base + (is_a ? L::QK : L::GK) + L::QT, BQ, 0);
      const uint64_t bm_h = mnmajor_desc(base + (is_a ? L::GM : L::QM), BQ, 0);
      const uint64_t bm_l = mnmajor_desc(base + (is_a ? L::GM : L::QM) + L::QT, BQ, 0);
      const uint32_t sd = tmem + (is_a ? L::ST : L::DPT);       // score accumulator; hi operand after
      const uint32_t lo_op = tmem + (is_a ? L::PL : L::DSL);    // lo operand
      const uint32_t acc_d = tmem + (is_a ? L::DV : L::DK);
      const int kfull = is_a ? QK_FULL : GK_FULL, kempty = is_a ? QK_EMPTY : GK_EMPTY;
      const int mfull = is_a ? GM_FULL : QM_FULL, mempty = is_a ? GM_EMPTY : QM_EMPTY;
      const int sdone = is_a ? SA_DONE : SB_DONE, gdone = is_a ? VA_DONE : KB_DONE;
      int s_issued = 0, g_issued = 0;
      bool ok = role_wait(B_(LO_FULL), 0u, a.error, abort);
      for (int j = 0; ok && j < n_it; j++) {
        const uint32_t par = (uint32_t)(j & 1);
        ok = role_wait(B_(kfull), par, a.error, abort);
        // the score columns are free once the previous block's gradient MMAs read them
        if (ok && j > 0) ok = role_wait(B_(gdone), (uint32_t)((j - 1) & 1), a.error, abort);
        // dP^T waits for S^T: S^T then has the tensor core to itself, and
        // dP^T runs while the SM turns S^T into P^T.  S^T of the next block
        // waits for dP^T of this one, which keeps both chains within one
        // phase of these two barriers.
        if (ok && !is_a) ok = role_wait(B_(SA_DONE), par, a.error, abort);
        if (ok && is_a && j > 0) ok = role_wait(B_(SB_DONE), (uint32_t)((j - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < DH / 8; k++) {
          const uint32_t acc = k > 0 ? 1u : 0u;
          umma_tf32_ts(sd, tmem + xh + 8 * k, kslice<BQ>(bk_h, k), idesc_s, acc);
          if (THREE) {
            umma_tf32_ts(sd, tmem + xh + 8 * k, kslice<BQ>(bk_l, k), idesc_s, 1u);
            umma_tf32(sd, kslice<BK>(xlo, k), kslice<BQ>(bk_h, k), idesc_s, 1u);
          }
        }
        umma_commit(B_(sdone));
        umma_commit(B_(kempty));
        s_issued++;
        ok = role_wait(B_(is_a ? P_READY : D_READY0 + (j & 1)), is_a ? par : (uint32_t)((j >> 1) & 1),
                       a.error, abort);
        if (ok) ok = role_wait(B_(mfull), par, a.error, abort);
        // a new chunk starts once the probability warps have added the last one
        const bool restart = j % kChunkBlocks == 0;
        if (ok && restart && j > 0)
          ok = role_wait(B_(CHUNK_DONE), (uint32_t)((j / kChunkBlocks - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BQ / 8; k++) {
          const uint32_t acc = (!restart || k > 0) ? 1u : 0u;
          umma_tf32_ts(acc_d, sd + 8 * k, mslice(bm_h, k), idesc_o, acc);
          if (THREE) {
            umma_tf32_ts(acc_d, sd + 8 * k, mslice(bm_l, k), idesc_o, 1u);
            umma_tf32_ts(acc_d, lo_op + 8 * k, mslice(bm_h, k), idesc_o, 1u);
          }
        }
        umma_commit(B_(gdone));
        umma_commit(B_(mempty));
        g_issued++;
      }
      // committed MMAs finish before TMEM and shared memory are released
      if (s_issued > 0) {
        mbar_wait(B_(sdone), (uint32_t)((s_issued - 1) & 1), a.error);
        mbar_wait(B_(kempty), (uint32_t)((s_issued - 1) & 1), a.error);
      }
      if (g_issued > 0) {
        mbar_wait(B_(gdone), (uint32_t)((g_issued - 1) & 1), a.error);
        mbar_wait(B_(mempty), (uint32_t)((g_issued - 1) & 1), a.error);
      }
    }
  } else {
    // ---- P^T = 2^(S^T scale log2(e) - lse2), then dS^T = P^T (dP^T - delta)
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int64_t kpos_row = valid_k ? kp[tk] : INT64_MAX;
    const bool keys_full = k0 + BK <= p.Tk;
    const int64_t kpos_last = kp[min(k0 + BK, p.Tk) - 1];
    const float c2 = p.scale * kLog2e;
    const int cb = 32 * khalf;  // this thread's first column of the block
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
      uint8_t keep[32];
      if (p.mask != nullptr) {  // issued ahead of the waits; clamped indices stay in bounds
        const int tkc = min(tk, p.Tk - 1);
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int q = min(q0 + cb + i, p.Tq - 1);
          keep[i] = p.mask[((int64_t)b * p.Tq + q) * p.Tk + tkc];
        }
      }
      ok = role_wait(B_(ST_FULL0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SA_DONE), par, a.error, abort);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld/st are warp-collective
      if (!ok) break;
      tc_fence_after();
      const bool full_block =
          p.mask == nullptr && keys_full && q0 + BQ <= p.Tq && qp_s[s * BQ] >= kpos_last;
      float pv[32];
      {
        float sv[32], hi[32], lo[32];
        tmem_ld32(trow + L::ST + cb, sv);
        const float4* l4 = reinterpret_cast<const float4*>(lse_s + s * BQ + cb);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 v = l4[i];
          hi[4 * i] = v.x; hi[4 * i + 1] = v.y; hi[4 * i + 2] = v.z; hi[4 * i + 3] = v.w;
        }
        if (full_block) {
#pragma unroll
          for (int i = 0; i < 32; i++) pv[i] = ex2(fmaf(sv[i], c2, -hi[i]));
        } else {
          // queries of the block see this key from the first whose position
          // reaches it, up to the last query of the sequence
          const int first = count_below(qp_s + s * BQ, BQ, kpos_row) - cb;
          const int last = p.Tq - q0 - cb;
#pragma unroll
          for (int i = 0; i < 32; i++) {
            bool adm = i >= first && i < last;
            if (p.mask != nullptr) adm = adm && keep[i] != 0;
            pv[i] = adm ? ex2(fmaf(sv[i], c2, -hi[i])) : 0.0f;
          }
        }
#pragma unroll
        for (int i = 0; i < 32; i++) {
          hi[i] = tf32_round(pv[i]);
          lo[i] = pv[i] - hi[i];
        }
        tmem_st32(trow + L::ST + cb, hi);
        tmem_st32(trow + L::PL + cb, lo);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(B_(P_READY));
      }
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
        const bool first = j == kChunkBlocks;
#pragma unroll
        for (int c = 0; c < DH / 32; c++) {
          float v[32];
          tmem_ld32(trow + (khalf == 0 ? L::DK : L::DV) + 32 * c, v);
          float4* dst = reinterpret_cast<float4*>(crow + 32 * c);
#pragma unroll
          for (int u = 0; u < 8; u++) {
            float4 x = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
            if (!first) {
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
      {
        float dp[32], hi[32], lo[32];
        tmem_ld32(trow + L::DPT + cb, dp);
        const float4* d4 = reinterpret_cast<const float4*>(dlt_s + s * BQ + cb);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 v = d4[i];
          lo[4 * i] = v.x; lo[4 * i + 1] = v.y; lo[4 * i + 2] = v.z; lo[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float ds = pv[i] * (dp[i] - lo[i]);
          hi[i] = tf32_hi(ds);
          lo[i] = ds - hi[i];
        }
        tmem_st32(trow + L::DPT + cb, hi);
        tmem_st32(trow + L::DSL + cb, lo);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(B_(D_READY0 + s));
      }
    }
    if (ok && n_it > 0) {
      const uint32_t last = (uint32_t)((n_it - 1) & 1);
      ok = role_wait(B_(VA_DONE), last, a.error, abort);
      if (ok) ok = role_wait(B_(KB_DONE), last, a.error, abort);
    }
    ok = __all_sync(0xffffffffu, ok);
    // warps 0-3 stage the raw dK rows, warps 4-7 the dV rows, in the free
    // operand buffers; the scale, the RoPE backward rotation (dK) and the
    // hi/lo split are applied while the rows are written out (coalesced)
    const uint32_t stage = base + (uint32_t)(khalf * 128 * (DH + 4) * 4);
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < DH / 32; c++) {
        float v[32];
        if (n_it > 0) {
          tmem_ld32(trow + (khalf == 0 ? L::DK : L::DV) + 32 * c, v);
          if (crow != nullptr) {  // plus the earlier chunks
            const float4* src = reinterpret_cast<const float4*>(crow + 32 * c);
#pragma unroll
            for (int u = 0; u < 8; u++) {
              const float4 y = src[u];
              v[4 * u] += y.x; v[4 * u + 1] += y.y; v[4 * u + 2] += y.z; v[4 * u + 3] += y.w;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = 0.0f;
        }
        stage_row32(stage, DH, row, 32 * c, v, 0, 32);
      }
    }
    named_sync(1, SOFT);
    // column-sum scratch behind the two staged tiles (one per output)
    const uint32_t red = base + (uint32_t)(2 * 128 * (DH + 4) * 4);
    float amax_k = 0.0f, amax_v = 0.0f;
    if (ok) {
      const bool split = dk.lo != nullptr && dv.lo != nullptr;
      const int rows = min(BK, p.Tk - k0);
      const int64_t ko = b * dk.sb + hkv * dk.sh + (int64_t)k0 * dk.st;
      const float4 sk = store_rows_split(
          base, DH, rows, dk.ptr, split ? dk.lo : nullptr, ko, dk.st, tid, SOFT,
          [&](int r, int c4, float4& v) {
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

// ---- dQ ----------------------------------------------------------------------------------

constexpr int QM = 128;  // queries per CTA (TMEM lanes)
constexpr int KN = 64;   // keys per block

template <int DH>
struct QLayout {
  static constexpr int KT = KN * DH * 4;  // [KN, DH] tile: DH/32 chunks of KN rows x 128 B
  static constexpr int RT = QM * DH * 4;  // [QM, DH] row tile
  // Q lo and dO lo rows stay in shared memory (A operands of the lo passes);
  // two stages of K-major K hi/lo, V hi/lo; one buffer of MN-major K hi/lo
  // (B of dQ, refilled once both dQ chains of the previous block are done)
  static constexpr int QL = 0, GL = RT, STAGE0 = 2 * RT;
  static constexpr int STAGE = 4 * KT;
  static constexpr int MN = STAGE0 + 2 * STAGE;
  static constexpr int KPOS = MN + 2 * KT;  // [2][KN] key positions
  static constexpr int BARS = KPOS + 2 * KN * 8;
  static constexpr int SMEM = BARS + 256 + 1024;
  // before the loop the Q hi and dO hi row tiles pass through stage 1
  static_assert(2 * RT <= STAGE, "row tiles in one stage");
  // TMEM: Q hi, dO hi (A operands); two slots of S, dP (dS hi over S, dS lo
  // over dP); dQ in two accumulators (one per chain), summed at the end
  static constexpr uint32_t QH = 0, GH = DH, SL0 = 2 * DH, SLOT = 2 * KN, DQA = SL0 + 2 * SLOT,
                            DQB = DQA + DH;
  static constexpr uint32_t COLS = 512;
  static_assert(DQB + DH <= COLS, "TMEM columns");
  static_assert(SMEM <= 232448, "shared memory");
};

// MASKED: the instance for calls with a boolean mask; the other one drops the
// mask code (smaller unrolled loops).
template <int DH, bool MASKED, bool THREE>
__global__ void __launch_bounds__(THREADS, 1)
attn_bwd_q_tc_kernel(const __grid_constant__ CUtensorMap qh_map,
                     const __grid_constant__ CUtensorMap ql_map,
                     const __grid_constant__ CUtensorMap gh_map,
                     const __grid_constant__ CUtensorMap gl_map,
                     const __grid_constant__ CUtensorMap kkh_map,
                     const __grid_constant__ CUtensorMap kkl_map,
                     const __grid_constant__ CUtensorMap vkh_map,
                     const __grid_constant__ CUtensorMap vkl_map,
                     const __grid_constant__ CUtensorMap kmh_map,
                     const __grid_constant__ CUtensorMap kml_map, AttnParams p, AttnOut dq,
                     TcBwdArgs a) {
  if constexpr (!MASKED) p.mask = nullptr;
  using L = QLayout<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  int64_t* kpos_s = reinterpret_cast<int64_t*>(smem + L::KPOS);  // [2][KN]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  // per-slot barriers come in pairs (slot 0, slot 1); a slot serves every
  // other block, so block j waits phase (j >> 1) & 1 of slot j & 1
  enum {
    FULL0, FULL1, EMPTY0, EMPTY1, SA0, SA1, SB0, SB1, DS0, DS1, QA0, QA1, QB0, QB1, KP0, KP1,
    MN_FULL, MN_EMPTY, ROWS_HI, ROWS_LO, NBARS
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
  if (tid == 0) {
    for (int i = 0; i < NBARS; i++) {
      const uint32_t n = (i == DS0 || i == DS1)                      ? SOFT
                         : (i == KP0 || i == KP1)                    ? 32
                         : (i == EMPTY0 || i == EMPTY1 || i == MN_EMPTY) ? 2
                                                                     : 1;
      mbar_init(B_(i), n);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
    // Q lo / dO lo rows to their resident buffers; Q hi / dO hi rows through
    // stage 1 on their way to TMEM (stage 0 receives the first block meanwhile)
    const int r = (int)(((int64_t)b * p.Hq + hq) * p.Tq + q0);
    mbar_expect_tx(B_(ROWS_LO), 2 * L::RT);
    mbar_expect_tx(B_(ROWS_HI), 2 * L::RT);
    const uint32_t hs = base + L::STAGE0 + L::STAGE;
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * QM * 128u;
      tma_load_2d(base + L::QL + o, &ql_map, B_(ROWS_LO), 32 * c, r);
      tma_load_2d(base + L::GL + o, &gl_map, B_(ROWS_LO), 32 * c, r);
      tma_load_2d(hs + o, &qh_map, B_(ROWS_HI), 32 * c, r);
      tma_load_2d(hs + L::RT + o, &gh_map, B_(ROWS_HI), 32 * c, r);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const int64_t kv_row0 = ((int64_t)b * p.Hkv + hkv) * p.Tk;
  auto load_kmajor = [&](int j) {  // K hi/lo, V hi/lo of block j into stage j & 1
    const uint32_t bar = B_(FULL0 + (j & 1)), dst = base + L::STAGE0 + (j & 1) * L::STAGE;
    const int r = (int)(kv_row0 + (int64_t)j * KN);
    mbar_expect_tx(bar, L::STAGE);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * KN * 128u;
      tma_load_2d(dst + o, &kkh_map, bar, 32 * c, r);
      tma_load_2d(dst + L::KT + o, &kkl_map, bar, 32 * c, r);
      tma_load_2d(dst + 2 * L::KT + o, &vkh_map, bar, 32 * c, r);
      tma_load_2d(dst + 3 * L::KT + o, &vkl_map, bar, 32 * c, r);
    }
  };
  auto load_mn = [&](int j) {  // MN-major K hi/lo of block j
    const uint32_t bar = B_(MN_FULL), dst = base + L::MN;
    const int r = (int)(kv_row0 + (int64_t)j * KN);
    mbar_expect_tx(bar, 2 * L::KT);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * KN * 128u;
      tma_load_2d(dst + o, &kmh_map, bar, 32 * c, r);
      tma_load_2d(dst + L::KT + o, &kml_map, bar, 32 * c, r);
    }
  };
  // Q hi and dO hi rows -> TMEM (warps 0-3 Q, 4-7 dO), while the loader
  // issues block 0
  if (warp < 8) {
    const bool ok = mbar_wait(B_(ROWS_HI), 0u, a.error);
    if (!ok) *abort = 1;
    if (__all_sync(0xffffffffu, ok)) {
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
      tile_row_to_tmem<DH>(base + L::STAGE0 + L::STAGE + (uint32_t)khalf * L::RT, row, trow,
                           khalf == 0 ? L::QH : L::GH);
      tmem_wait_st();
    }
  } else if (warp == LOADER && lane == 0 && nkb > 0) {
    load_kmajor(0);
    load_mn(0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == LOADER) {
    // ---- producer: K-major stages one block ahead of the MN-major buffer,
    // key positions by the lanes
    int nk = nkb > 0 ? 1 : 0, nm = nkb > 0 ? 1 : 0;  // blocks issued (lane 0)
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
    for (int j = 0; ok && j < nkb; j++) {
      const int jn = j + 1;
      if (jn < nkb) {
        // stage jn & 1 is free once S and dP of block jn - 2 completed
        if (lane == 0) {
          if (jn >= 2) ok = role_wait(B_(EMPTY0 + (jn & 1)), (uint32_t)(((jn >> 1) - 1) & 1), a.error, abort);
          if (ok) { load_kmajor(jn); nk++; }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        // position slot jn & 1 is free once block jn - 2's gradients are done
        if (ok && jn >= 2) ok = role_wait(B_(DS0 + (jn & 1)), (uint32_t)(((jn >> 1) - 1) & 1), a.error, abort);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) fill_kpos(jn);
      }
      // the MN-major buffer takes block j once both dQ chains of j - 1 are done
      if (ok && j >= 1 && lane == 0) {
        ok = role_wait(B_(MN_EMPTY), (uint32_t)((j - 1) & 1), a.error, abort);
        if (ok) { load_mn(j); nm++; }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {  // every copy has landed before the CTA releases its memory
      mbar_wait(B_(ROWS_LO), 0u, a.error);
      for (int j = nk - 2 < 0 ? 0 : nk - 2; j < nk; j++)
        mbar_wait(B_(FULL0 + (j & 1)), (uint32_t)((j >> 1) & 1), a.error);
      if (nm > 0) mbar_wait(B_(MN_FULL), (uint32_t)((nm - 1) & 1), a.error);
    }
  } else if (warp == MMA_A || warp == MMA_B) {
    // ---- MMA chains.  A: S = Q K^T, dQa += dS_hi K.  B: dP = dO V^T, dQb += dS_lo K_hi.
    // Issue order S(0), S(1), dQ(0), S(2), dQ(1), ...: the score MMAs of a
    // block run while the SM turns the previous block's scores into dS.
    const bool is_a = warp == MMA_A;
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc_s = idesc_tf32_m128(KN, 0);
      constexpr uint32_t idesc_q = idesc_tf32_m128(DH, 1);
      const uint32_t xh = tmem + (is_a ? L::QH : L::GH);
      const uint64_t xlo = kmajor_desc(base + (is_a ? L::QL : L::GL), QM, 0);
      const uint32_t col = is_a ? 0u : (uint32_t)KN;  // S or dP columns of a slot
      const uint32_t dqd = tmem + (is_a ? L::DQA : L::DQB);
      const int sdone = is_a ? SA0 : SB0, qdone = is_a ? QA0 : QB0;
      int s_issued = 0, q_issued = 0;
      bool ok = role_wait(B_(ROWS_LO), 0u, a.error, abort);
      auto issue_dq = [&](int i) {
        const int s = i & 1;
        const uint32_t par = (uint32_t)((i >> 1) & 1);
        ok = role_wait(B_(DS0 + s), par, a.error, abort);
        if (ok) ok = role_wait(B_(MN_FULL), (uint32_t)(i & 1), a.error, abort);
        if (!ok) return;
        tc_fence_after();
        const uint32_t sd = tmem + L::SL0 + (uint32_t)s * L::SLOT + col;
        const uint64_t kmh = mnmajor_desc(base + L::MN, KN, 0);
        const uint64_t kml = mnmajor_desc(base + L::MN + L::KT, KN, 0);
#pragma unroll
        for (int k = 0; k < KN / 8; k++) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          // one product (dS hi K hi, chain A) without THREE: chain B's
          // dQb accumulator stays unused
          if (THREE || is_a) umma_tf32_ts(dqd, sd + 8 * k, mslice(kmh, k), idesc_q, acc);
          if (THREE && is_a) umma_tf32_ts(dqd, sd + 8 * k, mslice(kml, k), idesc_q, 1u);
        }
        umma_commit(B_(qdone + s));
        umma_commit(B_(MN_EMPTY));
        q_issued++;
      };
      for (int j = 0; ok && j < nkb; j++) {
        const int s = j & 1;
        ok = role_wait(B_(FULL0 + s), (uint32_t)((j >> 1) & 1), a.error, abort);
        // the slot's columns are free once the dQ MMAs of block j - 2 read them
        if (ok && j >= 2) ok = role_wait(B_(qdone + s), (uint32_t)(((j >> 1) - 1) & 1), a.error, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t stg = base + L::STAGE0 + (uint32_t)s * L::STAGE;
        const uint64_t bh = kmajor_desc(stg + (is_a ? 0 : 2 * L::KT), KN, 0);
        const uint64_t bl = kmajor_desc(stg + (is_a ? L::KT : 3 * L::KT), KN, 0);
        const uint32_t sd = tmem + L::SL0 + (uint32_t)s * L::SLOT + col;
#pragma unroll
        for (int k = 0; k < DH / 8; k++) {
          const uint32_t acc = k > 0 ? 1u : 0u;
          umma_tf32_ts(sd, xh + 8 * k, kslice<KN>(bh, k), idesc_s, acc);
          if (THREE) {
            umma_tf32_ts(sd, xh + 8 * k, kslice<KN>(bl, k), idesc_s, 1u);
            umma_tf32(sd, kslice<QM>(xlo, k), kslice<KN>(bh, k), idesc_s, 1u);
          }
        }
        umma_commit(B_(sdone + s));
        umma_commit(B_(EMPTY0 + s));
        s_issued++;
        if (j >= 1) issue_dq(j - 1);
      }
      if (ok) issue_dq(nkb - 1);
      // committed MMAs finish before TMEM and shared memory are released
      if (s_issued > 0) {
        const int i = s_issued - 1;
        mbar_wait(B_(sdone + (i & 1)), (uint32_t)((i >> 1) & 1), a.error);
      }
      if (q_issued > 0) {
        const int i = q_issued - 1;
        mbar_wait(B_(qdone + (i & 1)), (uint32_t)((i >> 1) & 1), a.error);
      }
    }
  } else {
    // ---- dS = P (dP - delta), P = 2^(S scale log2(e) - lse2)
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
    const float lse_row = valid_q ? a.lse2[ri] : INFINITY;
    const float dlt_row = valid_q ? a.delta[ri] : 0.0f;
    const int64_t qpos_row = valid_q ? p.qpos[(int64_t)b * p.Tq + tq] : INT64_MIN;
    const float c2 = p.scale * kLog2e;
    const int cb = 32 * khalf;
    bool ok = true;
    for (int j = 0; ok && j < nkb; j++) {
      const int s = j & 1;
      const uint32_t spar = (uint32_t)((j >> 1) & 1);
      const bool full_block = j < full_kb;
      uint8_t keep[32];
      if (!full_block && p.mask != nullptr) {  // clamped indices stay in bounds
        const int64_t mrow = ((int64_t)b * p.Tq + min(tq, p.Tq - 1)) * p.Tk;
#pragma unroll
        for (int i = 0; i < 32; i++) keep[i] = p.mask[mrow + min(j * KN + cb + i, p.Tk - 1)];
      }
      ok = role_wait(B_(KP0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SA0 + s), spar, a.error, abort);
      if (ok) ok = role_wait(B_(SB0 + s), spar, a.error, abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // keys of the block this query sees: those whose position does not exceed its own
      const int seen = full_block ? KN : count_below(kpos_s + s * KN, KN, qpos_row + 1) - cb;
      const uint32_t slot = trow + L::SL0 + (uint32_t)s * L::SLOT;
      float sv[32], dp[32];
      tmem_ld32(slot + cb, sv);
      tmem_ld32(slot + KN + cb, dp);
#pragma unroll
      for (int i = 0; i < 32; i++) {
        bool adm = full_block;
        if (!full_block) {
          adm = i < seen;
          if (p.mask != nullptr) adm = adm && keep[i] != 0;
        }
        const float pv = adm ? ex2(fmaf(sv[i], c2, -lse_row)) : 0.0f;
        const float ds = pv * (dp[i] - dlt_row);
        sv[i] = tf32_hi(ds);
        dp[i] = ds - sv[i];
      }
      tmem_st32(slot + cb, sv);
      tmem_st32(slot + KN + cb, dp);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(B_(DS0 + s));
    }
    if (ok && nkb > 0) {
      const int i = nkb - 1;
      const uint32_t last = (uint32_t)((i >> 1) & 1);
      ok = role_wait(B_(QA0 + (i & 1)), last, a.error, abort);
      if (ok) ok = role_wait(B_(QB0 + (i & 1)), last, a.error, abort);
    }
    ok = __all_sync(0xffffffffu, ok);
    auto load_dq = [&](int col, float (&v)[32]) {
      if (nkb > 0) {
        tmem_ld32(trow + L::DQA + col, v);
        if (THREE) {
          float w[32];
          tmem_ld32(trow + L::DQB + col, w);
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = v[i] + w[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0.0f;
      }
    };
    // raw dQ rows staged in the free K/V stages; the scale, the RoPE
    // backward rotation and the hi/lo split are applied while the rows are
    // written out (coalesced)
    if (ok) {
      tc_fence_after();
      if constexpr (DH >= 64) {
#pragma unroll
        for (int c = 0; c < DH / 64; c++) {
          const int col = khalf * (DH / 2) + 32 * c;
          float v[32];
          load_dq(col, v);
          stage_row32(base, DH, row, col, v, 0, 32);
        }
      } else {
        float v[32];
        load_dq(0, v);
        if (khalf == 0) stage_row32(base, DH, row, 0, v, 0, 16);
        else stage_row32(base, DH, row, 16, v, 16, 16);
      }
    }
    named_sync(1, SOFT);
    // column-sum scratch behind the staged tile
    const uint32_t red = base + (uint32_t)(128 * (DH + 4) * 4);
    float amax = 0.0f;
    if (ok) {
      const int64_t qo = b * dq.sb + hq * dq.sh + (int64_t)q0 * dq.st;
      const float4 sq = store_rows_split(
          base, DH, min(QM, p.Tq - q0), dq.ptr, dq.lo, qo, dq.st, tid, SOFT,
          [&](int r, int c4, float4& v) {
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
bool launch_bwd_tc(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                   const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                   AttnOut dk, AttnOut dv, cudaStream_t stream) {
  const AttnWs w = attn_ws(p);
  const int64_t qrows = (int64_t)p.B * p.Hq * p.Tq, krows = (int64_t)p.B * p.Hkv * p.Tk;
  if (qrows >= ((int64_t)1 << 31) || krows >= ((int64_t)1 << 31)) return false;
  constexpr auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  constexpr auto SW32 = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  CUtensorMap kh, vh, kl, vl, qkh, qkl, gkh, gkl, qmh, qml, gmh, gml;
  CUtensorMap qh128, ql128, gh128, gl128, kkh, kkl, vkh, vkl, kmh, kml;
  bool built = make_map(&kh, w.kh, DH, krows, DH, BK, SW) && make_map(&vh, w.vh, DH, krows, DH, BK, SW) &&
               make_map(&kl, w.kl, DH, krows, DH, BK, SW) && make_map(&vl, w.vl, DH, krows, DH, BK, SW) &&
               make_map(&qh128, w.qh, DH, qrows, DH, QM, SW) && make_map(&ql128, w.ql, DH, qrows, DH, QM, SW) &&
               make_map(&gh128, w.doh, DH, qrows, DH, QM, SW) && make_map(&gl128, w.dol, DH, qrows, DH, QM, SW) &&
               make_map(&qkh, w.qh, DH, qrows, DH, BQ, SW) && make_map(&qkl, w.ql, DH, qrows, DH, BQ, SW) &&
               make_map(&gkh, w.doh, DH, qrows, DH, BQ, SW) && make_map(&gkl, w.dol, DH, qrows, DH, BQ, SW) &&
               make_map(&qmh, w.qh, DH, qrows, DH, BQ, SW32) && make_map(&qml, w.ql, DH, qrows, DH, BQ, SW32) &&
               make_map(&gmh, w.doh, DH, qrows, DH, BQ, SW32) && make_map(&gml, w.dol, DH, qrows, DH, BQ, SW32) &&
               make_map(&kkh, w.kh, DH, krows, DH, KN, SW) && make_map(&kkl, w.kl, DH, krows, DH, KN, SW) &&
               make_map(&vkh, w.vh, DH, krows, DH, KN, SW) && make_map(&vkl, w.vl, DH, krows, DH, KN, SW) &&
               make_map(&kmh, w.kh, DH, krows, DH, KN, SW32) && make_map(&kml, w.kl, DH, krows, DH, KN, SW32);
  if (!built) return false;
  if (!p.ws_ready) attention_prepare_qkv(p, w, stream);
  if (!p.grad_ready) {
    attn_bwd_prepare_kernel<<<(unsigned)((qrows + 7) / 8), 256, 0, stream>>>(
        p, o, o_lo, dout, row_max, row_sum, delta, w.lse2, w.doh, w.dol);
    count_launch();
  }
  cudaMemsetAsync(w.slot_flags, 0, (size_t)w.chunk_slots * sizeof(int), stream);
  TcBwdArgs a{w.kh,    w.vh,    w.qh,     w.ql,           w.doh,        w.dol,
              w.lse2,  delta,   device_error_word(),       w.chunks,     w.slot_flags,
              w.chunk_slots};
  dim3 g1((p.Tk + BK - 1) / BK, p.Hkv, p.B);  // THREADS: 8 probability warps, MMA, loads
  dim3 g2((p.Tq + QM - 1) / QM, p.Hq, p.B);
  // instances: with / without the mask code, three products / one
  auto go = [&](auto masked, auto three) {
    constexpr bool M = decltype(masked)::value, T3 = decltype(three)::value;
    cudaFuncSetAttribute(attn_bwd_kv_tc_kernel<DH, M, T3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, KvLayout<DH>::SMEM);
    cudaFuncSetAttribute(attn_bwd_q_tc_kernel<DH, M, T3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, QLayout<DH>::SMEM);
    attn_bwd_kv_tc_kernel<DH, M, T3><<<g1, THREADS, KvLayout<DH>::SMEM, stream>>>(
        kh, vh, kl, vl, qkh, qkl, gkh, gkl, qmh, qml, gmh, gml, p, dk, dv, a);
    attn_bwd_q_tc_kernel<DH, M, T3><<<g2, THREADS, QLayout<DH>::SMEM, stream>>>(
        qh128, ql128, gh128, gl128, kkh, kkl, vkh, vkl, kmh, kml, p, dq, a);
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

bool attention_backward_tc(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                           const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                           AttnOut dk, AttnOut dv, cudaStream_t stream) {
  if (p.ws == nullptr || encode_fn() == nullptr || p.Tq == 0 || p.Tk == 0) return false;
  if ((reinterpret_cast<uintptr_t>(p.ws) | reinterpret_cast<uintptr_t>(p.ws_grad)) & 15) return false;
  if (p.pairs16 || (attention_uses_pairs16(p) && !p.grad_ready))
    return attention_backward_f16(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
  switch (p.Dh) {
    case 32:
      return launch_bwd_tc<32>(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
    case 64:
      return launch_bwd_tc<64>(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
    default:
      return false;
  }
}

bool attention_grad_prep(const AttnParams& p, AttnTensor o, const float* o_lo,
                         const float* row_max, const float* row_sum, float* delta,
                         AttnGradPrep* out) {
  if (p.ws == nullptr) return false;
  if (p.pairs16 ? p.Dh != 64 && p.Dh != 128 : p.Dh != 32 && p.Dh != 64) return false;
  if (p.pairs16 && p.pair_exps == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(p.ws) | reinterpret_cast<uintptr_t>(p.ws_grad)) & 15) return false;
  // o as merged token-major rows [B*Tq, Hq*Dh]
  const int64_t ld = (int64_t)p.Hq * p.Dh;
  if (o.st != ld || o.sh != p.Dh || o.sb != (int64_t)p.Tq * ld) return false;
  const AttnWs w = attn_ws(p);
  AttnGradPrep g{};
  g.T = p.Tq; g.H = p.Hq; g.Dh = p.Dh;
  g.o = o.ptr; g.o_lo = o_lo;
  g.row_max = row_max; g.row_sum = row_sum;
  g.doh = w.doh; g.dol = w.dol; g.delta = delta; g.lse2 = w.lse2;
  if (p.pairs16) {
    g.g16h = w.g16h; g.g16l = w.g16l;
    g.g_exp = p.pair_exps + 3;
  }
  g.g_amax = p.pair_amax != nullptr ? p.pair_amax + 3 : nullptr;
  *out = g;
  return true;
}

void attention_prepare_grad_from(const float* dout, int64_t ld, int rows, const AttnGradPrep& g,
                                 cudaStream_t stream) {
  AttnParams p{};
  p.B = rows / g.T; p.Hq = g.H; p.Hkv = g.H; p.Tq = g.T; p.Tk = g.T; p.Dh = g.Dh;
  const int64_t ldo = (int64_t)g.H * g.Dh;
  const int64_t qrows = (int64_t)p.B * p.Hq * p.Tq;
  if (qrows == 0) return;
  attn_bwd_prepare_kernel<<<(unsigned)((qrows + 7) / 8), 256, 0, stream>>>(
      p, AttnTensor{g.o, (int64_t)g.T * ldo, g.Dh, ldo}, g.o_lo,
      AttnTensor{dout, (int64_t)g.T * ld, g.Dh, ld}, g.row_max, g.row_sum, g.delta, g.lse2, g.doh,
      g.dol);
  count_launch();
}

}  // namespace etb
