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
//
// A prepass writes the RoPE'd, TF32-split head-major Q/K/V (shared with the
// forward) and a second one dO hi/lo, delta and the base-2 log-sum-exp of
// every query row, so P = 2^(s scale log2(e) - lse2).  8 warps: warp w serves
// lanes 32*(w%4).. and columns 32*(w/4).. of each 64-wide block.  All
// mbarrier waits are bounded; a timeout is taken block-uniformly, in-flight
// copies and MMAs are waited for (bounded) and TMEM is always released.
#include "attention_tc.cuh"

namespace etb {

namespace {

constexpr int THREADS = 256;

// ---- prepass -----------------------------------------------------------------------

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
    const float l = row_sum[row];
    lse2[row] = l > 0.0f ? (row_max[row] + logf(l)) * kLog2e : INFINITY;
  }
}

struct TcBwdArgs {
  const float *kh, *vh;     // head-major K, V hi (dK/dV kernel)
  const float *qh, *ql;     // head-major Q hi/lo (dQ kernel)
  const float *doh, *dol;   // head-major dO hi/lo (dQ kernel)
  const float *lse2, *delta;
  int* error;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// Loads 32 floats of a row (zeros when the row is invalid) into TMEM.
__device__ __forceinline__ void row_to_tmem(uint32_t taddr, const float* src, bool valid) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 x = valid ? *reinterpret_cast<const float4*>(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
  }
  tmem_st32(taddr, v);
}

// Scales 2m columns of an accumulator row, applies the RoPE backward
// rotation to each (even, odd) pair when a table is given, and stores them.
template <int N>
__device__ __forceinline__ void store_grad_row(const float (&acc)[32], int first, float* dst,
                                               float scale, const float* ct, const float* st,
                                               int64_t trow, int col0) {
#pragma unroll
  for (int i = first; i < first + N; i += 2) {
    float x0 = rn_mul(acc[i], scale), x1 = rn_mul(acc[i + 1], scale);
    if (ct != nullptr) {
      const int64_t ti = trow + (col0 + i - first) / 2;
      const float c = ct[ti], s = st[ti];
      const float a = rn_mul(x0, c), bb = rn_mul(x1, s), cc = rn_mul(x0, s), dd = rn_mul(x1, c);
      x0 = rn_add(a, bb);
      x1 = rn_add(-cc, dd);
    }
    dst[i - first] = x0;
    dst[i - first + 1] = x1;
  }
}

// ---- dK / dV ---------------------------------------------------------------------------

constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 64;   // queries per step

template <int DH>
struct KvLayout {
  static constexpr int QT = BQ * DH * 4;      // [BQ, DH] tile: DH/32 chunks of BQ rows x 128 B
  static constexpr int KT = BK * DH * 4;      // [BK, DH] tile
  static constexpr int KL = 0, VL = KT;       // K lo, V lo (smem A operands)
  static constexpr int KSET = 2 * KT;         // Q hi, Q lo, dO hi, dO lo (K-major)
  static constexpr int MSET = KSET + 4 * QT;  // Q hi, Q lo, dO hi, dO lo (MN-major)
  static constexpr int SMEM_BUF = MSET + 4 * QT;
  static constexpr int SMEM = SMEM_BUF + 1024 + 256 + BQ * 16;
  static constexpr uint32_t KH = 0, VH = DH, DK = 2 * DH, DV = 3 * DH, ST = 4 * DH,
                            DPT = ST + BQ, PL = ST + 2 * BQ, DSL = ST + 3 * BQ;
  static constexpr uint32_t COLS = 512;
  static_assert(DSL + BQ <= COLS, "TMEM columns");
};

template <int DH>
__global__ void __launch_bounds__(THREADS, 1)
attn_bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap kl_map,
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
  using L = KvLayout<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::SMEM_BUF);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 5);
  float* lse_s = reinterpret_cast<float*>(smem + L::SMEM_BUF + 256);  // [BQ]
  float* dlt_s = lse_s + BQ;                                            // [BQ]
  int64_t* qp_s = reinterpret_cast<int64_t*>(dlt_s + BQ);               // [BQ]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, khalf = warp >> 2;
  const int row = quarter * 32 + lane;
  const int k0 = blockIdx.x * BK, hkv = blockIdx.y, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int tk = k0 + row;
  const bool valid_k = tk < p.Tk;
  const uint32_t lobar = smem_u32(bars), kfull = lobar + 8, mfull = lobar + 16, sbar = lobar + 24,
                 pvbar = lobar + 32;
  if (tid == 0) {
    for (int i = 0; i < 5; i++) mbar_init(lobar + 8 * i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  // query blocks that can see a key of this tile: from the first query whose
  // position reaches the first key's, for every query head of the group
  const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
  const int64_t* qp = p.qpos + (int64_t)b * p.Tq;
  int q_begin = 0;
  {
    const int64_t first = kp[k0];
    int lo = 0, hi = p.Tq;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (qp[mid] < first) lo = mid + 1; else hi = mid;
    }
    q_begin = lo;
  }
  const int jb = q_begin / BQ, nqb = (p.Tq + BQ - 1) / BQ;
  const int per_head = q_begin < p.Tq ? nqb - jb : 0;
  const int n_it = G * per_head;
  const int64_t kpos_row = valid_k ? kp[tk] : INT64_MAX;
  const bool keys_full = k0 + BK <= p.Tk;
  const int64_t kpos_last = kp[min(k0 + BK, p.Tk) - 1];
  auto q0_of = [&](int it) { return (jb + it % per_head) * BQ; };
  auto hq_of = [&](int it) { return hkv * G + it / per_head; };

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);

  // producer state (thread 0)
  bool t0ok = true;
  int k_loads = 0, k_waits = 0, m_loads = 0, m_waits = 0, s_issued = 0, pv_issued = 0;
  bool lo_loaded = false, lo_waited = false;
  const uint32_t base = smem_u32(smem);
  auto load_set = [&](int it, bool kset) {
    const uint32_t bar = kset ? kfull : mfull;
    mbar_expect_tx(bar, 4 * L::QT);
    const int r = (int)(((int64_t)b * p.Hq + hq_of(it)) * p.Tq + q0_of(it));
    const uint32_t dst = base + (kset ? L::KSET : L::MSET);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * BQ * 128u;
      tma_load_2d(dst + o, kset ? &qkh_map : &qmh_map, bar, 32 * c, r);
      tma_load_2d(dst + L::QT + o, kset ? &qkl_map : &qml_map, bar, 32 * c, r);
      tma_load_2d(dst + 2 * L::QT + o, kset ? &gkh_map : &gmh_map, bar, 32 * c, r);
      tma_load_2d(dst + 3 * L::QT + o, kset ? &gkl_map : &gml_map, bar, 32 * c, r);
    }
    if (kset) k_loads++; else m_loads++;
  };
  if (tid == 0 && n_it > 0) {
    mbar_expect_tx(lobar, 2 * L::KT);
    const int r = (int)(((int64_t)b * p.Hkv + hkv) * p.Tk + k0);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      tma_load_2d(base + L::KL + c * BK * 128, &kl_map, lobar, 32 * c, r);
      tma_load_2d(base + L::VL + c * BK * 128, &vl_map, lobar, 32 * c, r);
    }
    lo_loaded = true;
    load_set(0, true);
    load_set(0, false);
  }

  // K hi (warps 0-3) and V hi (warps 4-7) rows -> TMEM
  {
    const float* src = (khalf == 0 ? a.kh : a.vh) + (((int64_t)b * p.Hkv + hkv) * p.Tk + tk) * DH;
#pragma unroll
    for (int c = 0; c < DH / 32; c++)
      row_to_tmem(trow + (khalf == 0 ? L::KH : L::VH) + 32 * c, src + 32 * c, valid_k);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();

  const float c2 = p.scale * kLog2e;
  constexpr uint32_t idesc_s = idesc_tf32_m128(BQ, 0);
  constexpr uint32_t idesc_o = idesc_tf32_m128(DH, 1);
  bool ok = true;
  for (int it = 0; ok && it < n_it; it++) {
    const int q0 = q0_of(it), hq = hq_of(it);
    if (tid == 0 && t0ok) {
      if (!lo_waited) {
        t0ok = mbar_wait(lobar, 0u, a.error);
        lo_waited = true;
      }
      if (t0ok) t0ok = mbar_wait(kfull, (uint32_t)(k_waits & 1), a.error);
      k_waits++;
      if (t0ok) {
        tc_fence_after();
        const uint32_t qkh = base + L::KSET, qkl = qkh + L::QT, gkh = qkh + 2 * L::QT,
                       gkl = qkh + 3 * L::QT, klo = base + L::KL, vlo = base + L::VL;
#pragma unroll
        for (int j = 0; j < DH / 8; j++) {
          const uint32_t acc = j > 0 ? 1u : 0u;
          umma_tf32_ts(tmem + L::ST, tmem + L::KH + 8 * j, kmajor_desc(qkh, BQ, j), idesc_s, acc);
          umma_tf32_ts(tmem + L::ST, tmem + L::KH + 8 * j, kmajor_desc(qkl, BQ, j), idesc_s, 1u);
          umma_tf32(tmem + L::ST, kmajor_desc(klo, BK, j), kmajor_desc(qkh, BQ, j), idesc_s, 1u);
          umma_tf32_ts(tmem + L::DPT, tmem + L::VH + 8 * j, kmajor_desc(gkh, BQ, j), idesc_s, acc);
          umma_tf32_ts(tmem + L::DPT, tmem + L::VH + 8 * j, kmajor_desc(gkl, BQ, j), idesc_s, 1u);
          umma_tf32(tmem + L::DPT, kmajor_desc(vlo, BK, j), kmajor_desc(gkh, BQ, j), idesc_s, 1u);
        }
        umma_commit(sbar);
        s_issued++;
      }
    }
    // statistics of this query block (their previous readers passed the
    // barrier that ended the last iteration)
    if (tid < BQ) {
      const int q = q0 + tid;
      const int64_t r = ((int64_t)b * p.Hq + hq) * p.Tq + q;
      lse_s[tid] = q < p.Tq ? a.lse2[r] : INFINITY;
      dlt_s[tid] = q < p.Tq ? a.delta[r] : 0.0f;
      qp_s[tid] = q < p.Tq ? qp[q] : INT64_MIN;
    }
    const bool full_block =
        p.mask == nullptr && keys_full && q0 + BQ <= p.Tq && qp[q0] >= kpos_last;
    bool good = mbar_wait(sbar, (uint32_t)(it & 1), a.error);
    good = __all_sync(0xffffffffu, good) && (tid != 0 || t0ok);
    if (__syncthreads_or(!good)) { ok = false; break; }
    tc_fence_after();
    if (tid == 0 && it + 1 < n_it) load_set(it + 1, true);  // S^T and dP^T consumed the K-major set
    float st[32], dpt[32];
    tmem_ld32(trow + L::ST + 32 * khalf, st);
    tmem_ld32(trow + L::DPT + 32 * khalf, dpt);
    float ph[32], pl[32], dh[32], dl[32];
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int c = 32 * khalf + i;
      bool adm = full_block;
      if (!full_block) {
        adm = kpos_row <= qp_s[c];
        if (adm && p.mask != nullptr)
          adm = p.mask[((int64_t)b * p.Tq + q0 + c) * p.Tk + tk] != 0;
      }
      const float pv = adm ? ex2(st[i] * c2 - lse_s[c]) : 0.0f;
      const float ds = pv * (dpt[i] - dlt_s[c]);
      ph[i] = tf32_round(pv);
      pl[i] = pv - ph[i];
      dh[i] = tf32_hi(ds);
      dl[i] = ds - dh[i];
    }
    tmem_st32(trow + L::ST + 32 * khalf, ph);
    tmem_st32(trow + L::PL + 32 * khalf, pl);
    tmem_st32(trow + L::DPT + 32 * khalf, dh);
    tmem_st32(trow + L::DSL + 32 * khalf, dl);
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && t0ok) {
      t0ok = mbar_wait(mfull, (uint32_t)(m_waits & 1), a.error);
      m_waits++;
      if (t0ok) {
        tc_fence_after();
        const uint32_t qmh = base + L::MSET, qml = qmh + L::QT, gmh = qmh + 2 * L::QT,
                       gml = qmh + 3 * L::QT;
#pragma unroll
        for (int j = 0; j < BQ / 8; j++) {
          const uint32_t acc = (it > 0 || j > 0) ? 1u : 0u;
          umma_tf32_ts(tmem + L::DV, tmem + L::ST + 8 * j, mnmajor_desc(gmh, BQ, j), idesc_o, acc);
          umma_tf32_ts(tmem + L::DV, tmem + L::ST + 8 * j, mnmajor_desc(gml, BQ, j), idesc_o, 1u);
          umma_tf32_ts(tmem + L::DV, tmem + L::PL + 8 * j, mnmajor_desc(gmh, BQ, j), idesc_o, 1u);
          umma_tf32_ts(tmem + L::DK, tmem + L::DPT + 8 * j, mnmajor_desc(qmh, BQ, j), idesc_o, acc);
          umma_tf32_ts(tmem + L::DK, tmem + L::DPT + 8 * j, mnmajor_desc(qml, BQ, j), idesc_o, 1u);
          umma_tf32_ts(tmem + L::DK, tmem + L::DSL + 8 * j, mnmajor_desc(qmh, BQ, j), idesc_o, 1u);
        }
        umma_commit(pvbar);
        pv_issued++;
        // S^T / dP^T of the next block overwrite what these MMAs read
        t0ok = mbar_wait(pvbar, (uint32_t)(it & 1), a.error);
        if (t0ok && it + 1 < n_it) load_set(it + 1, false);
      }
    }
  }
  if (ok && n_it > 0) {
    bool good = mbar_wait(pvbar, (uint32_t)((n_it - 1) & 1), a.error);
    good = good && (tid != 0 || t0ok);
    if (__syncthreads_or(!good)) ok = false;
    tc_fence_after();
  }

  if (ok) {
    // warps 0-3: dK (scale, RoPE backward); warps 4-7: dV
    const AttnOut& out = khalf == 0 ? dk : dv;
    float* orow = out.ptr + b * out.sb + hkv * out.sh + (int64_t)tk * out.st;
    const float* ct = khalf == 0 ? p.k_cos : nullptr;
    const float* sn = khalf == 0 ? p.k_sin : nullptr;
    const int64_t trw = (int64_t)(p.k_rope_batched ? b * p.Tk + tk : tk) * (DH / 2);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      float v[32];
      if (n_it > 0) {
        tmem_ld32(trow + (khalf == 0 ? L::DK : L::DV) + 32 * c, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0.0f;
      }
      if (valid_k)
        store_grad_row<32>(v, 0, orow + 32 * c, khalf == 0 ? p.scale : 1.0f, ct, sn, trw, 32 * c);
    }
  } else if (tid == 0) {
    if (lo_loaded && !lo_waited) mbar_wait(lobar, 0u, a.error);
    for (int k = k_waits; k < k_loads; k++) mbar_wait(kfull, (uint32_t)(k & 1), a.error);
    for (int k = m_waits; k < m_loads; k++) mbar_wait(mfull, (uint32_t)(k & 1), a.error);
    if (s_issued > 0) mbar_wait(sbar, (uint32_t)((s_issued - 1) & 1), a.error);
    if (pv_issued > 0) mbar_wait(pvbar, (uint32_t)((pv_issued - 1) & 1), a.error);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::COLS);
  }
}

// ---- dQ ----------------------------------------------------------------------------------

constexpr int QM = 128;  // queries per CTA
constexpr int KN = 64;   // keys per step

template <int DH>
struct QLayout {
  static constexpr int KT = KN * DH * 4;  // one [KN, DH] tile
  static constexpr int STAGE = 6 * KT;    // K hi/lo, V hi/lo (K-major), K hi/lo (MN-major)
  static constexpr int NBUF = 2;
  static constexpr int SMEM_BUF = NBUF * STAGE;
  static constexpr int SMEM = SMEM_BUF + 1024 + 256 + KN * 8;
  static constexpr uint32_t QH = 0, QL = DH, GH = 2 * DH, GL = 3 * DH, S = 4 * DH, DP = S + KN,
                            DQ = DP + KN;
  static constexpr uint32_t COLS = DQ + DH <= 256 ? 256 : 512;
  static_assert(DQ + DH <= 512, "TMEM columns");
};

template <int DH>
__global__ void __launch_bounds__(THREADS, 1)
attn_bwd_q_tc_kernel(const __grid_constant__ CUtensorMap kkh_map,
                     const __grid_constant__ CUtensorMap kkl_map,
                     const __grid_constant__ CUtensorMap vkh_map,
                     const __grid_constant__ CUtensorMap vkl_map,
                     const __grid_constant__ CUtensorMap kmh_map,
                     const __grid_constant__ CUtensorMap kml_map, AttnParams p, AttnOut dq,
                     TcBwdArgs a) {
  using L = QLayout<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::SMEM_BUF);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + L::NBUF + 2);
  int64_t* kpos_s = reinterpret_cast<int64_t*>(smem + L::SMEM_BUF + 256);  // [KN]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, khalf = warp >> 2;
  const int row = quarter * 32 + lane;
  const int q0 = blockIdx.x * QM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / (p.Hq / p.Hkv);
  const int tq = q0 + row;
  const bool valid_q = tq < p.Tq;
  const uint32_t full0 = smem_u32(bars), sbar = full0 + 8 * L::NBUF, pvbar = sbar + 8;
  if (tid == 0) {
    for (int i = 0; i < L::NBUF + 2; i++) mbar_init(full0 + 8 * i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);

  int nkb = 0, full_kb = 0;
  {
    const int qlast = min(q0 + QM, p.Tq) - 1;
    const int64_t qmax = p.qpos[(int64_t)b * p.Tq + qlast];
    const int64_t qmin = p.qpos[(int64_t)b * p.Tq + q0];
    const int64_t* kp = p.kpos + (int64_t)b * p.Tk;
    int lo = 0, hi = p.Tk;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (kp[mid] <= qmax) lo = mid + 1; else hi = mid;
    }
    nkb = (lo + KN - 1) / KN;
    int lo2 = 0, hi2 = lo;
    while (lo2 < hi2) {
      const int mid = (lo2 + hi2) >> 1;
      if (kp[mid] <= qmin) lo2 = mid + 1; else hi2 = mid;
    }
    full_kb = (p.mask == nullptr && q0 + QM <= p.Tq) ? lo2 / KN : 0;
  }
  auto load_kpos = [&](int kb) {
    if (kb < nkb && kb >= full_kb && tid < KN) {
      const int t = kb * KN + tid;
      kpos_s[tid] = t < p.Tk ? p.kpos[(int64_t)b * p.Tk + t] : INT64_MAX;
    }
  };
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);

  bool t0ok = true;
  int next_load = 0, waits = 0, s_issued = 0, pv_issued = 0;
  const uint32_t base = smem_u32(smem);
  const int64_t kv_row0 = ((int64_t)b * p.Hkv + hkv) * p.Tk;
  auto stage_addr = [&](int kb) { return base + (uint32_t)((kb % L::NBUF) * L::STAGE); };
  auto issue_load = [&]() {
    const int kb = next_load++;
    const uint32_t bar = full0 + 8 * (kb % L::NBUF);
    mbar_expect_tx(bar, L::STAGE);
    const int r = (int)(kv_row0 + (int64_t)kb * KN);
    const uint32_t dst = stage_addr(kb);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      const uint32_t o = (uint32_t)c * KN * 128u;
      tma_load_2d(dst + o, &kkh_map, bar, 32 * c, r);
      tma_load_2d(dst + L::KT + o, &kkl_map, bar, 32 * c, r);
      tma_load_2d(dst + 2 * L::KT + o, &vkh_map, bar, 32 * c, r);
      tma_load_2d(dst + 3 * L::KT + o, &vkl_map, bar, 32 * c, r);
      tma_load_2d(dst + 4 * L::KT + o, &kmh_map, bar, 32 * c, r);
      tma_load_2d(dst + 5 * L::KT + o, &kml_map, bar, 32 * c, r);
    }
  };
  if (tid == 0)
    while (next_load < L::NBUF && next_load < nkb) issue_load();

  // Q hi/lo and dO hi/lo rows -> TMEM
  {
    const int64_t off = (((int64_t)b * p.Hq + hq) * p.Tq + tq) * DH;
    const float* s1 = (khalf == 0 ? a.qh : a.ql) + off;
    const float* s2 = (khalf == 0 ? a.doh : a.dol) + off;
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      row_to_tmem(trow + (khalf == 0 ? L::QH : L::QL) + 32 * c, s1 + 32 * c, valid_q);
      row_to_tmem(trow + (khalf == 0 ? L::GH : L::GL) + 32 * c, s2 + 32 * c, valid_q);
    }
    tmem_wait_st();
  }
  const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
  const float lse_row = valid_q ? a.lse2[ri] : INFINITY;
  const float dlt_row = valid_q ? a.delta[ri] : 0.0f;
  const int64_t qpos_row = valid_q ? p.qpos[(int64_t)b * p.Tq + tq] : -1;
  tc_fence_before();
  __syncthreads();

  const float c2 = p.scale * kLog2e;
  constexpr uint32_t idesc_s = idesc_tf32_m128(KN, 0);
  constexpr uint32_t idesc_q = idesc_tf32_m128(DH, 1);
  bool ok = true;
  for (int kb = 0; ok && kb < nkb; kb++) {
    const bool full_block = kb < full_kb;
    if (tid == 0 && t0ok) {
      const int k = waits++;
      t0ok = mbar_wait(full0 + 8 * (k % L::NBUF), (uint32_t)((k / L::NBUF) & 1), a.error);
      if (t0ok) {
        tc_fence_after();
        const uint32_t kkh = stage_addr(kb), kkl = kkh + L::KT, vkh = kkh + 2 * L::KT,
                       vkl = kkh + 3 * L::KT;
#pragma unroll
        for (int j = 0; j < DH / 8; j++) {
          const uint32_t acc = j > 0 ? 1u : 0u;
          umma_tf32_ts(tmem + L::S, tmem + L::QH + 8 * j, kmajor_desc(kkh, KN, j), idesc_s, acc);
          umma_tf32_ts(tmem + L::S, tmem + L::QH + 8 * j, kmajor_desc(kkl, KN, j), idesc_s, 1u);
          umma_tf32_ts(tmem + L::S, tmem + L::QL + 8 * j, kmajor_desc(kkh, KN, j), idesc_s, 1u);
          umma_tf32_ts(tmem + L::DP, tmem + L::GH + 8 * j, kmajor_desc(vkh, KN, j), idesc_s, acc);
          umma_tf32_ts(tmem + L::DP, tmem + L::GH + 8 * j, kmajor_desc(vkl, KN, j), idesc_s, 1u);
          umma_tf32_ts(tmem + L::DP, tmem + L::GL + 8 * j, kmajor_desc(vkh, KN, j), idesc_s, 1u);
        }
        umma_commit(sbar);
        s_issued++;
      }
    }
    load_kpos(kb);  // the previous block's readers passed the last barrier
    bool good = mbar_wait(sbar, (uint32_t)(kb & 1), a.error);
    good = __all_sync(0xffffffffu, good) && (tid != 0 || t0ok);
    if (__syncthreads_or(!good)) { ok = false; break; }
    tc_fence_after();
    float s[32], dp[32];
    tmem_ld32(trow + L::S + 32 * khalf, s);
    tmem_ld32(trow + L::DP + 32 * khalf, dp);
    float dh[32], dl[32];
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int k = 32 * khalf + i;
      bool adm = full_block;
      if (!full_block) {
        adm = valid_q && kpos_s[k] <= qpos_row;
        if (adm && p.mask != nullptr)
          adm = p.mask[((int64_t)b * p.Tq + tq) * p.Tk + kb * KN + k] != 0;
      }
      const float pv = adm ? ex2(s[i] * c2 - lse_row) : 0.0f;
      const float ds = pv * (dp[i] - dlt_row);
      dh[i] = tf32_hi(ds);
      dl[i] = ds - dh[i];
    }
    tmem_st32(trow + L::S + 32 * khalf, dh);
    tmem_st32(trow + L::DP + 32 * khalf, dl);
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && t0ok) {
      tc_fence_after();
      const uint32_t kmh = stage_addr(kb) + 4 * L::KT, kml = kmh + L::KT;
#pragma unroll
      for (int j = 0; j < KN / 8; j++) {
        const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
        umma_tf32_ts(tmem + L::DQ, tmem + L::S + 8 * j, mnmajor_desc(kmh, KN, j), idesc_q, acc);
        umma_tf32_ts(tmem + L::DQ, tmem + L::S + 8 * j, mnmajor_desc(kml, KN, j), idesc_q, 1u);
        umma_tf32_ts(tmem + L::DQ, tmem + L::DP + 8 * j, mnmajor_desc(kmh, KN, j), idesc_q, 1u);
      }
      umma_commit(pvbar);
      pv_issued++;
      // the next S / dP overwrite what these MMAs read; the stage is free after
      t0ok = mbar_wait(pvbar, (uint32_t)(kb & 1), a.error);
      if (t0ok && next_load < nkb) issue_load();
    }
  }
  if (ok && nkb > 0) {
    bool good = mbar_wait(pvbar, (uint32_t)((nkb - 1) & 1), a.error);
    good = good && (tid != 0 || t0ok);
    if (__syncthreads_or(!good)) ok = false;
    tc_fence_after();
  }

  if (ok) {
    float* orow = dq.ptr + b * dq.sb + hq * dq.sh + (int64_t)tq * dq.st;
    const int64_t trw = (int64_t)(p.q_rope_batched ? b * p.Tq + tq : tq) * (DH / 2);
    if constexpr (DH >= 64) {
#pragma unroll
      for (int c = 0; c < DH / 64; c++) {
        const int col = khalf * (DH / 2) + 32 * c;
        float v[32];
        if (nkb > 0) {
          tmem_ld32(trow + L::DQ + col, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = 0.0f;
        }
        if (valid_q) store_grad_row<32>(v, 0, orow + col, p.scale, p.q_cos, p.q_sin, trw, col);
      }
    } else {
      float v[32];
      if (nkb > 0) {
        tmem_ld32(trow + L::DQ, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0.0f;
      }
      if (valid_q) {
        if (khalf == 0) store_grad_row<16>(v, 0, orow, p.scale, p.q_cos, p.q_sin, trw, 0);
        else store_grad_row<16>(v, 16, orow + 16, p.scale, p.q_cos, p.q_sin, trw, 16);
      }
    }
  } else if (tid == 0) {
    for (int k = waits; k < next_load; k++)
      mbar_wait(full0 + 8 * (k % L::NBUF), (uint32_t)((k / L::NBUF) & 1), a.error);
    if (s_issued > 0) mbar_wait(sbar, (uint32_t)((s_issued - 1) & 1), a.error);
    if (pv_issued > 0) mbar_wait(pvbar, (uint32_t)((pv_issued - 1) & 1), a.error);
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
  CUtensorMap kl, vl, qkh, qkl, gkh, gkl, qmh, qml, gmh, gml;
  CUtensorMap kkh, kkl, vkh, vkl, kmh, kml;
  bool built = make_map(&kl, w.kl, DH, krows, DH, BK, SW) && make_map(&vl, w.vl, DH, krows, DH, BK, SW) &&
               make_map(&qkh, w.qh, DH, qrows, DH, BQ, SW) && make_map(&qkl, w.ql, DH, qrows, DH, BQ, SW) &&
               make_map(&gkh, w.doh, DH, qrows, DH, BQ, SW) && make_map(&gkl, w.dol, DH, qrows, DH, BQ, SW) &&
               make_map(&qmh, w.qh, DH, qrows, DH, BQ, SW32) && make_map(&qml, w.ql, DH, qrows, DH, BQ, SW32) &&
               make_map(&gmh, w.doh, DH, qrows, DH, BQ, SW32) && make_map(&gml, w.dol, DH, qrows, DH, BQ, SW32) &&
               make_map(&kkh, w.kh, DH, krows, DH, KN, SW) && make_map(&kkl, w.kl, DH, krows, DH, KN, SW) &&
               make_map(&vkh, w.vh, DH, krows, DH, KN, SW) && make_map(&vkl, w.vl, DH, krows, DH, KN, SW) &&
               make_map(&kmh, w.kh, DH, krows, DH, KN, SW32) && make_map(&kml, w.kl, DH, krows, DH, KN, SW32);
  if (!built) return false;
  attention_prepare_qkv(p, w, stream);
  attn_bwd_prepare_kernel<<<(unsigned)((qrows + 7) / 8), 256, 0, stream>>>(
      p, o, o_lo, dout, row_max, row_sum, delta, w.lse2, w.doh, w.dol);
  count_launch();
  TcBwdArgs a{w.kh, w.vh, w.qh, w.ql, w.doh, w.dol, w.lse2, delta, device_error_word()};
  cudaFuncSetAttribute(attn_bwd_kv_tc_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       KvLayout<DH>::SMEM);
  cudaFuncSetAttribute(attn_bwd_q_tc_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       QLayout<DH>::SMEM);
  dim3 g1((p.Tk + BK - 1) / BK, p.Hkv, p.B);
  attn_bwd_kv_tc_kernel<DH><<<g1, THREADS, KvLayout<DH>::SMEM, stream>>>(
      kl, vl, qkh, qkl, gkh, gkl, qmh, qml, gmh, gml, p, dk, dv, a);
  dim3 g2((p.Tq + QM - 1) / QM, p.Hq, p.B);
  attn_bwd_q_tc_kernel<DH><<<g2, THREADS, QLayout<DH>::SMEM, stream>>>(kkh, kkl, vkh, vkl, kmh,
                                                                        kml, p, dq, a);
  count_launch(2);
  return true;
}

}  // namespace

bool attention_backward_tc(const AttnParams& p, AttnTensor o, const float* o_lo, AttnTensor dout,
                           const float* row_max, const float* row_sum, float* delta, AttnOut dq,
                           AttnOut dk, AttnOut dv, cudaStream_t stream) {
  if (p.ws == nullptr || encode_fn() == nullptr || p.Tq == 0 || p.Tk == 0) return false;
  if (reinterpret_cast<uintptr_t>(p.ws) & 15) return false;
  switch (p.Dh) {
    case 32:
      return launch_bwd_tc<32>(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
    case 64:
      return launch_bwd_tc<64>(p, o, o_lo, dout, row_max, row_sum, delta, dq, dk, dv, stream);
    default:
      return false;
  }
}

}  // namespace etb
