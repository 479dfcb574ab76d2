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
// is query row r.  8 warps: warp w handles rows 32*(w%4).. and key columns
// 32*(w/4).. of each 64-key block, so two threads share a row and exchange
// their row max / exp-sum through shared memory.
//   Q hi/lo  global -> registers -> TMEM (A operand of every S MMA)
//   K, V     TMA (128-byte swizzle; K 16-byte atoms, V 32-byte atoms),
//            hi and lo tiles, 3 stages (1 for Dh 128)
//   S        = Q K^T, tcgen05.mma kind::tf32 with A from TMEM, 3 passes;
//            for Dh <= 64 two S slots, so S of block j+1 is computed while
//            the SM runs the softmax of block j
//   softmax  base-2 online softmax in registers; P hi/lo -> TMEM (P_hi over S);
//            the O rows are rescaled in TMEM only when their max grows
//   O       += P V, A = P from TMEM, B = V (MN-major), 3 passes
// Key blocks entirely visible to every row of the tile skip the per-element
// admission test.  All mbarrier waits are bounded; a timeout is taken
// block-uniformly so the CTA always releases its TMEM.
#include "attention_tc.cuh"

namespace etb {

namespace {

constexpr int QM = 128;  // query rows per CTA
constexpr int KN = 64;   // keys per block
constexpr int THREADS = 256;

// Dh <= 64: S is double buffered in TMEM, so Q K^T of the next key block runs
// on the tensor cores while this block's softmax runs on the SM; Dh 128 has no
// TMEM room for that and runs the stages back to back.
template <int DH>
struct FwdLayout {
  static constexpr bool PIPE = DH <= 64;
  static constexpr int NBUF = PIPE ? 3 : 1;
  static constexpr int KTILE = KN * DH * 4;  // DH/32 chunks of KN rows x 128 B
  static constexpr int BUF = 4 * KTILE;      // K hi, K lo, V hi, V lo
  static constexpr int SMEM_BUF = NBUF * BUF;
  static constexpr int SMEM = SMEM_BUF + 1024 + 256 + 2 * 2 * QM * 4 + KN * 8;
  static constexpr uint32_t QH = 0, QL = DH, S0 = 2 * DH, NS = PIPE ? 2 : 1,
                            PL = S0 + NS * KN, O = PL + KN;
  static constexpr uint32_t COLS = (O + DH) <= 256 ? 256 : 512;
  static_assert(O + DH <= 512, "TMEM columns");
};

struct TcFwdArgs {
  const float *qh, *ql;  // head-major [B, Hq, Tq, Dh]
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

// ---- forward kernel --------------------------------------------------------------

template <int DH>
__global__ void __launch_bounds__(THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap kh_map, const __grid_constant__ CUtensorMap kl_map,
                   const __grid_constant__ CUtensorMap vh_map, const __grid_constant__ CUtensorMap vl_map,
                   AttnParams p, AttnOut o, float* __restrict__ row_max,
                   float* __restrict__ row_sum, TcFwdArgs a) {
  using L = FwdLayout<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::SMEM_BUF);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + L::NBUF + 2);
  float* xmax = reinterpret_cast<float*>(smem + L::SMEM_BUF + 256);  // [2][QM]
  float* xsum = xmax + 2 * QM;                                          // [2][QM]
  int64_t* kpos_s = reinterpret_cast<int64_t*>(xsum + 2 * QM);          // [KN]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, khalf = warp >> 2;
  const int row = quarter * 32 + lane;  // query row in the tile == TMEM lane
  const int q0 = blockIdx.x * QM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / (p.Hq / p.Hkv);
  const uint32_t full0 = smem_u32(bars), sbar = smem_u32(bars + L::NBUF),
                 pvbar = smem_u32(bars + L::NBUF + 1);
  if (tid == 0) {
    for (int i = 0; i < L::NBUF; i++) mbar_init(full0 + 8 * i, 1);
    mbar_init(sbar, 1);
    mbar_init(pvbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), L::COLS);
  const int tq = q0 + row;
  const bool valid_q = tq < p.Tq;

  // key blocks that can hold an admitted key, and the number of leading
  // blocks visible to every row of the tile (positions strictly increase)
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
      const int tk = kb * KN + tid;
      kpos_s[tid] = tk < p.Tk ? p.kpos[(int64_t)b * p.Tk + tk] : INT64_MAX;
    }
  };
  load_kpos(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);

  // producer / MMA state, meaningful in thread 0 only
  int next_load = 0, next_full = 0, s_issued = 0, pv_issued = 0;
  const int64_t kv_row0 = ((int64_t)b * p.Hkv + hkv) * p.Tk;
  auto buf_addr = [&](int kb) { return smem_u32(smem) + (uint32_t)((kb % L::NBUF) * L::BUF); };
  auto issue_load = [&]() {  // next_load into its buffer
    const int kb = next_load++;
    const uint32_t full = full0 + 8 * (kb % L::NBUF);
    mbar_expect_tx(full, 4 * L::KTILE);
    const int r = (int)(kv_row0 + (int64_t)kb * KN);
    const uint32_t base = buf_addr(kb);
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      tma_load_2d(base + c * KN * 128, &kh_map, full, 32 * c, r);
      tma_load_2d(base + L::KTILE + c * KN * 128, &kl_map, full, 32 * c, r);
      tma_load_2d(base + 2 * L::KTILE + c * KN * 128, &vh_map, full, 32 * c, r);
      tma_load_2d(base + 3 * L::KTILE + c * KN * 128, &vl_map, full, 32 * c, r);
    }
  };
  const uint32_t idesc_s = idesc_tf32_m128(KN, 0);
  const uint32_t idesc_o = idesc_tf32_m128(DH, 1);
  auto s_slot = [&](int kb) { return L::S0 + (uint32_t)(L::PIPE ? (kb & 1) * KN : 0); };
  auto issue_s = [&](int kb) -> bool {  // thread 0: S(kb) = Q K(kb)^T
    const int k = next_full++;
    if (!mbar_wait(full0 + 8 * (k % L::NBUF), (uint32_t)((k / L::NBUF) & 1), a.error))
      return false;
    tc_fence_after();
    const uint32_t khs = buf_addr(kb), kls = khs + L::KTILE;
    const uint32_t d = tmem + s_slot(kb);
#pragma unroll
    for (int j = 0; j < DH / 8; j++) {
      const uint64_t dh = kmajor_desc(khs, KN, j);
      const uint64_t dl = kmajor_desc(kls, KN, j);
      umma_tf32_ts(d, tmem + L::QH + 8 * j, dh, idesc_s, j > 0 ? 1u : 0u);
      umma_tf32_ts(d, tmem + L::QH + 8 * j, dl, idesc_s, 1u);
      umma_tf32_ts(d, tmem + L::QL + 8 * j, dh, idesc_s, 1u);
    }
    umma_commit(sbar);
    s_issued++;
    return true;
  };
  auto issue_pv = [&](int kb) {  // thread 0: O += P(kb) V(kb)
    tc_fence_after();
    const uint32_t vhs = buf_addr(kb) + 2 * L::KTILE, vls = vhs + L::KTILE;
    const uint32_t ph = tmem + s_slot(kb);
#pragma unroll
    for (int j = 0; j < KN / 8; j++) {
      const uint64_t dh = mnmajor_desc(vhs, KN, j);
      const uint64_t dl = mnmajor_desc(vls, KN, j);
      const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
      umma_tf32_ts(tmem + L::O, ph + 8 * j, dh, idesc_o, acc);
      umma_tf32_ts(tmem + L::O, ph + 8 * j, dl, idesc_o, 1u);
      umma_tf32_ts(tmem + L::O, tmem + L::PL + 8 * j, dh, idesc_o, 1u);
    }
    umma_commit(pvbar);
    pv_issued++;
  };

  bool ok = true;
  if (tid == 0) {
    while (next_load < L::NBUF && next_load < nkb) issue_load();
  }

  // ---- Q hi/lo rows -> TMEM (warps 0-3 hi, 4-7 lo)
  {
    const float* src = khalf == 0 ? a.qh : a.ql;
    const float* qrow = src + (((int64_t)b * p.Hq + hq) * p.Tq + tq) * DH;
#pragma unroll
    for (int c = 0; c < DH / 32; c++) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 x = valid_q ? *reinterpret_cast<const float4*>(qrow + c * 32 + i)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
      }
      tmem_st32(trow + (khalf == 0 ? L::QH : L::QL) + c * 32, v);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (L::PIPE && tid == 0 && nkb > 0) ok = issue_s(0);
  if (__syncthreads_or(!ok)) ok = false;

  const float c2 = p.scale * kLog2e;  // base-2 score scale
  float m = -INFINITY, l = 0.0f;      // base-2 running max, exp-sum
  const int64_t qpos_row = valid_q ? p.qpos[(int64_t)b * p.Tq + tq] : -1;
  for (int kb = 0; ok && kb < nkb; kb++) {
    const bool full_block = kb < full_kb;
    bool good = true;
    if (!L::PIPE && tid == 0) good = issue_s(kb);
    // S(kb) ready
    if (good) good = mbar_wait(sbar, (uint32_t)(kb & 1), a.error);
    good = __all_sync(0xffffffffu, good);  // tcgen05.ld/st are warp-collective
    float s[32];
    if (good) {
      tc_fence_after();
      tmem_ld32(trow + s_slot(kb) + 32 * khalf, s);
    }
    float bmax = -INFINITY;
    if (full_block) {
#pragma unroll
      for (int i = 0; i < 32; i++) {
        s[i] *= c2;
        bmax = fmaxf(bmax, s[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const int k = 32 * khalf + i;
        bool adm = valid_q && kpos_s[k] <= qpos_row;
        if (adm && p.mask != nullptr)
          adm = p.mask[((int64_t)b * p.Tq + tq) * p.Tk + kb * KN + k] != 0;
        s[i] = adm ? s[i] * c2 : -INFINITY;
        bmax = fmaxf(bmax, s[i]);
      }
    }
    xmax[khalf * QM + row] = bmax;
    if (__syncthreads_or(!good)) { ok = false; break; }
    bmax = fmaxf(bmax, xmax[(1 - khalf) * QM + row]);
    if (L::PIPE) {
      // PV(kb-1) done: its K/V buffer, P columns and O are free
      if (kb > 0) good = mbar_wait(pvbar, (uint32_t)((kb - 1) & 1), a.error);
      if (tid == 0 && good) {
        if (kb > 0 && next_load < nkb) issue_load();  // into the buffer of block kb-1
        if (kb + 1 < nkb) good = issue_s(kb + 1);
      }
      good = __all_sync(0xffffffffu, good);
      tc_fence_after();
    }
    const float m_new = fmaxf(m, bmax);
    float corr = 1.0f;
    if (m_new != -INFINITY) corr = (m == -INFINITY) ? 0.0f : ex2(m - m_new);
    float psum = 0.0f;
    float ph[32], pl[32];
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const float pv = (s[i] == -INFINITY) ? 0.0f : ex2(s[i] - m_new);
      psum += pv;
      ph[i] = tf32_round(pv);
      pl[i] = pv - ph[i];
    }
    xsum[khalf * QM + row] = psum;
    // rescale this thread's half of the O row (warp-uniform branch)
    if (good && kb > 0 && __any_sync(0xffffffffu, corr != 1.0f)) {
      if constexpr (DH >= 64) {
#pragma unroll
        for (int c = 0; c < DH / 64; c++) {
          float ov[32];
          const uint32_t col = L::O + (uint32_t)(khalf * (DH / 2) + c * 32);
          tmem_ld32(trow + col, ov);
#pragma unroll
          for (int i = 0; i < 32; i++) ov[i] *= corr;
          tmem_st32(trow + col, ov);
        }
      } else if (khalf == 0) {  // Dh 32: warps 0-3 rescale the whole row
        float ov[32];
        tmem_ld32(trow + L::O, ov);
#pragma unroll
        for (int i = 0; i < 32; i++) ov[i] *= corr;
        tmem_st32(trow + L::O, ov);
      }
    }
    if (good) {
      tmem_st32(trow + s_slot(kb) + 32 * khalf, ph);
      tmem_st32(trow + L::PL + 32 * khalf, pl);
      tmem_wait_st();
    }
    load_kpos(kb + 1);
    tc_fence_before();
    if (__syncthreads_or(!good)) { ok = false; break; }
    l = l * corr + (xsum[row] + xsum[QM + row]);
    m = m_new;
    if (tid == 0) issue_pv(kb);
    if (!L::PIPE) {
      good = mbar_wait(pvbar, (uint32_t)(kb & 1), a.error);
      if (tid == 0 && good && next_load < nkb) issue_load();
      if (__syncthreads_or(!good)) { ok = false; break; }
      tc_fence_after();
    }
  }
  if (L::PIPE && ok && nkb > 0) {
    if (__syncthreads_or(!mbar_wait(pvbar, (uint32_t)((nkb - 1) & 1), a.error))) ok = false;
    tc_fence_after();
  }

  // ---- epilogue: O / l (each thread writes its half of the row), statistics
  if (ok) {
    const bool empty = l == 0.0f;
    float* orow = o.ptr + b * o.sb + hq * o.sh + (int64_t)tq * o.st;
    if (valid_q && khalf == 0) {
      const int64_t ri = ((int64_t)b * p.Hq + hq) * p.Tq + tq;
      row_max[ri] = empty ? 0.0f : m * kLn2;
      row_sum[ri] = empty ? 0.0f : l;
    }
    if (nkb > 0) {
      if constexpr (DH >= 64) {
#pragma unroll
        for (int c = 0; c < DH / 64; c++) {
          float ov[32];
          tmem_ld32(trow + L::O + khalf * (DH / 2) + c * 32, ov);
          if (valid_q) {
            float* dst = orow + khalf * (DH / 2) + c * 32;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 w;
              w.x = empty ? 0.0f : rn_div(ov[i], l);
              w.y = empty ? 0.0f : rn_div(ov[i + 1], l);
              w.z = empty ? 0.0f : rn_div(ov[i + 2], l);
              w.w = empty ? 0.0f : rn_div(ov[i + 3], l);
              if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                *reinterpret_cast<float4*>(dst + i) = w;
              } else {
                dst[i] = w.x; dst[i + 1] = w.y; dst[i + 2] = w.z; dst[i + 3] = w.w;
              }
            }
          }
        }
      } else {
        float ov[32];
        tmem_ld32(trow + L::O, ov);
        if (valid_q) {
#pragma unroll
          for (int i = 0; i < 32; i++)
            if ((i >> 4) == khalf) orow[i] = empty ? 0.0f : rn_div(ov[i], l);
        }
      }
    } else if (valid_q) {
      for (int i = khalf * (DH / 2); i < (khalf + 1) * (DH / 2); i++) orow[i] = 0.0f;
    }
  } else if (tid == 0) {
    // a wait ran out: let every copy and MMA still in flight land (bounded)
    // before the shared memory and TMEM are released
    for (int k = next_full; k < next_load; k++)
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
bool launch_fwd_tc(const AttnParams& p, AttnOut o, float* m, float* l, cudaStream_t stream) {
  using L = FwdLayout<DH>;
  const AttnWs w = attn_ws(p);
  const int64_t krows = (int64_t)p.B * p.Hkv * p.Tk;
  if (krows >= ((int64_t)1 << 31)) return false;
  CUtensorMap mkh, mkl, mvh, mvl;
  if (!make_map(&mkh, w.kh, DH, krows, DH, KN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mkl, w.kl, DH, krows, DH, KN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mvh, w.vh, DH, krows, DH, KN, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !make_map(&mvl, w.vl, DH, krows, DH, KN, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return false;
  attention_prepare_qkv(p, w, stream);
  TcFwdArgs a{w.qh, w.ql, device_error_word()};
  cudaFuncSetAttribute(attn_fwd_tc_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       L::SMEM);
  dim3 grid((p.Tq + QM - 1) / QM, p.Hq, p.B);
  attn_fwd_tc_kernel<DH><<<grid, THREADS, L::SMEM, stream>>>(mkh, mkl, mvh, mvl, p, o, m, l, a);
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

size_t attention_workspace_floats(const AttnParams& p) {
  const size_t nq = (size_t)p.B * p.Hq * p.Tq * p.Dh, nk = (size_t)p.B * p.Hkv * p.Tk * p.Dh;
  const size_t rows = (size_t)p.B * p.Hq * p.Tq;
  return 4 * nq + 4 * nk + rows + 64;
}

bool attention_forward_tc(const AttnParams& p, AttnOut o, float* row_max, float* row_sum,
                          cudaStream_t stream) {
  if (p.ws == nullptr || encode_fn() == nullptr) return false;
  if (reinterpret_cast<uintptr_t>(p.ws) & 15) return false;
  switch (p.Dh) {
    case 32: return launch_fwd_tc<32>(p, o, row_max, row_sum, stream);
    case 64: return launch_fwd_tc<64>(p, o, row_max, row_sum, stream);
    case 128: return launch_fwd_tc<128>(p, o, row_max, row_sum, stream);
    default: return false;
  }
}

}  // namespace etb
