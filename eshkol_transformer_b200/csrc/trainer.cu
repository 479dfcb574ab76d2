// Decoder-only LM training step on one B200 (and across ranks with NCCL).
//
// The composition follows the reference's fixed M3 schedule
// (native/m3_schedule.esk:3-52; roles in src/eshkol_transformer/m3t_transport.c:
// 516-563) with RoPE on Q/K instead of learned positions and biased linears:
//   forward   x0 = E[ids]; per layer h = LN1(x); qkv = h Wqkv^T + b;
//             o = attention(RoPE(q), RoPE(k), v); x' = x + o Wo^T + b;
//             h2 = LN2(x'); x'' = x' + GELU(h2 W1^T + b1) W2^T + b2;
//             logits = LN_f(x_L) E^T; loss = CE(logits, targets)
//   backward  the reverse schedule, with the tied embedding gradient summed
//             head first (m3t_transport.c:562);
//   update    AdamW over every tensor (o2_optimizer.c:1738-1756).
// The CE backward carries the 1/N token weight (N = global tokens) that the
// reference applies as the O2 normalisation weight; for N = 2^k that move is
// exact.  Activations live in HBM for the whole step (f32), laid out token-
// major [rows, features]; attention reads Q/K/V straight out of the fused
// [rows, 3d] QKV buffer and writes its output merged into [rows, d].  In the
// 3xTF32 mode every GEMM operand is kept as a (hi, lo) pair: producers' outputs
// are split once, weights after every update.
//
// Split-f16 mode (ET_B200_PRECISION_F16X3): the operand pairs are binary16
// (hi, lo) arrays of x 2^e with one power-of-two exponent e per operand
// tensor ("slot"), taken from the tensor's max |x| in the previous step so
// that it sits near 2^10, 64x below binary16's overflow (delayed scaling).
// Producers write the pairs and record the new max in the same pass.  The
// first step, and any step in which some operand reached the overflow, runs
// 3xTF32 instead (recording every slot's max); a step whose check fails is
// not applied (AdamW skips on a flag that the data-parallel reduction sums
// across ranks) and the host-synchronised entry points redo it in 3xTF32.
//
// Data parallelism: each rank runs its own batch; after a layer's backward its
// contiguous gradient slice is summed across ranks by ncclAllReduce on a side
// stream while the next layer's backward runs; AdamW waits for the last bucket.
#include <math.h>

#include <cmath>

#include <algorithm>
#include <string>
#include <vector>

#include "nccl_loader.cuh"
#include "ops.cuh"

using namespace etb;

namespace {

enum { kPerLayer = 12 };
// split-f16 operand slots of one layer
// (S_Q, S_K, S_V, S_DO: the attention's binary16 operand pairs, consecutive
// as AttnParams.pair_exps / pair_amax take them)
enum { S_H1 = 0, S_AO, S_H2, S_G, S_DXF, S_DU, S_DXA, S_DQKV, S_Q, S_K, S_V, S_DO,
       kSlotsPerLayer };
// a slot's max |x| 2^e lands in [2^(target-1), 2^target): 64x below
// binary16's overflow.  ET_B200_F16_SCALE_TARGET (2 .. 17) overrides it; 17
// puts every slot's max above 65,504, which exercises the overflow check and
// the 3xTF32 redo.
constexpr int kScaleTarget = 10;
// Step-void flag increment for an out-of-range token id or target; below it,
// the count of ranks whose split-f16 operands overflowed (exact in f32 for
// any world size below 256).
constexpr float kVoidIndex = 65536.0f;
enum {
  T_LN1G = 0, T_LN1B, T_WQKV, T_BQKV, T_WO, T_BO, T_LN2G, T_LN2B, T_W1, T_B1, T_W2, T_B2
};

// Profile classes reported by et_b200_lm_profile_read_v1.
enum {
  P_GEMM = 0, P_ATTN_FWD, P_ATTN_BWD, P_CE, P_ADAMW, P_NORM, P_ELEMENTWISE, P_EMBED,
  P_SPLIT, P_ALLREDUCE_WAIT, P_ADAMW_CHECK, P_COUNT
};

struct LayerActs {
  float *x = nullptr, *h1 = nullptr, *h1lo = nullptr, *mu1 = nullptr, *rs1 = nullptr;
  float *qkv = nullptr, *ao = nullptr, *aolo = nullptr, *am = nullptr, *al = nullptr;
  float *xmid = nullptr, *h2 = nullptr, *h2lo = nullptr, *mu2 = nullptr, *rs2 = nullptr;
  float *u = nullptr, *g = nullptr, *glo = nullptr;
  float* ao16 = nullptr;  // split-f16: binary16 hi then lo of the attention output
};

struct ProfileMark {
  int cls;
  double flop, bytes;
  cudaEvent_t start, stop;
};

}  // namespace

struct et_b200_lm {
  et_b200_lm_config_v1 cfg{};
  int device = 0;
  cudaStream_t stream = nullptr, comm = nullptr;
  int64_t L = 0, d = 0, H = 0, Dh = 0, F = 0, V = 0, T = 0, B = 0, R = 0;
  float ce_scale = 0, eps = 0, attn_scale = 0;
  int precision = 0;
  bool three = false;  // (hi, lo) operand pairs (3xTF32 or split-f16)
  int gprec = 0;       // contraction mode of the GEMMs without binary16 operands
  // split-f16: model mode, scales measured, this step's operand format, and
  // whether whi / wlo hold the weights' binary16 pair
  bool f16 = false, calibrated = false, step16 = false, w16_valid = false;
  int nslots = 0;
  int scale_target = kScaleTarget;
  int redone_steps = 0;       // split-f16 steps redone in 3xTF32 (host-synchronised calls)
  int* sexp = nullptr;        // per slot exponent e
  unsigned* samax = nullptr;  // per slot max |x| (f32 bits)
  float* dqkv16 = nullptr;    // binary16 hi then lo of dqkv
  // parameters (flat, tensor order as documented in et_b200.h)
  size_t P = 0;
  std::vector<size_t> off, sz;
  float *params = nullptr, *grads = nullptr, *m1 = nullptr, *m2 = nullptr;
  float *whi = nullptr, *wlo = nullptr;
  AdamwTensor* d_adam = nullptr;
  uint64_t* d_prefix = nullptr;
  uint64_t updates = 0;          // host copy of *d_completed at the last synchronisation
  uint64_t* d_completed = nullptr;  // applied AdamW updates (device counter)
  uint64_t skipped = 0;          // device-enqueued steps whose update was not applied
  // activations
  std::vector<LayerActs> layers;
  float *x_final = nullptr, *xf = nullptr, *xflo = nullptr, *muf = nullptr, *rsf = nullptr;
  float *logits = nullptr, *logits_lo = nullptr, *loss_rows = nullptr, *loss_mean = nullptr;
  // backward scratch
  float *dx = nullptr, *dxhi = nullptr, *dxlo = nullptr, *dtmp = nullptr, *dqkv = nullptr,
        *dqkvlo = nullptr, *du = nullptr, *dulo = nullptr, *delta = nullptr;
  float *ln_ws = nullptr, *col_ws = nullptr, *splitk_ws = nullptr, *epi_ws = nullptr;
  float* chunk_ws = nullptr;  // the f32-grade GEMMs' K-chunk running sums
  size_t chunk_ws_floats = 0;
  // per-128-row-tile column sums of dqkv from the attention backward (bqkv gradient)
  float* qkv_colpart = nullptr;
  int64_t qkv_colrows = 0;
  // attention: per-layer prepared Q/K/V (written by the forward, reused by
  // the backward) and one shared backward scratch
  std::vector<float*> attn_qkv_ws;
  std::vector<char> attn_prepared;
  float* attn_grad_ws = nullptr;
  size_t splitk_floats = 0;
  void* emb_scratch = nullptr;
  int64_t *ids = nullptr, *targets = nullptr, *pos = nullptr;
  // the loss mask of the steps (L3S masked objective; `masked` false = every
  // token counts), its numerator seed, and the power of two 2^-ceil(log2 N)
  // (N = global tokens) the seed carries
  uint8_t* loss_mask = nullptr;
  float* upstream = nullptr;
  bool masked = false;
  float mask_scale = 0;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  // [0] a token id or target of this step is out of range; [1] this step's
  // AdamW check bits (kAdamw*); [2] updates skipped since the last host read
  int* status = nullptr;
  std::vector<void*> allocations;
  // data parallel
  ncclComm_t nccl_comm = nullptr;
  int rank = 0, world = 1;
  bool dp = false;
  std::vector<cudaEvent_t> layer_done;
  cudaEvent_t tail_done = nullptr, comm_done = nullptr;
  // profiling
  bool profile = false;
  std::vector<ProfileMark> marks;
  size_t mark_used = 0;
  double prof[P_COUNT][4] = {};  // launches, ms, flop, bytes

  // weight operand t: f32, its TF32 pair, or (split-f16 steps) its binary16 pair
  const float* W(int t) const {
    if (step16) return reinterpret_cast<const float*>(reinterpret_cast<const uint16_t*>(whi) + off[t]);
    return (three ? whi : params) + off[t];
  }
  const float* Wlo(int t) const {
    if (step16) return reinterpret_cast<const float*>(reinterpret_cast<const uint16_t*>(wlo) + off[t]);
    return three ? wlo + off[t] : nullptr;
  }
  int slot(int l, int k) const { return l * kSlotsPerLayer + k; }
  int slot_xf() const { return (int)L * kSlotsPerLayer; }
  int slot_dlog() const { return slot_xf() + 1; }
  int slot_w() const { return slot_xf() + 2; }
  float* Pp(int t) { return params + off[t]; }
  float* G(int t) { return grads + off[t]; }
  int lt(int l, int j) const { return 1 + l * kPerLayer + j; }
  int lnf_g() const { return 1 + (int)L * kPerLayer; }
  int lnf_b() const { return 2 + (int)L * kPerLayer; }
};

namespace {

// RAII profiling bracket: records an event pair around a launch group when
// profiling is on.
struct Mark {
  et_b200_lm* lm;
  ProfileMark* m = nullptr;
  Mark(et_b200_lm* l, int cls, double flop, double bytes) : lm(l) {
    if (!lm->profile) return;
    if (lm->mark_used == lm->marks.size()) {
      ProfileMark pm{};
      cudaEventCreate(&pm.start);
      cudaEventCreate(&pm.stop);
      lm->marks.push_back(pm);
    }
    m = &lm->marks[lm->mark_used++];
    m->cls = cls;
    m->flop = flop;
    m->bytes = bytes;
    cudaEventRecord(m->start, lm->stream);
  }
  ~Mark() {
    if (m) cudaEventRecord(m->stop, lm->stream);
  }
};

template <typename T>
T* dalloc(et_b200_lm* lm, size_t count, cudaError_t* err) {
  void* p = nullptr;
  if (count == 0) count = 1;
  cudaError_t st = cudaMalloc(&p, count * sizeof(T));
  if (st != cudaSuccess) {
    *err = st;
    return nullptr;
  }
  lm->allocations.push_back(p);
  return static_cast<T*>(p);
}

void tensor_sizes(const et_b200_lm_config_v1& c, std::vector<size_t>& sz) {
  const size_t d = c.d_model, F = c.ffn, V = c.vocabulary;
  sz.clear();
  sz.push_back(V * d);
  for (int64_t l = 0; l < c.layers; l++) {
    sz.push_back(d); sz.push_back(d);
    sz.push_back(3 * d * d); sz.push_back(3 * d);
    sz.push_back(d * d); sz.push_back(d);
    sz.push_back(d); sz.push_back(d);
    sz.push_back(F * d); sz.push_back(F);
    sz.push_back(d * F); sz.push_back(d);
  }
  sz.push_back(d);
  sz.push_back(d);
}

float fbits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }

// Square-and-multiply power with one f32 rounding per product
// (o2_optimizer.c:419-435).
float pow_steps(float base, uint64_t e) {
  volatile float result = 1.0f;
  volatile float b = base;
  while (e != 0u) {
    if (e & 1u) result = result * b;
    e >>= 1u;
    if (e != 0u) b = b * b;
  }
  return result;
}

void split(et_b200_lm* lm, float* x, float* lo, size_t n) {
  Mark mk(lm, P_SPLIT, 0, 12.0 * n);
  split_tf32(x, x, lo, n, lm->stream);
}

// Head widths whose attention runs on the tensor-core kernels both ways.
// split-f16 steps at head_dim 64 / 128: the binary16 attention, whose
// operand pairs the QKV and dO GEMM epilogues write with slot exponents
bool attn16(const et_b200_lm* lm) { return lm->step16 && (lm->Dh == 64 || lm->Dh == 128); }
// the tensor-core attention reads only the operands the GEMM epilogues write
bool tc_attention(const et_b200_lm* lm) { return lm->Dh == 32 || lm->Dh == 64 || attn16(lm); }
// A step that cannot be computed as enqueued fails through the device error
// word (the host-synchronised entry points report it).
void fail_step(const char* why) {
  fprintf(stderr, "et_b200: %s\n", why);
  static const int one = 1;
  cudaMemcpy(device_error_word(), &one, sizeof(int), cudaMemcpyHostToDevice);
}

// Output format of the producer of slot s: the binary16 pair in split-f16
// steps, and its max |x| in every step of a split-f16 model.
OperandScale osc(et_b200_lm* lm, int s) {
  if (!lm->f16) return OperandScale{};
  return OperandScale{lm->sexp + s, lm->samax + s, lm->step16 ? 1 : 0};
}
// `elems` binary16 values past base, as the float pointer GemmArgs carries
float* half_at(float* base, size_t elems) {
  return reinterpret_cast<float*>(reinterpret_cast<uint16_t*>(base) + elems);
}
// split-f16 steps: A and B are binary16 pairs scaled by slots sa and sb
void set16(et_b200_lm* lm, GemmArgs& g, int sa, int sb) {
  if (!lm->step16) return;
  g.f16 = true;
  g.exp_a = lm->sexp + sa;
  g.exp_b = lm->sexp + sb;
}
// A tensor that attention wrote as a TF32 pair, as the binary16 pair of
// slot s (split-f16 steps), or only its max |x| (3xTF32 steps of the model).
void operand16(et_b200_lm* lm, const float* hi, const float* lo, size_t n, float* out, int s) {
  if (!lm->f16) return;
  Mark mk(lm, P_SPLIT, 0, (lm->step16 ? 12.0 : 4.0) * n);
  if (lm->step16)
    split_f16(hi, lo, n, reinterpret_cast<uint16_t*>(out), reinterpret_cast<uint16_t*>(out) + n,
              lm->sexp + s, lm->samax + s, lm->stream);
  else
    abs_max(hi, n, lm->samax + s, lm->stream);
}

// ---- linear wrappers ---------------------------------------------------------

// y = x W^T + bias, optionally with a fused epilogue (GemmArgs::epilogue):
// RESIDUAL adds `aux`; GELU_FWD also writes GELU(y) to out2 (hi) / out3 (lo)
// in the format of slot `sout`; QKV also writes the attention operands
// described by `qkv`.  `sa`: the split-f16 slot of x.
void linear_forward(et_b200_lm* lm, const float* x, const float* xlo, int64_t rows, int64_t din,
                    int64_t dout, int wt, const float* bias, float* y,
                    int epilogue = GEMM_EPI_PLAIN, const float* aux = nullptr,
                    float* out2 = nullptr, float* out3 = nullptr, const QkvPrep* qkv = nullptr,
                    int sa = -1, int sout = -1, bool skip_c = false) {
  GemmArgs g{};
  g.M = (int)rows; g.N = (int)dout; g.K = (int)din;
  g.A = x; g.A_lo = xlo; g.lda = din; g.a_kmajor = true;
  g.B = lm->W(wt); g.B_lo = lm->Wlo(wt); g.ldb = din; g.b_kmajor = true;
  g.C = y; g.ldc = dout; g.bias = bias; g.accumulate = false;
  g.epilogue = epilogue; g.aux = aux; g.out2 = out2; g.out3 = out3; g.qkv = qkv;
  g.skip_c = skip_c;
  g.chunk_ws = lm->chunk_ws; g.chunk_ws_floats = lm->chunk_ws_floats;
  set16(lm, g, sa, lm->slot_w());
  if (epilogue == GEMM_EPI_GELU_FWD && sout >= 0) g.out_sc = osc(lm, sout);
  // split-f16 models keep GELU'(u) (not u) for the backward's epilogue
  if (epilogue == GEMM_EPI_GELU_FWD) g.gelu_slope_c = lm->f16;
  Mark mk(lm, P_GEMM, 2.0 * rows * din * dout, 0);
  gemm(g, lm->gprec, lm->stream);
}

// dX = dY W; with gelu_in the epilogue applies the GELU backward of the layer
// whose output this is (dX = dY W * GELU'(gelu_in), hi into dxo and lo into
// dxo_lo) and writes the column sums (that layer's bias gradient) to dsum.
void linear_backward_dx(et_b200_lm* lm, const float* dy, const float* dylo, int64_t rows,
                        int64_t din, int64_t dout, int wt, float* dxo,
                        const float* gelu_in = nullptr, float* dxo_lo = nullptr,
                        float* dsum = nullptr, const AttnGradPrep* dprep = nullptr, int sa = -1,
                        int sout = -1, bool skip_c = false) {
  GemmArgs g{};
  g.M = (int)rows; g.N = (int)din; g.K = (int)dout;
  g.A = dy; g.A_lo = dylo; g.lda = dout; g.a_kmajor = true;
  g.B = lm->W(wt); g.B_lo = lm->Wlo(wt); g.ldb = din; g.b_kmajor = false;
  g.C = dxo; g.ldc = din; g.bias = nullptr; g.accumulate = false;
  if (gelu_in != nullptr) {
    g.epilogue = GEMM_EPI_GELU_BWD; g.aux = gelu_in; g.out2 = dxo_lo; g.dsum = dsum;
    g.epi_ws = lm->epi_ws;
    if (sout >= 0) g.out_sc = osc(lm, sout);
    g.gelu_slope_c = lm->f16;  // gelu_in holds GELU'(u)
  }
  if (dprep != nullptr) {
    g.epilogue = GEMM_EPI_ATTN_DO;
    g.dprep = dprep;
    g.skip_c = skip_c;
  }
  g.chunk_ws = lm->chunk_ws; g.chunk_ws_floats = lm->chunk_ws_floats;
  set16(lm, g, sa, lm->slot_w());
  Mark mk(lm, P_GEMM, 2.0 * rows * din * dout, 0);
  gemm(g, lm->gprec, lm->stream);
}

void linear_backward_dw(et_b200_lm* lm, const float* dy, const float* dylo, const float* x,
                        const float* xlo, int64_t rows, int64_t din, int64_t dout, float* dw,
                        int sa = -1, int sb = -1) {
  GemmArgs g{};
  g.M = (int)dout; g.N = (int)din; g.K = (int)rows;
  g.A = dy; g.A_lo = dylo; g.lda = dout; g.a_kmajor = false;
  g.B = x; g.B_lo = xlo; g.ldb = din; g.b_kmajor = false;
  g.C = dw; g.ldc = din; g.bias = nullptr; g.accumulate = false;
  g.workspace = lm->splitk_ws; g.workspace_floats = lm->splitk_floats;
  g.chunk_ws = lm->chunk_ws; g.chunk_ws_floats = lm->chunk_ws_floats;
  set16(lm, g, sa, sb);
  Mark mk(lm, P_GEMM, 2.0 * rows * din * dout, 0);
  gemm(g, lm->gprec, lm->stream);
}

// db = column sums of dy (+ dy_lo when dy holds only the TF32 hi part).
void bias_grad(et_b200_lm* lm, const float* dy, int64_t rows, int64_t n, float* db,
               const float* dy_lo = nullptr) {
  Mark mk(lm, P_ELEMENTWISE, 0, (dy_lo ? 8.0 : 4.0) * rows * n);
  column_sum(dy, db, rows, n, lm->col_ws, lm->stream, dy_lo);
}

AttnParams attn_params(et_b200_lm* lm, const float* qkv, int layer) {
  AttnParams p{};
  p.B = (int)lm->B; p.Hq = (int)lm->H; p.Hkv = (int)lm->H;
  p.Tq = (int)lm->T; p.Tk = (int)lm->T; p.Dh = (int)lm->Dh;
  p.scale = lm->attn_scale;
  const int64_t w = 3 * lm->d;
  p.q = AttnTensor{qkv, lm->T * w, lm->Dh, w};
  p.k = AttnTensor{qkv + lm->d, lm->T * w, lm->Dh, w};
  p.v = AttnTensor{qkv + 2 * lm->d, lm->T * w, lm->Dh, w};
  p.qpos = lm->pos; p.kpos = lm->pos; p.mask = nullptr;
  p.q_cos = lm->rope_cos; p.q_sin = lm->rope_sin;
  p.k_cos = lm->rope_cos; p.k_sin = lm->rope_sin;
  p.q_rope_batched = 0; p.k_rope_batched = 0;
  p.ws = lm->attn_qkv_ws[layer];
  p.ws_grad = lm->attn_grad_ws;
  p.ws_ready = 0;
  // every step of a split-f16 model records the operands' maxima (the next
  // step's exponents); its split-f16 steps write binary16 operand pairs
  if (lm->f16) p.pair_amax = lm->samax + lm->slot(layer, S_Q);
  if (attn16(lm)) {
    p.pairs16 = 1;
    p.pair_exps = lm->sexp + lm->slot(layer, S_Q);
  }
  return p;
}

double attn_flop(et_b200_lm* lm, double gemms) {
  // causal: half of the dense B*H*T^2*Dh work per 2-FLOP GEMM
  return gemms * 2.0 * lm->B * lm->H * (double)lm->T * lm->T * lm->Dh * 0.5;
}

// ---- forward -------------------------------------------------------------------

void forward(et_b200_lm* lm) {
  const int64_t R = lm->R, d = lm->d, F = lm->F, V = lm->V;
  cudaStream_t s = lm->stream;
  {
    Mark mk(lm, P_EMBED, 0, 8.0 * R * d);
    embedding_forward(lm->ids, lm->Pp(0), lm->layers[0].x, R, V, d, lm->status, s);
  }
  for (int l = 0; l < lm->L; l++) {
    LayerActs& a = lm->layers[l];
    float* xnext = (l + 1 < lm->L) ? lm->layers[l + 1].x : lm->x_final;
    bool fused_o = false;
    {
      Mark mk(lm, P_NORM, 0, 8.0 * R * d);
      // with 3xTF32 the producers write each GEMM operand as a hi/lo pair
      // (split-f16 steps: the binary16 pair, in the same buffers)
      layer_norm_forward(a.x, lm->Pp(lm->lt(l, T_LN1G)), lm->Pp(lm->lt(l, T_LN1B)), lm->eps, a.h1,
                         a.mu1, a.rs1, R, d, s, a.h1lo, osc(lm, lm->slot(l, S_H1)));
    }
    {
      // the QKV epilogue also writes the attention operands (RoPE'd, hi/lo, head-major)
      AttnParams p = attn_params(lm, a.qkv, l);
      QkvPrep prep;
      p.qkv_ready = attention_qkv_prep(p, &prep) ? 1 : 0;
      // the tensor-core attention (forward and backward) reads only the
      // operands the epilogue writes, so the f32 qkv itself is not stored
      const bool skip = p.qkv_ready && tc_attention(lm);
      linear_forward(lm, a.h1, a.h1lo, R, d, 3 * d, lm->lt(l, T_WQKV), lm->Pp(lm->lt(l, T_BQKV)),
                     a.qkv, p.qkv_ready ? GEMM_EPI_QKV : GEMM_EPI_PLAIN, nullptr, nullptr,
                     nullptr, p.qkv_ready ? &prep : nullptr, lm->slot(l, S_H1), -1, skip);
      Mark mk(lm, P_ATTN_FWD, attn_flop(lm, 2), 0);
      // split-f16 steps: the tensor-core forward writes o's binary16 pair
      // itself; in every step of such a model it records o's max
      const bool o16 = lm->step16 && skip;
      AttnOut out = o16 ? AttnOut{a.ao16, lm->T * d, lm->Dh, d, half_at(a.ao16, R * d)}
                        : AttnOut{a.ao, lm->T * d, lm->Dh, d, a.aolo};
      if (lm->f16 && p.qkv_ready && (o16 || !lm->step16)) out.sc = osc(lm, lm->slot(l, S_AO));
      lm->attn_prepared[l] = attention_forward(p, out, a.am, a.al, s);
      if (skip && !lm->attn_prepared[l]) fail_step("attention forward left the tensor-core path");
      fused_o = lm->attn_prepared[l] && out.sc.amax != nullptr;
    }
    if (lm->three && !lm->attn_prepared[l]) split(lm, a.ao, a.aolo, R * d);
    // the output projection's operand (split-f16: the binary16 pair of o),
    // unless the attention epilogue produced it
    if (!fused_o) operand16(lm, a.ao, a.aolo, R * d, a.ao16, lm->slot(l, S_AO));
    const float* aoh = lm->step16 ? a.ao16 : a.ao;
    const float* aol = lm->step16 ? half_at(a.ao16, R * d) : a.aolo;
    // x' = x + o Wo^T + bo (the residual add in the GEMM epilogue)
    linear_forward(lm, aoh, aol, R, d, d, lm->lt(l, T_WO), lm->Pp(lm->lt(l, T_BO)), a.xmid,
                   GEMM_EPI_RESIDUAL, a.x, nullptr, nullptr, nullptr, lm->slot(l, S_AO));
    {
      Mark mk(lm, P_NORM, 0, 8.0 * R * d);
      layer_norm_forward(a.xmid, lm->Pp(lm->lt(l, T_LN2G)), lm->Pp(lm->lt(l, T_LN2B)), lm->eps,
                         a.h2, a.mu2, a.rs2, R, d, s, a.h2lo, osc(lm, lm->slot(l, S_H2)));
    }
    // u = h2 W1^T + b1 and g = GELU(u) (hi/lo) from the same epilogue
    linear_forward(lm, a.h2, a.h2lo, R, d, F, lm->lt(l, T_W1), lm->Pp(lm->lt(l, T_B1)), a.u,
                   GEMM_EPI_GELU_FWD, nullptr, a.g, a.glo, nullptr, lm->slot(l, S_H2),
                   lm->slot(l, S_G));
    linear_forward(lm, a.g, a.glo, R, F, d, lm->lt(l, T_W2), lm->Pp(lm->lt(l, T_B2)), xnext,
                   GEMM_EPI_RESIDUAL, a.xmid, nullptr, nullptr, nullptr, lm->slot(l, S_G));
  }
  {
    Mark mk(lm, P_NORM, 0, 8.0 * R * d);
    layer_norm_forward(lm->x_final, lm->Pp(lm->lnf_g()), lm->Pp(lm->lnf_b()), lm->eps, lm->xf,
                       lm->muf, lm->rsf, R, d, s, lm->xflo, osc(lm, lm->slot_xf()));
  }
  linear_forward(lm, lm->xf, lm->xflo, R, d, V, 0, nullptr, lm->logits, GEMM_EPI_PLAIN, nullptr,
                 nullptr, nullptr, nullptr, lm->slot_xf());
  {
    Mark mk(lm, P_CE, 0, (lm->step16 ? 8.0 : 12.0) * R * V + 12.0 * R);
    // dlogits in place of the logits (TF32 hi, lo in logits_lo), or
    // (split-f16 steps) its binary16 pair in logits_lo: hi, then lo
    float* dh = lm->step16 ? lm->logits_lo : lm->logits;
    float* dl = lm->step16 ? half_at(lm->logits_lo, (size_t)R * V) : lm->logits_lo;
    // a loss mask seeds each row with its numerator (mask 2^-k) and puts
    // the mask's sum, the objective's weight, behind the step-void flag
    // (grads[P + 1]), which the last gradient all-reduce sums over ranks
    if (lm->masked)
      loss_mask_seed(lm->loss_mask, R, lm->mask_scale, lm->upstream, lm->grads + lm->P + 1,
                     lm->status, s);
    ce_fused(lm->logits, dh, lm->targets, lm->masked ? lm->upstream : nullptr, lm->ce_scale,
             lm->loss_rows, R, V, lm->status, s, dl, osc(lm, lm->slot_dlog()));
    mean_loss(lm->loss_rows, R, lm->loss_mean, s, lm->masked ? lm->loss_mask : nullptr);
  }
}

// ---- backward --------------------------------------------------------------------

void allreduce_range(et_b200_lm* lm, int t_begin, int t_end, cudaEvent_t ready) {
  if (!lm->dp) return;
  cudaEventRecord(ready, lm->stream);
  cudaStreamWaitEvent(lm->comm, ready, 0);
  const size_t begin = lm->off[t_begin];
  const size_t end = lm->off[t_end - 1] + lm->sz[t_end - 1];
  nccl().AllReduce(lm->grads + begin, lm->grads + begin, end - begin, ncclFloat32, ncclSum,
                   lm->nccl_comm, lm->comm);
}

void backward(et_b200_lm* lm) {
  const int64_t R = lm->R, d = lm->d, F = lm->F, V = lm->V;
  cudaStream_t s = lm->stream;
  const bool three = lm->three;
  // head (tied): dlogits already in place of the logits (split-f16 steps:
  // its binary16 pair in logits_lo)
  float* dlog = lm->step16 ? lm->logits_lo : lm->logits;
  float* dlog_lo = lm->step16 ? half_at(lm->logits_lo, (size_t)R * V) : lm->logits_lo;
  linear_backward_dx(lm, dlog, dlog_lo, R, d, V, 0, lm->dtmp, nullptr, nullptr, nullptr, nullptr,
                     lm->slot_dlog());
  linear_backward_dw(lm, dlog, dlog_lo, lm->xf, lm->xflo, R, d, V, lm->G(0), lm->slot_dlog(),
                     lm->slot_xf());
  {
    Mark mk(lm, P_NORM, 0, 16.0 * R * d);
    // the column sums of this dx are the last layer's b2 gradient
    layer_norm_backward(lm->x_final, lm->Pp(lm->lnf_g()), lm->muf, lm->rsf, lm->dtmp, lm->dx, 0,
                        lm->G(lm->lnf_g()), lm->G(lm->lnf_b()), lm->ln_ws, R, d, s, lm->dxhi,
                        lm->dxlo, lm->G(lm->lt((int)lm->L - 1, T_B2)),
                        osc(lm, lm->slot((int)lm->L - 1, S_DXF)));
  }
  for (int l = (int)lm->L - 1; l >= 0; l--) {
    LayerActs& a = lm->layers[l];
    bool dqkv_split = false, bqkv_done = false;
    // FFN down: dY = dx (flows to the skip and the branch)
    // dx arrives with its hi/lo pair and its column sums (this layer's b2
    // gradient) from the LayerNorm backward above
    const float* dyh = three ? lm->dxhi : lm->dx;
    const float* dyl = three ? lm->dxlo : nullptr;
    // du = (dy W2) * GELU'(u) (hi/lo) and the b1 gradient, from the epilogue
    linear_backward_dx(lm, dyh, dyl, R, F, d, lm->lt(l, T_W2), lm->du, a.u, lm->dulo,
                       lm->G(lm->lt(l, T_B1)), nullptr, lm->slot(l, S_DXF), lm->slot(l, S_DU));
    linear_backward_dw(lm, dyh, dyl, a.g, a.glo, R, F, d, lm->G(lm->lt(l, T_W2)),
                       lm->slot(l, S_DXF), lm->slot(l, S_G));
    linear_backward_dx(lm, lm->du, lm->dulo, R, d, F, lm->lt(l, T_W1), lm->dtmp, nullptr, nullptr,
                       nullptr, nullptr, lm->slot(l, S_DU));
    linear_backward_dw(lm, lm->du, lm->dulo, a.h2, a.h2lo, R, d, F, lm->G(lm->lt(l, T_W1)),
                       lm->slot(l, S_DU), lm->slot(l, S_H2));
    {
      Mark mk(lm, P_NORM, 0, 20.0 * R * d);
      layer_norm_backward(a.xmid, lm->Pp(lm->lt(l, T_LN2G)), a.mu2, a.rs2, lm->dtmp, lm->dx, 1,
                          lm->G(lm->lt(l, T_LN2G)), lm->G(lm->lt(l, T_LN2B)), lm->ln_ws, R, d, s,
                          lm->dxhi, lm->dxlo, lm->G(lm->lt(l, T_BO)),  // + the bo gradient
                          osc(lm, lm->slot(l, S_DXA)));
    }
    // attention output projection: dY = dx
    dyh = three ? lm->dxhi : lm->dx;
    dyl = three ? lm->dxlo : nullptr;
    // dO = dY Wo; its epilogue also writes the attention backward's dO
    // operands and delta
    AttnParams p = attn_params(lm, a.qkv, l);
    p.ws_ready = lm->attn_prepared[l];
    // o as the forward left it: its binary16 pair (split-f16 steps on the
    // tensor-core path) or its TF32 pair
    const bool o16 = lm->step16 && p.ws_ready && tc_attention(lm);
    const AttnTensor ao{o16 ? a.ao16 : a.ao, lm->T * d, lm->Dh, d};
    const float* ao_lo = o16 ? half_at(a.ao16, R * d) : a.aolo;
    AttnGradPrep dprep;
    p.grad_ready = attention_grad_prep(p, ao, ao_lo, a.am, a.al, lm->delta, &dprep) ? 1 : 0;
    if (o16) dprep.o_exp = lm->sexp + lm->slot(l, S_AO);
    if (o16 && !p.grad_ready) fail_step("attention backward cannot read a binary16 output");
    // dO itself (dtmp) is not stored when the tensor-core backward reads only
    // the epilogue's operands
    const bool skip_do = p.grad_ready && p.ws_ready && tc_attention(lm);
    linear_backward_dx(lm, dyh, dyl, R, d, d, lm->lt(l, T_WO), lm->dtmp, nullptr, nullptr, nullptr,
                       p.grad_ready ? &dprep : nullptr, lm->slot(l, S_DXA), -1, skip_do);
    // dO's max where no epilogue recorded it (the next split-f16 step's exponent)
    if (p.pair_amax != nullptr && !p.grad_ready) abs_max(lm->dtmp, R * d, p.pair_amax + 3, s);
    linear_backward_dw(lm, dyh, dyl, lm->step16 ? a.ao16 : a.ao,
                       lm->step16 ? half_at(a.ao16, R * d) : a.aolo, R, d, d,
                       lm->G(lm->lt(l, T_WO)), lm->slot(l, S_DXA), lm->slot(l, S_AO));
    bool fused_g = false;
    {
      Mark mk(lm, P_ATTN_BWD, attn_flop(lm, 4), 0);
      const int64_t w = 3 * d;
      // the tensor-core backward also writes per-tile column sums of dq, dk,
      // dv; in split-f16 steps it writes dqkv's binary16 pair itself, and in
      // every step of such a model it records dqkv's max
      const bool g16 = lm->step16 && skip_do;
      float* base = g16 ? lm->dqkv16 : lm->dqkv;
      float* lo = g16 ? half_at(lm->dqkv16, R * w) : lm->dqkvlo;  // null unless pairs
      auto at = [&](float* x, int64_t e) { return x == nullptr ? nullptr : g16 ? half_at(x, e) : x + e; };
      float* cp = lm->qkv_colpart;
      AttnOut dq{base, lm->T * w, lm->Dh, w, lo, cp, w};
      AttnOut dk{at(base, d), lm->T * w, lm->Dh, w, at(lo, d), cp + d, w};
      AttnOut dv{at(base, 2 * d), lm->T * w, lm->Dh, w, at(lo, 2 * d), cp + 2 * d, w};
      if (lm->f16 && (g16 || !lm->step16))
        dq.sc = dk.sc = dv.sc = osc(lm, lm->slot(l, S_DQKV));
      const bool tc = attention_backward(p, ao, ao_lo, AttnTensor{lm->dtmp, lm->T * d, lm->Dh, d},
                                         a.am, a.al, lm->delta, dq, dk, dv, s);
      dqkv_split = tc && three;
      bqkv_done = tc;
      fused_g = tc && dq.sc.amax != nullptr;
      if (skip_do && !tc) fail_step("attention backward left the tensor-core path");
    }
    if (three && !dqkv_split) split(lm, lm->dqkv, lm->dqkvlo, R * 3 * d);
    // the QKV projection's operand (split-f16: the binary16 pair of dqkv),
    // unless the attention epilogues produced it
    if (!fused_g) operand16(lm, lm->dqkv, lm->dqkvlo, R * 3 * d, lm->dqkv16, lm->slot(l, S_DQKV));
    if (bqkv_done) {
      Mark mk(lm, P_ELEMENTWISE, 0, 4.0 * lm->qkv_colrows * 3 * d);
      reduce_partials(lm->qkv_colpart, (int)lm->qkv_colrows, 3 * d, 3 * d,
                      lm->G(lm->lt(l, T_BQKV)), nullptr, nullptr, s);
    } else {
      bias_grad(lm, lm->dqkv, R, 3 * d, lm->G(lm->lt(l, T_BQKV)), three ? lm->dqkvlo : nullptr);
    }
    const float* gq = lm->step16 ? lm->dqkv16 : lm->dqkv;
    const float* gql = lm->step16 ? half_at(lm->dqkv16, R * 3 * d) : lm->dqkvlo;
    linear_backward_dx(lm, gq, gql, R, d, 3 * d, lm->lt(l, T_WQKV), lm->dtmp, nullptr, nullptr,
                       nullptr, nullptr, lm->slot(l, S_DQKV));
    linear_backward_dw(lm, gq, gql, a.h1, a.h1lo, R, d, 3 * d, lm->G(lm->lt(l, T_WQKV)),
                       lm->slot(l, S_DQKV), lm->slot(l, S_H1));
    {
      Mark mk(lm, P_NORM, 0, 20.0 * R * d);
      // layer 0's dx only feeds the embedding gradient: no operand pair
      // + the b2 gradient of the layer below
      layer_norm_backward(a.x, lm->Pp(lm->lt(l, T_LN1G)), a.mu1, a.rs1, lm->dtmp, lm->dx, 1,
                          lm->G(lm->lt(l, T_LN1G)), lm->G(lm->lt(l, T_LN1B)), lm->ln_ws, R, d, s,
                          l > 0 ? lm->dxhi : nullptr, l > 0 ? lm->dxlo : nullptr,
                          l > 0 ? lm->G(lm->lt(l - 1, T_B2)) : nullptr,
                          l > 0 ? osc(lm, lm->slot(l - 1, S_DXF)) : OperandScale{});
    }
    allreduce_range(lm, lm->lt(l, 0), lm->lt(l, 0) + kPerLayer, lm->layer_done[l]);
  }
  {
    Mark mk(lm, P_EMBED, 0, 12.0 * V * d + 8.0 * R * d);
    embedding_backward(lm->ids, lm->dx, lm->G(0), lm->G(0), R, V, d, lm->emb_scratch, s);
  }
  // The step-void flag at grads[P] rides the last gradient reduction, so
  // every rank agrees on skipping AdamW: + kVoidIndex for a token id or
  // target out of range (or a loss mask byte other than 0 / 1), + 1
  // (split-f16 steps) for an operand that reached binary16's overflow.  The
  // loss mask's weight at grads[P + 1] rides along (summed: the global
  // weight).
  fold_index_flag(lm->status, lm->grads + lm->P, kVoidIndex, s);
  if (lm->step16)
    operand_range_check(lm->samax, lm->sexp, lm->nslots, lm->slot_w(), lm->grads + lm->P, s);
  if (lm->dp) {
    allreduce_range(lm, 0, 1, lm->tail_done);
    const int lg = lm->lnf_g();
    const size_t end = lm->P + 2;
    nccl().AllReduce(lm->G(lg), lm->G(lg), end - lm->off[lg], ncclFloat32, ncclSum,
                     lm->nccl_comm, lm->comm);
    cudaEventRecord(lm->comm_done, lm->comm);
    Mark mk(lm, P_ALLREDUCE_WAIT, 0, 0);
    cudaStreamWaitEvent(s, lm->comm_done, 0);
  }
}

void refresh_weight_split(et_b200_lm* lm) {
  if (!lm->three) return;
  Mark mk(lm, P_SPLIT, 0, 12.0 * lm->P);
  split_tf32(lm->params, lm->whi, lm->wlo, lm->P, lm->stream);
  lm->w16_valid = false;
}

// The weights' exponent from their current max |w| (kept until the weights
// are split again: AdamW writes the next pair with it).
void weight_scale(et_b200_lm* lm) {
  unsigned* am = lm->samax + lm->slot_w();
  cudaMemsetAsync(am, 0, sizeof(unsigned), lm->stream);
  abs_max(lm->params, lm->P, am, lm->stream);
  scale_from_amax(am, lm->sexp + lm->slot_w(), 1, lm->scale_target, 1, lm->stream);
}

// Operand formats for the step about to be enqueued (split-f16 models):
// binary16 pairs once a finished step has measured every slot, else 3xTF32
// with the TF32 weight pair and every slot's max recorded.
void begin_step(et_b200_lm* lm) {
  // the step-void flag and the loss mask's weight behind the gradients, and
  // this step's status words
  cudaMemsetAsync(lm->grads + lm->P, 0, 2 * sizeof(float), lm->stream);
  cudaMemsetAsync(lm->status, 0, 2 * sizeof(int), lm->stream);
  if (!lm->f16) return;
  lm->step16 = lm->calibrated;
  if (lm->step16) {
    // exponents of the activation / gradient slots from the last step's maxima
    scale_from_amax(lm->samax, lm->sexp, lm->slot_w(), lm->scale_target, 1, lm->stream);
    if (!lm->w16_valid) {
      Mark mk(lm, P_SPLIT, 0, 8.0 * lm->P);
      weight_scale(lm);
      split_f16(lm->params, nullptr, lm->P, reinterpret_cast<uint16_t*>(lm->whi),
                reinterpret_cast<uint16_t*>(lm->wlo), lm->sexp + lm->slot_w(),
                lm->samax + lm->slot_w(), lm->stream);
      lm->w16_valid = true;
    }
  } else {
    cudaMemsetAsync(lm->samax, 0, lm->nslots * sizeof(unsigned), lm->stream);
    refresh_weight_split(lm);
    weight_scale(lm);
  }
}

void optimizer_step(et_b200_lm* lm) {
  const et_b200_lm_config_v1& c = lm->cfg;
  AdamwTensor h{};
  h.value = lm->params;
  h.grad = lm->grads;
  h.exp_avg = lm->m1;
  h.exp_avg_sq = lm->m2;
  h.count = lm->P;
  volatile float b1 = fbits(c.beta1_bits), b2 = fbits(c.beta2_bits);
  volatile float one = 1.0f;
  h.beta1 = b1;
  h.beta2 = b2;
  h.one_minus_beta1 = one - b1;
  h.one_minus_beta2 = one - b2;
  // bias1 / bias2 come from the device's update counter (adamw_prepare)
  volatile float lr = fbits(c.learning_rate_bits) * 1.0f;  // constant schedule factor 1
  volatile float lrwd = lr * fbits(c.weight_decay_bits);
  h.lr = lr;
  h.decay = one - lrwd;
  h.epsilon = fbits(c.epsilon_bits);
  h.envelope = adamw_envelope_ok(h) ? 1 : 0;
  // with 3xTF32 the same pass refreshes the weights' (hi, lo) operand pair;
  // split-f16 models always write the binary16 pair (the next step's format)
  h.value_hi = lm->three ? lm->whi : nullptr;
  h.value_lo = lm->three ? lm->wlo : nullptr;
  if (lm->f16) h.value_sc = OperandScale{lm->sexp + lm->slot_w(), lm->samax + lm->slot_w(), 1};
  cudaMemcpyAsync(lm->d_adam, &h, sizeof(h), cudaMemcpyHostToDevice, lm->stream);
  adamw_prepare(lm->d_adam, lm->d_completed, lm->stream);
  // all or nothing: skipped when the step is void (flag summed across ranks)
  // or when the check pass finds a nonfinite gradient, moment or result
  // with a loss mask the gradients hold numerators 2^-k: AdamW divides them
  // by the global weight 2^-k (the reference's O2 division by the
  // accumulated weight, o2_optimizer.c:1738, exact in the scaling)
  const AdamwControl ctl{lm->grads + lm->P, lm->status, lm->d_completed,
                         lm->masked ? lm->grads + lm->P + 1 : nullptr, lm->mask_scale};
  {
    Mark mk(lm, P_ADAMW_CHECK, 0, 16.0 * lm->P);
    adamw_check(lm->d_adam, lm->d_prefix, 1, lm->P, 1.0f, 1.0f, ctl, true, lm->stream);
  }
  {
    Mark mk(lm, P_ADAMW, 0, (lm->f16 ? 32.0 : lm->three ? 36.0 : 28.0) * lm->P);
    adamw_apply(lm->d_adam, lm->d_prefix, 1, lm->P, 1.0f, 1.0f, ctl, true, lm->stream);
  }
  if (lm->f16) lm->w16_valid = true;
}

int32_t check_ready(et_b200_lm* lm, et_kernel_error* e, const char* op) {
  if (lm == nullptr) return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op, "model is null");
  cudaSetDevice(lm->device);
  return 0;
}

// Reads the loss and the flags of the step just enqueued.  *redo: a
// split-f16 step that was not applied (an operand reached binary16's
// overflow on some rank); `update`: the step ran the AdamW passes.  A step
// that fails here has left parameters, moments and the update counter as
// they were.  Updates skipped by steps enqueued with
// et_b200_lm_step_device_v1 since the last synchronised call are added to
// the skipped-update counter, not reported as this call's error.
int32_t finish_host_step(et_b200_lm* lm, float* host_loss, et_kernel_error* e, const char* op,
                         bool update, bool* redo) {
  float loss = 0.0f, flag = 0.0f, weight = 1.0f;
  int flags[3] = {0, 0, 0};
  int word = 0;
  uint64_t completed = 0;
  *redo = false;
  cudaMemcpyAsync(&loss, lm->loss_mean, sizeof(float), cudaMemcpyDeviceToHost, lm->stream);
  cudaMemcpyAsync(flags, lm->status, sizeof(flags), cudaMemcpyDeviceToHost, lm->stream);
  cudaMemcpyAsync(&word, device_error_word(), sizeof(int), cudaMemcpyDeviceToHost, lm->stream);
  cudaMemcpyAsync(&flag, lm->grads + lm->P, sizeof(float), cudaMemcpyDeviceToHost, lm->stream);
  if (lm->masked)
    cudaMemcpyAsync(&weight, lm->grads + lm->P + 1, sizeof(float), cudaMemcpyDeviceToHost,
                    lm->stream);
  cudaMemcpyAsync(&completed, lm->d_completed, sizeof(completed), cudaMemcpyDeviceToHost,
                  lm->stream);
  cudaError_t st = cudaStreamSynchronize(lm->stream);
  if (st != cudaSuccess) return cuda_error(e, st, op);
  if (host_loss) *host_loss = loss;
  lm->updates = completed;
  const bool void_step = flag != 0.0f || (update && flags[1] != 0);
  if (flags[2] != 0) {
    lm->skipped += (uint64_t)(flags[2] - (update && void_step ? 1 : 0));
    cudaMemsetAsync(lm->status + 2, 0, sizeof(int), lm->stream);
    cudaStreamSynchronize(lm->stream);
    // a skipped device step may have been a split-f16 overflow: re-measure
    if (lm->f16) lm->calibrated = false;
  }
  if (word != 0) {
    cudaMemset(device_error_word(), 0, sizeof(int));
    return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "a device pipeline wait timed out");
  }
  if (flag >= kVoidIndex)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     (flags[0] & 1) ? "token id or target outside the vocabulary; nothing was updated"
                     : (flags[0] & 2) ? "loss mask byte other than 0 or 1; nothing was updated"
                                      : "another rank's token id, target or loss mask byte is "
                                        "invalid; nothing was updated");
  if (flag != 0.0f && lm->step16) {
    *redo = true;
    return 0;
  }
  if (lm->masked && weight == 0.0f)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     update ? "the loss mask selects no token on any rank; nothing was updated"
                            : "the loss mask selects no token on any rank");
  if (update && (flags[1] & kAdamwInputNonfinite))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "parameter, gradient, or moment is nonfinite; nothing was updated");
  if (update && (flags[1] & kAdamwProducedNonfinite))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "AdamW produced a nonfinite value; nothing was updated");
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

void collect_profile(et_b200_lm* lm);

// One host-synchronised step (forward, backward and, with `update`, AdamW).
// A split-f16 step whose operand check fails was not applied; it is redone
// with 3xTF32 contractions, which also re-measure every operand's scale.
int32_t run_host_step(et_b200_lm* lm, bool update, float* host_loss, et_kernel_error* e,
                      const char* op) {
  for (int attempt = 0; attempt < 2; attempt++) {
    begin_step(lm);
    forward(lm);
    backward(lm);
    if (update) optimizer_step(lm);
    bool redo = false;
    const int32_t rc = finish_host_step(lm, host_loss, e, op, update, &redo);
    collect_profile(lm);
    if (rc != 0) return rc;
    if (!redo) {
      if (lm->f16) lm->calibrated = true;
      return 0;
    }
    lm->calibrated = false;
    lm->redone_steps++;
  }
  return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                   "the step's operands stayed outside their binary16 range");
}

void collect_profile(et_b200_lm* lm) {
  if (!lm->profile) return;
  for (size_t i = 0; i < lm->mark_used; i++) {
    ProfileMark& m = lm->marks[i];
    float ms = 0.0f;
    if (cudaEventSynchronize(m.stop) == cudaSuccess &&
        cudaEventElapsedTime(&ms, m.start, m.stop) == cudaSuccess) {
      lm->prof[m.cls][0] += 1;
      lm->prof[m.cls][1] += ms;
      lm->prof[m.cls][2] += m.flop;
      lm->prof[m.cls][3] += m.bytes;
    }
  }
  lm->mark_used = 0;
}

}  // namespace

extern "C" {

int32_t et_b200_lm_create_v1(const et_b200_lm_config_v1* c, et_b200_lm** out,
                             et_kernel_error* e) {
  const char* op = "lm-create";
  if (c == nullptr || out == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op, "config and output are required");
  *out = nullptr;
  if (c->struct_size < sizeof(et_b200_lm_config_v1))
    return set_error(e, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_INVALID_STRUCT_SIZE, op, "config is truncated");
  if (c->layers < 1 || c->d_model < 2 || c->heads < 1 || c->d_model % c->heads != 0 ||
      (c->d_model / c->heads) % 2 != 0 || c->d_model / c->heads > 128 || c->ffn < 1 ||
      c->vocabulary < 1 || c->seq_len < 1 || c->batch < 1 || c->precision > 3)
    return set_error(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                     "unsupported model shape (head dim must be even and <= 128)");
  int32_t rc = et_b200_device_check_v1(e);
  if (rc != 0) return rc;
  et_b200_lm* lm = new et_b200_lm();
  lm->cfg = *c;
  cudaGetDevice(&lm->device);
  lm->L = c->layers; lm->d = c->d_model; lm->H = c->heads; lm->Dh = c->d_model / c->heads;
  lm->F = c->ffn; lm->V = c->vocabulary; lm->T = c->seq_len; lm->B = c->batch;
  lm->R = lm->B * lm->T;
  const double global = c->global_tokens > 0 ? (double)c->global_tokens : (double)lm->R;
  lm->ce_scale = (float)(1.0 / global);
  lm->mask_scale = std::ldexp(1.0f, -(int)std::ceil(std::log2(global)));
  lm->eps = fbits(c->ln_epsilon_bits);
  {
    volatile float root = sqrtf((float)lm->Dh);
    lm->attn_scale = 1.0f / root;
  }
  lm->precision = (int)c->precision;
  lm->three = c->precision == ET_B200_PRECISION_TF32X3 || c->precision == ET_B200_PRECISION_F16X3;
  lm->gprec = lm->three ? (int)ET_B200_PRECISION_TF32X3 : lm->precision;
  // split-f16 needs binary16 rows of 16-byte multiples and the register-row
  // LayerNorm backward; other shapes run the whole step 3xTF32
  lm->f16 = c->precision == ET_B200_PRECISION_F16X3 && c->d_model % 128 == 0 &&
            c->d_model <= 1024 && c->ffn % 8 == 0 && c->vocabulary % 8 == 0;
  if (const char* t = getenv("ET_B200_F16_SCALE_TARGET")) {
    const int v = atoi(t);
    if (v >= 2 && v <= 17) lm->scale_target = v;
  }
  tensor_sizes(*c, lm->sz);
  lm->off.resize(lm->sz.size());
  size_t total = 0;
  for (size_t i = 0; i < lm->sz.size(); i++) {
    lm->off[i] = total;
    total += (lm->sz[i] + 7) & ~(size_t)7;  // every tensor 16-byte aligned, also as binary16
  }
  lm->P = total;
  cudaError_t err = cudaSuccess;
  const int64_t R = lm->R, d = lm->d, F = lm->F, V = lm->V, L = lm->L;
  cudaStreamCreateWithFlags(&lm->stream, cudaStreamNonBlocking);
  cudaStreamCreateWithFlags(&lm->comm, cudaStreamNonBlocking);
  lm->params = dalloc<float>(lm, lm->P, &err);
  lm->grads = dalloc<float>(lm, lm->P + 8, &err);  // + the step-void flag [P], mask weight [P + 1]
  lm->m1 = dalloc<float>(lm, lm->P, &err);
  lm->m2 = dalloc<float>(lm, lm->P, &err);
  if (lm->three) {
    lm->whi = dalloc<float>(lm, lm->P, &err);
    lm->wlo = dalloc<float>(lm, lm->P, &err);
  }
  lm->d_adam = dalloc<AdamwTensor>(lm, 1, &err);
  lm->d_prefix = dalloc<uint64_t>(lm, 2, &err);
  lm->layers.resize(L);
  for (int64_t l = 0; l < L; l++) {
    LayerActs& a = lm->layers[l];
    a.x = dalloc<float>(lm, R * d, &err);
    a.h1 = dalloc<float>(lm, R * d, &err);
    a.mu1 = dalloc<float>(lm, R, &err);
    a.rs1 = dalloc<float>(lm, R, &err);
    a.qkv = dalloc<float>(lm, R * 3 * d, &err);
    a.ao = dalloc<float>(lm, R * d, &err);
    a.am = dalloc<float>(lm, R * lm->H, &err);
    a.al = dalloc<float>(lm, R * lm->H, &err);
    a.xmid = dalloc<float>(lm, R * d, &err);
    a.h2 = dalloc<float>(lm, R * d, &err);
    a.mu2 = dalloc<float>(lm, R, &err);
    a.rs2 = dalloc<float>(lm, R, &err);
    a.u = dalloc<float>(lm, R * F, &err);
    a.g = dalloc<float>(lm, R * F, &err);
    if (lm->three) {
      a.h1lo = dalloc<float>(lm, R * d, &err);
      a.aolo = dalloc<float>(lm, R * d, &err);
      a.h2lo = dalloc<float>(lm, R * d, &err);
      a.glo = dalloc<float>(lm, R * F, &err);
    }
    if (lm->f16) a.ao16 = dalloc<float>(lm, R * d, &err);
  }
  lm->x_final = dalloc<float>(lm, R * d, &err);
  lm->xf = dalloc<float>(lm, R * d, &err);
  lm->muf = dalloc<float>(lm, R, &err);
  lm->rsf = dalloc<float>(lm, R, &err);
  lm->logits = dalloc<float>(lm, (size_t)R * V, &err);
  lm->loss_rows = dalloc<float>(lm, R, &err);
  lm->loss_mean = dalloc<float>(lm, 1, &err);
  lm->dx = dalloc<float>(lm, R * d, &err);
  lm->dtmp = dalloc<float>(lm, R * d, &err);
  lm->dqkv = dalloc<float>(lm, R * 3 * d, &err);
  lm->du = dalloc<float>(lm, R * F, &err);
  lm->delta = dalloc<float>(lm, R * lm->H, &err);
  if (lm->three) {
    lm->xflo = dalloc<float>(lm, R * d, &err);
    lm->logits_lo = dalloc<float>(lm, (size_t)R * V, &err);
    lm->dxhi = dalloc<float>(lm, R * d, &err);
    lm->dxlo = dalloc<float>(lm, R * d, &err);
    lm->dqkvlo = dalloc<float>(lm, R * 3 * d, &err);
    lm->dulo = dalloc<float>(lm, R * F, &err);
  }
  if (lm->f16) {
    lm->dqkv16 = dalloc<float>(lm, R * 3 * d, &err);
    lm->nslots = (int)L * kSlotsPerLayer + 3;
    lm->sexp = dalloc<int>(lm, lm->nslots, &err);
    lm->samax = dalloc<unsigned>(lm, lm->nslots, &err);
  }
  const size_t widest = (size_t)std::max<int64_t>(3 * d, F);
  lm->ln_ws = dalloc<float>(lm, ln_workspace_floats(R, d), &err);
  lm->col_ws = dalloc<float>(lm, colsum_workspace_floats(R, widest), &err);
  lm->emb_scratch = dalloc<uint8_t>(lm, embedding_scratch_bytes(R, V), &err);
  lm->epi_ws = dalloc<float>(lm, gemm_epilogue_ws_floats((int)R, (int)F), &err);
  lm->qkv_colrows = (int64_t)lm->B * ((lm->T + 127) / 128);
  lm->qkv_colpart = dalloc<float>(lm, (size_t)lm->qkv_colrows * 3 * d, &err);
  // split-K partials for the weight-gradient GEMMs of the layers (K = rows)
  lm->splitk_floats = gemm_splitk_floats((int)std::max<int64_t>(3 * d, F), (int)std::max<int64_t>(d, F));
  lm->splitk_ws = dalloc<float>(lm, lm->splitk_floats, &err);
  lm->chunk_ws_floats = gemm_chunk_ws_floats();
  lm->chunk_ws = dalloc<float>(lm, lm->chunk_ws_floats, &err);
  {
    AttnParams shape{};
    shape.B = (int)lm->B; shape.Hq = (int)lm->H; shape.Hkv = (int)lm->H;
    shape.Tq = (int)lm->T; shape.Tk = (int)lm->T; shape.Dh = (int)lm->Dh;
    lm->attn_qkv_ws.resize(L);
    lm->attn_prepared.assign(L, 0);
    for (int64_t l = 0; l < L; l++)
      lm->attn_qkv_ws[l] = dalloc<float>(lm, attention_qkv_workspace_floats(shape), &err);
    lm->attn_grad_ws = dalloc<float>(lm, attention_grad_workspace_floats(shape), &err);
  }
  lm->ids = dalloc<int64_t>(lm, R, &err);
  lm->targets = dalloc<int64_t>(lm, R, &err);
  lm->loss_mask = dalloc<uint8_t>(lm, R, &err);
  lm->upstream = dalloc<float>(lm, R, &err);
  lm->pos = dalloc<int64_t>(lm, R, &err);
  lm->rope_cos = dalloc<float>(lm, lm->T * lm->Dh / 2, &err);
  lm->rope_sin = dalloc<float>(lm, lm->T * lm->Dh / 2, &err);
  lm->status = dalloc<int>(lm, 4, &err);
  lm->d_completed = dalloc<uint64_t>(lm, 1, &err);
  if (err != cudaSuccess) {
    et_b200_lm_destroy_v1(&lm);
    return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_ALLOCATION_FAILED, op,
                     "device memory for the model and activations is insufficient");
  }
  // positions 0..T-1 per sequence; RoPE tables from libm on the host
  std::vector<int64_t> pos(R);
  for (int64_t b = 0; b < lm->B; b++)
    for (int64_t t = 0; t < lm->T; t++) pos[b * lm->T + t] = t;
  const int64_t half = lm->Dh / 2;
  std::vector<float> inv(half), ct(lm->T * half), st(lm->T * half);
  for (int64_t i = 0; i < half; i++)
    inv[i] = (float)(1.0 / pow(c->rope_base, (double)(2 * i) / (double)lm->Dh));
  for (int64_t t = 0; t < lm->T; t++)
    for (int64_t i = 0; i < half; i++) {
      volatile float angle = (float)t * inv[i];
      ct[t * half + i] = cosf(angle);
      st[t * half + i] = sinf(angle);
    }
  const uint64_t prefix[2] = {0, lm->P};
  cudaMemcpy(lm->pos, pos.data(), R * sizeof(int64_t), cudaMemcpyHostToDevice);
  cudaMemcpy(lm->rope_cos, ct.data(), ct.size() * sizeof(float), cudaMemcpyHostToDevice);
  cudaMemcpy(lm->rope_sin, st.data(), st.size() * sizeof(float), cudaMemcpyHostToDevice);
  cudaMemcpy(lm->d_prefix, prefix, sizeof(prefix), cudaMemcpyHostToDevice);
  cudaMemset(lm->params, 0, lm->P * sizeof(float));
  cudaMemset(lm->grads, 0, (lm->P + 8) * sizeof(float));
  if (lm->f16) {
    cudaMemset(lm->sexp, 0, lm->nslots * sizeof(int));
    cudaMemset(lm->samax, 0, lm->nslots * sizeof(unsigned));
  }
  cudaMemset(lm->m1, 0, lm->P * sizeof(float));
  cudaMemset(lm->m2, 0, lm->P * sizeof(float));
  cudaMemset(lm->status, 0, 4 * sizeof(int));
  cudaMemset(lm->d_completed, 0, sizeof(uint64_t));
  lm->layer_done.resize(L);
  for (auto& ev : lm->layer_done) cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  cudaEventCreateWithFlags(&lm->tail_done, cudaEventDisableTiming);
  cudaEventCreateWithFlags(&lm->comm_done, cudaEventDisableTiming);
  err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    et_b200_lm_destroy_v1(&lm);
    return cuda_error(e, err, op);
  }
  *out = lm;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

void et_b200_lm_destroy_v1(et_b200_lm** slot) {
  if (slot == nullptr || *slot == nullptr) return;
  et_b200_lm* lm = *slot;
  cudaSetDevice(lm->device);
  if (lm->stream) cudaStreamSynchronize(lm->stream);
  if (lm->comm) cudaStreamSynchronize(lm->comm);
  if (lm->nccl_comm && nccl().ok) nccl().CommDestroy(lm->nccl_comm);
  for (void* p : lm->allocations) cudaFree(p);
  for (auto& ev : lm->layer_done) cudaEventDestroy(ev);
  if (lm->tail_done) cudaEventDestroy(lm->tail_done);
  if (lm->comm_done) cudaEventDestroy(lm->comm_done);
  for (auto& m : lm->marks) {
    cudaEventDestroy(m.start);
    cudaEventDestroy(m.stop);
  }
  if (lm->stream) cudaStreamDestroy(lm->stream);
  if (lm->comm) cudaStreamDestroy(lm->comm);
  delete lm;
  *slot = nullptr;
}

size_t et_b200_lm_tensor_count_v1(const et_b200_lm* lm) { return lm ? lm->sz.size() : 0; }

size_t et_b200_lm_parameter_count_v1(const et_b200_lm* lm) {
  if (!lm) return 0;
  size_t n = 0;
  for (size_t s : lm->sz) n += s;
  return n;
}

int32_t et_b200_lm_tensor_sizes_v1(const et_b200_lm* lm, size_t* sizes) {
  if (!lm || !sizes) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  for (size_t i = 0; i < lm->sz.size(); i++) sizes[i] = lm->sz[i];
  return 0;
}

// Host copies use the packed order (tensor after tensor, no alignment gaps).
static int32_t transfer(et_b200_lm* lm, int32_t which, float* host, const float* src_host,
                        size_t count, et_kernel_error* e, bool to_device) {
  const char* op = to_device ? "lm-write" : "lm-read";
  if (check_ready(lm, e, op)) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  float* base = which == 0 ? lm->params : which == 1 ? lm->grads : which == 2 ? lm->m1 :
                which == 3 ? lm->m2 : nullptr;
  if (base == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_ENUM, op, "unknown buffer selector");
  if (count != et_b200_lm_parameter_count_v1(lm))
    return set_error(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_BUFFER_TOO_SMALL, op, "count must equal the parameter count");
  cudaStreamSynchronize(lm->stream);
  size_t packed = 0;
  for (size_t t = 0; t < lm->sz.size(); t++) {
    cudaError_t st = to_device
        ? cudaMemcpy(base + lm->off[t], src_host + packed, lm->sz[t] * 4, cudaMemcpyHostToDevice)
        : cudaMemcpy(host + packed, base + lm->off[t], lm->sz[t] * 4, cudaMemcpyDeviceToHost);
    if (st != cudaSuccess) return cuda_error(e, st, op);
    packed += lm->sz[t];
  }
  if (to_device && which == 0) {
    refresh_weight_split(lm);
    lm->calibrated = false;  // new weights: the next split-f16 step re-measures the scales
  }
  cudaError_t st = cudaStreamSynchronize(lm->stream);
  if (st != cudaSuccess) return cuda_error(e, st, op);
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_lm_read_v1(et_b200_lm* lm, int32_t which, float* host, size_t count,
                           et_kernel_error* e) {
  return transfer(lm, which, host, nullptr, count, e, false);
}

int32_t et_b200_lm_write_v1(et_b200_lm* lm, int32_t which, const float* host, size_t count,
                            et_kernel_error* e) {
  return transfer(lm, which, nullptr, host, count, e, true);
}

int32_t et_b200_lm_init_v1(et_b200_lm* lm, uint64_t seed, et_kernel_error* e) {
  if (check_ready(lm, e, "lm-init")) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  const size_t n = et_b200_lm_parameter_count_v1(lm);
  std::vector<float> host(n);
  size_t packed = 0;
  const size_t count = lm->sz.size();
  for (size_t t = 0; t < count; t++) {
    int kind;  // 0 weight N(0, 0.02), 1 gamma, 2 zero
    if (t == 0) kind = 0;
    else if (t >= count - 2) kind = (t == count - 2) ? 1 : 2;
    else {
      const size_t j = (t - 1) % kPerLayer;
      kind = (j == T_LN1G || j == T_LN2G) ? 1
             : (j == T_WQKV || j == T_WO || j == T_W1 || j == T_W2) ? 0 : 2;
    }
    if (kind == 0) et_b200_fill_normal_v1(seed, t, lm->sz[t], 0.0, 0.02, host.data() + packed);
    else
      for (size_t i = 0; i < lm->sz[t]; i++) host[packed + i] = kind == 1 ? 1.0f : 0.0f;
    packed += lm->sz[t];
  }
  cudaStreamSynchronize(lm->stream);
  lm->updates = 0;
  cudaMemset(lm->d_completed, 0, sizeof(uint64_t));
  cudaMemset(lm->m1, 0, lm->P * sizeof(float));
  cudaMemset(lm->m2, 0, lm->P * sizeof(float));
  return et_b200_lm_write_v1(lm, 0, host.data(), n, e);
}

static int32_t stage_tokens(et_b200_lm* lm, const int64_t* ids, const int64_t* targets,
                            cudaMemcpyKind kind) {
  cudaMemcpyAsync(lm->ids, ids, lm->R * sizeof(int64_t), kind, lm->stream);
  cudaMemcpyAsync(lm->targets, targets, lm->R * sizeof(int64_t), kind, lm->stream);
  return 0;
}

int32_t et_b200_lm_step_device_v1(et_b200_lm* lm, const int64_t* device_ids,
                                  const int64_t* device_targets, float* device_loss,
                                  et_kernel_error* e) {
  if (check_ready(lm, e, "lm-step")) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  if (device_ids == nullptr || device_targets == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, "lm-step", "ids and targets are required");
  if (device_ids != lm->ids) stage_tokens(lm, device_ids, device_targets, cudaMemcpyDeviceToDevice);
  begin_step(lm);
  forward(lm);
  backward(lm);
  optimizer_step(lm);
  if (lm->f16) lm->calibrated = true;  // (a failed operand check is reported by the next host call)
  if (device_loss)
    cudaMemcpyAsync(device_loss, lm->loss_mean, sizeof(float), cudaMemcpyDeviceToDevice, lm->stream);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return cuda_error(e, st, "lm-step");
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_lm_step_v1(et_b200_lm* lm, const int64_t* host_ids, const int64_t* host_targets,
                           float* host_loss, et_kernel_error* e) {
  if (check_ready(lm, e, "lm-step")) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  if (host_ids == nullptr || host_targets == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, "lm-step", "ids and targets are required");
  stage_tokens(lm, host_ids, host_targets, cudaMemcpyHostToDevice);
  return run_host_step(lm, true, host_loss, e, "lm-step");
}

int32_t et_b200_lm_forward_backward_v1(et_b200_lm* lm, const int64_t* host_ids,
                                       const int64_t* host_targets, float* host_loss,
                                       et_kernel_error* e) {
  if (check_ready(lm, e, "lm-forward-backward")) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  if (host_ids == nullptr || host_targets == nullptr)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, "lm-forward-backward", "ids and targets are required");
  stage_tokens(lm, host_ids, host_targets, cudaMemcpyHostToDevice);
  return run_host_step(lm, false, host_loss, e, "lm-forward-backward");
}

int32_t et_b200_lm_set_loss_mask_v1(et_b200_lm* lm, const uint8_t* mask, int32_t on_device,
                                    et_kernel_error* e) {
  const char* op = "lm-loss-mask";
  if (check_ready(lm, e, op)) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  if (mask == nullptr) {
    lm->masked = false;
    if (e) memset(e, 0, sizeof(*e));
    return 0;
  }
  if (!on_device) {
    // the L3S rule (l3s_masked_objective_provider.c:130-134): bytes are 0 or 1
    for (int64_t i = 0; i < lm->R; i++)
      if (mask[i] > 1)
        return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                         "loss mask byte other than 0 or 1");
  }
  // ordered on the model's stream after every step enqueued before it
  cudaMemcpyAsync(lm->loss_mask, mask, (size_t)lm->R, on_device ? cudaMemcpyDeviceToDevice
                                                                : cudaMemcpyHostToDevice,
                  lm->stream);
  if (!on_device) {
    const cudaError_t st = cudaStreamSynchronize(lm->stream);  // the host buffer is the caller's
    if (st != cudaSuccess) return cuda_error(e, st, op);
  }
  lm->masked = true;
  const cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return cuda_error(e, st, op);
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

void* et_b200_lm_stream_v1(et_b200_lm* lm) { return lm ? (void*)lm->stream : nullptr; }

int32_t et_b200_nccl_unique_id_v1(uint8_t unique_id[128], et_kernel_error* e) {
  if (!nccl().ok)
    return set_error(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_SYMBOL_MISSING, "nccl-id", "libnccl.so.2 is not available");
  ncclUniqueId id;
  if (nccl().GetUniqueId(&id) != ncclSuccess)
    return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_PROVIDER_REJECTED, "nccl-id", "ncclGetUniqueId failed");
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  memcpy(unique_id, &id, 128);
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_lm_enable_data_parallel_v1(et_b200_lm* lm, const uint8_t unique_id[128],
                                           int32_t rank, int32_t world, et_kernel_error* e) {
  const char* op = "lm-data-parallel";
  if (check_ready(lm, e, op)) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  if (world < 1 || rank < 0 || rank >= world)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_SHAPE, op, "rank must lie in [0, world)");
  if (world == 1) {
    lm->dp = false;
    return 0;
  }
  if (!nccl().ok)
    return set_error(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_SYMBOL_MISSING, op, "libnccl.so.2 is not available");
  ncclUniqueId id;
  memcpy(&id, unique_id, 128);
  ncclResult_t r = nccl().CommInitRank(&lm->nccl_comm, world, id, rank);
  if (r != ncclSuccess) {
    char msg[160];
    snprintf(msg, sizeof(msg), "ncclCommInitRank failed: %s",
             nccl().GetErrorString ? nccl().GetErrorString(r) : "?");
    return set_error(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_PROVIDER_REJECTED, op, msg);
  }
  lm->rank = rank;
  lm->world = world;
  lm->dp = true;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

// Profiling: when enabled, every launch group of a step is bracketed by CUDA
// events on the model's stream.  et_b200_lm_profile_read_v1 returns, per
// class, {launch groups, milliseconds, algorithmic FLOP, algorithmic bytes}.
int32_t et_b200_lm_profile_v1(et_b200_lm* lm, int32_t enable) {
  if (!lm) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  lm->profile = enable != 0;
  memset(lm->prof, 0, sizeof(lm->prof));
  lm->mark_used = 0;
  return 0;
}

int32_t et_b200_lm_profile_collect_v1(et_b200_lm* lm) {
  if (!lm) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  collect_profile(lm);
  return 0;
}

int32_t et_b200_lm_f16_redone_steps_v1(const et_b200_lm* lm) {
  return lm ? lm->redone_steps : 0;
}

int32_t et_b200_lm_update_counts_v1(et_b200_lm* lm, uint64_t* completed, uint64_t* skipped,
                                    et_kernel_error* e) {
  const char* op = "lm-update-counts";
  if (check_ready(lm, e, op)) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  uint64_t done = 0;
  int pending = 0;
  cudaMemcpyAsync(&done, lm->d_completed, sizeof(done), cudaMemcpyDeviceToHost, lm->stream);
  cudaMemcpyAsync(&pending, lm->status + 2, sizeof(int), cudaMemcpyDeviceToHost, lm->stream);
  cudaMemsetAsync(lm->status + 2, 0, sizeof(int), lm->stream);
  cudaError_t st = cudaStreamSynchronize(lm->stream);
  if (st != cudaSuccess) return cuda_error(e, st, op);
  lm->updates = done;
  lm->skipped += (uint64_t)pending;
  if (pending != 0 && lm->f16) lm->calibrated = false;
  if (completed) *completed = lm->updates;
  if (skipped) *skipped = lm->skipped;
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t et_b200_lm_profile_read_v1(et_b200_lm* lm, double* out, size_t count) {
  if (!lm || !out || count < (size_t)P_COUNT * 4) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  memcpy(out, lm->prof, sizeof(lm->prof));
  return 0;
}

}  // extern "C"
