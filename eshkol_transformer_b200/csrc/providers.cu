// K1 providers: drop-in replacements for the reference's A2, N2, N3K and L2
// providers (native/a2_attention_provider.c, native/n2_primitives_provider.c,
// native/n3k_primitives_provider.c, native/indexed_cross_entropy.c).
//
// Two-phase contract (native/kernel_abi.c:1287-1324): validate_call checks
// every view and the numerical domain and returns the error category; it then
// runs the operation into provider scratch and rejects a nonfinite result,
// exactly as the reference's preflight does, so invoke_call cannot fail and a
// rejected call leaves the caller's outputs untouched.  invoke_call computes
// into the outputs and returns with the results complete.
//
// Views on device "cuda" are device pointers used in place; views on device
// "cpu" are host pointers staged through provider scratch.  Scratch is a
// per-device pool that grows on demand and is kept between calls.  Calls are
// not thread-safe (the reference's providers are not either).
#include <math.h>

#include <mutex>
#include <string>
#include <vector>

#include "ops.cuh"

using namespace etb;

namespace {

// ---------------------------------------------------------------- scratch pool

struct Pool {
  std::vector<std::pair<uint8_t*, size_t>> chunks;
  size_t chunk = 0, used = 0;
  cudaStream_t stream = nullptr;
  int* flag = nullptr;
  void reset() { chunk = 0; used = 0; }
  void* alloc(size_t bytes) {
    bytes = (bytes + 255) & ~(size_t)255;
    if (bytes == 0) bytes = 256;
    while (chunk < chunks.size()) {
      if (used + bytes <= chunks[chunk].second) {
        void* p = chunks[chunk].first + used;
        used += bytes;
        return p;
      }
      chunk++;
      used = 0;
    }
    const size_t size = bytes > ((size_t)256 << 20) ? bytes : ((size_t)256 << 20);
    uint8_t* p = nullptr;
    if (cudaMalloc(&p, size) != cudaSuccess) return nullptr;
    chunks.push_back({p, size});
    chunk = chunks.size() - 1;
    used = bytes;
    return p;
  }
};

Pool& pool() {
  static std::mutex mu;
  static std::vector<Pool*> pools;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if ((int)pools.size() <= dev) pools.resize(dev + 1, nullptr);
  if (pools[dev] == nullptr) {
    pools[dev] = new Pool();
    cudaStreamCreateWithFlags(&pools[dev]->stream, cudaStreamNonBlocking);
    cudaMalloc(&pools[dev]->flag, 4 * sizeof(int));
  }
  return *pools[dev];
}

uint32_t g_precision = ET_B200_PRECISION_TF32X3;

// ---------------------------------------------------------------- view helpers

bool text_is(const char* a, const char* b) { return a != nullptr && strcmp(a, b) == 0; }

const et_kernel_tensor_view_v1* view_at(const void* base, size_t stride, size_t i) {
  return reinterpret_cast<const et_kernel_tensor_view_v1*>(static_cast<const uint8_t*>(base) +
                                                           i * stride);
}

struct Spec {
  const char* dtype;
  size_t rank;
  uint64_t shape[6];
};

size_t dtype_bytes(const char* d) {
  if (text_is(d, "f32")) return 4;
  if (text_is(d, "i64")) return 8;
  if (text_is(d, "bool")) return 1;
  return 0;
}

struct Call {
  const et_kernel_call_v1* call = nullptr;
  const char* op = "";
  bool host = false;
  std::vector<const et_kernel_tensor_view_v1*> in, out;
};

int32_t fail(et_kernel_error* e, uint32_t cat, uint32_t code, const char* op, const char* msg) {
  return set_error(e, cat, code, op, msg);
}

// Common structure checks shared by every operation: tensor tables, device,
// dtype, density, shape and byte spans of each view.
int32_t check_tables(const et_kernel_call_v1* c, const char* op, size_t nin, size_t nout,
                     const Spec* ins, const Spec* outs, Call* out, et_kernel_error* e) {
  if (c->input_count != nin || c->output_count != nout || c->inputs == nullptr ||
      (nout > 0 && c->outputs == nullptr))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor count does not match the operation");
  if (c->input_stride < ET_KERNEL_TENSOR_VIEW_V1_0_SIZE ||
      (nout > 0 && c->output_stride < ET_KERNEL_TENSOR_VIEW_V1_0_SIZE))
    return fail(e, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_INVALID_STRUCT_SIZE, op,
                "tensor table stride truncates the K1 v1 prefix");
  if (c->input_bytes != nin * c->input_stride || c->output_bytes != nout * c->output_stride)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor table span is invalid");
  out->call = c;
  out->op = op;
  out->host = text_is(c->request->device, "cpu");
  if (!out->host && !text_is(c->request->device, "cuda"))
    return fail(e, ET_KERNEL_ERROR_DEVICE_MISMATCH, ET_KERNEL_CODE_INVALID_TEXT, op,
                "B200 kernels accept cpu or cuda tensor views");
  for (size_t k = 0; k < nin + nout; k++) {
    const bool is_out = k >= nin;
    const et_kernel_tensor_view_v1* v = is_out ? view_at(c->outputs, c->output_stride, k - nin)
                                               : view_at(c->inputs, c->input_stride, k);
    const Spec& s = is_out ? outs[k - nin] : ins[k];
    if (v->struct_size < ET_KERNEL_TENSOR_VIEW_V1_0_SIZE)
      return fail(e, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_INVALID_STRUCT_SIZE, op,
                  "tensor descriptor is truncated");
    if (!text_is(v->dtype, s.dtype))
      return fail(e, ET_KERNEL_ERROR_DTYPE_MISMATCH, ET_KERNEL_CODE_INVALID_TEXT, op,
                  "tensor dtype does not match the operation schema");
    if (!text_is(v->device, c->request->device))
      return fail(e, ET_KERNEL_ERROR_DEVICE_MISMATCH, ET_KERNEL_CODE_INVALID_TEXT, op,
                  "tensor device differs from the request device");
    if (v->layout != ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR || v->offset_bytes != 0)
      return fail(e, ET_KERNEL_ERROR_NONCONTIGUOUS, ET_KERNEL_CODE_INVALID_BUFFER, op,
                  "tensors must be dense zero-offset views");
    if (v->rank != s.rank || (s.rank > 0 && v->shape == nullptr))
      return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                  "tensor rank does not match the operation schema");
    uint64_t elems = 1;
    for (size_t i = 0; i < s.rank; i++) {
      if (v->shape[i] != s.shape[i])
        return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                    "tensor extent does not match the operation schema");
      elems *= s.shape[i];
    }
    const size_t eb = dtype_bytes(s.dtype);
    if (v->byte_length != elems * eb || (elems > 0 && v->data == nullptr) ||
        (reinterpret_cast<uintptr_t>(v->data) % eb) != 0)
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                  "tensor data alignment or byte span is invalid");
    (is_out ? out->out : out->in).push_back(v);
  }
  // outputs must be disjoint from inputs and from each other (K1 generic rule)
  auto overlap = [](const et_kernel_tensor_view_v1* a, const et_kernel_tensor_view_v1* b) {
    if (a->byte_length == 0 || b->byte_length == 0) return false;
    const uintptr_t a0 = (uintptr_t)a->data, b0 = (uintptr_t)b->data;
    return a0 < b0 + b->byte_length && b0 < a0 + a->byte_length;
  };
  for (size_t i = 0; i < out->out.size(); i++) {
    for (auto* v : out->in)
      if (overlap(out->out[i], v))
        return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                    "output storage aliases borrowed input storage");
    for (size_t j = 0; j < i; j++)
      if (overlap(out->out[i], out->out[j]))
        return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                    "output storage aliases another output");
  }
  // "cuda" views are borrowed like host memory: the call reads them once
  // every kernel and copy already enqueued on the device, on any stream, has
  // finished (the caller may have produced them on its own stream just
  // before the call; the provider's stream is not ordered after it).
  if (!out->host) {
    const cudaError_t st = cudaDeviceSynchronize();
    if (st != cudaSuccess) return cuda_error(e, st, op);
  }
  return 0;
}

// Device pointer of an input view (host views are copied into scratch).
const void* dev_in(Call& cl, size_t i) {
  const et_kernel_tensor_view_v1* v = cl.in[i];
  if (!cl.host) return v->data;
  Pool& P = pool();
  void* p = P.alloc(v->byte_length);
  if (p && v->byte_length)
    cudaMemcpyAsync(p, v->data, v->byte_length, cudaMemcpyHostToDevice, P.stream);
  return p;
}

// Device pointer an output is computed into: scratch in the preflight and for
// host views, the caller's buffer otherwise.
void* dev_out(Call& cl, size_t i, bool scratch) {
  const et_kernel_tensor_view_v1* v = cl.out[i];
  if (!cl.host && !scratch) return v->data;
  return pool().alloc(v->byte_length);
}

// Host copy of a small input (positions, epsilon, inverse frequencies).
template <typename T>
std::vector<T> host_copy(Call& cl, size_t i) {
  const et_kernel_tensor_view_v1* v = cl.in[i];
  std::vector<T> h(v->byte_length / sizeof(T));
  if (h.empty()) return h;
  if (cl.host) memcpy(h.data(), v->data, v->byte_length);
  else cudaMemcpy(h.data(), v->data, v->byte_length, cudaMemcpyDeviceToHost);
  return h;
}

bool inputs_finite(Call& cl, std::initializer_list<size_t> idx) {
  Pool& P = pool();
  for (size_t i : idx) {
    const et_kernel_tensor_view_v1* v = cl.in[i];
    const size_t n = v->byte_length / 4;
    if (cl.host) {
      const float* f = static_cast<const float*>(v->data);
      for (size_t k = 0; k < n; k++)
        if (!isfinite(f[k])) return false;
    } else {
      int flag = 0;
      cudaMemsetAsync(P.flag, 0, sizeof(int), P.stream);
      check_finite(static_cast<const float*>(v->data), n, P.flag, P.stream);
      cudaMemcpyAsync(&flag, P.flag, sizeof(int), cudaMemcpyDeviceToHost, P.stream);
      cudaStreamSynchronize(P.stream);
      if (flag) return false;
    }
  }
  return true;
}

bool device_finite(const float* p, size_t n) {
  Pool& P = pool();
  int flag = 0;
  cudaMemsetAsync(P.flag, 0, sizeof(int), P.stream);
  check_finite(p, n, P.flag, P.stream);
  cudaMemcpyAsync(&flag, P.flag, sizeof(int), cudaMemcpyDeviceToHost, P.stream);
  cudaStreamSynchronize(P.stream);
  return flag == 0;
}

// Copies device results to host outputs (host views) and waits.  The kernel
// ABI's invoke returns nothing, so a CUDA error raised by this call's
// launches, or a device-side wait that timed out, is reported on stderr and
// the outputs are filled with NaN rather than left holding stale memory.
void finish(Call& cl, const std::vector<void*>& outs) {
  Pool& P = pool();
  // a launch error, or a bounded device-side wait that gave up (the device
  // error word), fails the call loudly
  int word = 0;
  cudaMemcpyAsync(&word, device_error_word(), sizeof(int), cudaMemcpyDeviceToHost, P.stream);
  cudaStreamSynchronize(P.stream);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess || word != 0) {
    if (st != cudaSuccess)
      fprintf(stderr, "et_b200: CUDA error in a kernel call: %s\n", cudaGetErrorString(st));
    else
      fprintf(stderr, "et_b200: a kernel gave up a bounded wait (error word 0x%x)\n", word);
    cudaMemsetAsync(device_error_word(), 0, sizeof(int), P.stream);
    for (size_t i = 0; i < cl.out.size() && i < outs.size(); i++)
      if (cl.out[i]->byte_length && outs[i] != nullptr)
        cudaMemsetAsync(outs[i], 0xff, cl.out[i]->byte_length, P.stream);  // all-ones: NaN
  }
  if (cl.host)
    for (size_t i = 0; i < cl.out.size(); i++)
      if (cl.out[i]->byte_length)
        cudaMemcpyAsync(cl.out[i]->data, outs[i], cl.out[i]->byte_length, cudaMemcpyDeviceToHost,
                        P.stream);
  cudaStreamSynchronize(P.stream);
}

bool request_shape(const et_kernel_call_v1* c, size_t rank, uint64_t* dims) {
  if (c->request->rank != rank || c->request->shape == nullptr) return false;
  for (size_t i = 0; i < rank; i++) {
    dims[i] = c->request->shape[i];
    if (dims[i] == 0 || dims[i] > ((uint64_t)1 << 31)) return false;
  }
  return true;
}

int32_t common_request(const et_kernel_call_v1* c, const char* capability, const char* op,
                       et_kernel_error* e) {
  if (c == nullptr || c->request == nullptr || c->request->operation == nullptr)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, "b200.provider",
                "call, request, and operation are required");
  if (c->struct_size < ET_KERNEL_CALL_V1_0_SIZE || c->request->struct_size < ET_KERNEL_REQUEST_V1_0_SIZE)
    return fail(e, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_INVALID_STRUCT_SIZE, op,
                "call or request truncates the K1 v1 prefix");
  if (!text_is(c->capability, capability) || !text_is(c->request->dtype, "f32") ||
      !(text_is(c->request->device, "cpu") || text_is(c->request->device, "cuda")))
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "request is outside this provider's capabilities");
  return 0;
}

int32_t preflight_fail(et_kernel_error* e, const char* op) {
  return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
              "operation would produce a nonfinite result");
}

// ============================================================== A2 attention

struct AttShape {
  uint64_t n, hq, hkv, tq, tk, dh;
};

int32_t attention_checks(const et_kernel_call_v1* c, bool backward, Call& cl, AttShape& s,
                         et_kernel_error* e) {
  const char* op = backward ? "causal-attention.backward" : "causal-attention.forward";
  int32_t r = common_request(c, "kernel.causal-attention", op, e);
  if (r) return r;
  uint64_t d[6];
  if (!text_is(c->request->operation, op) || !request_shape(c, 6, d))
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "attention request is outside this provider's capabilities");
  s = AttShape{d[0], d[1], d[2], d[3], d[4], d[5]};
  if (s.hkv < 2 || s.hq < s.hkv || s.hq % s.hkv != 0)
    return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "attention requires Hkv>=2 and Hq divisible by Hkv");
  if (s.dh > 128)
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "head dimension above 128 is unsupported");
  const Spec q{"f32", 4, {s.n, s.hq, s.tq, s.dh}}, kv{"f32", 4, {s.n, s.hkv, s.tk, s.dh}};
  const Spec qp{"i64", 2, {s.n, s.tq}}, kp{"i64", 2, {s.n, s.tk}};
  const Spec mk{"bool", 3, {s.n, s.tq, s.tk}};
  const Spec ins[7] = {q, kv, kv, qp, kp, mk, q};
  const Spec outs[3] = {q, kv, kv};
  r = check_tables(c, op, backward ? 7 : 6, backward ? 3 : 1, ins, outs, &cl, e);
  if (r) return r;
  {
    const et_kernel_tensor_view_v1 *k = cl.in[1], *v = cl.in[2];
    const uintptr_t k0 = (uintptr_t)k->data, v0 = (uintptr_t)v->data;
    if (k->byte_length && v->byte_length && k0 < v0 + v->byte_length && v0 < k0 + k->byte_length)
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                  "attention key and value storage must be distinct");
  }
  if (!inputs_finite(cl, {0, 1, 2}) || (backward && !inputs_finite(cl, {6})))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "attention floating inputs must be finite");
  for (size_t which = 3; which <= 4; which++) {
    auto pos = host_copy<int64_t>(cl, which);
    const uint64_t t = which == 3 ? s.tq : s.tk;
    for (uint64_t b = 0; b < s.n; b++) {
      int64_t prev = -1;
      for (uint64_t i = 0; i < t; i++) {
        const int64_t p = pos[b * t + i];
        if (p < 0 || p > INT64_C(16777215) || p <= prev)
          return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                      "attention positions must be strictly increasing and exact");
        prev = p;
      }
    }
  }
  {
    auto mask = host_copy<uint8_t>(cl, 5);
    for (uint8_t m : mask)
      if (m > 1)
        return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                    "attention bool mask contains a noncanonical value");
  }
  return 0;
}

AttnParams attention_params(const AttShape& s, const float* q, const float* k, const float* v,
                            const int64_t* qp, const int64_t* kp, const uint8_t* mask) {
  AttnParams p{};
  p.B = (int)s.n; p.Hq = (int)s.hq; p.Hkv = (int)s.hkv;
  p.Tq = (int)s.tq; p.Tk = (int)s.tk; p.Dh = (int)s.dh;
  volatile float root = sqrtf((float)s.dh);
  p.scale = 1.0f / root;
  p.q = AttnTensor{q, (int64_t)(s.hq * s.tq * s.dh), (int64_t)(s.tq * s.dh), (int64_t)s.dh};
  p.k = AttnTensor{k, (int64_t)(s.hkv * s.tk * s.dh), (int64_t)(s.tk * s.dh), (int64_t)s.dh};
  p.v = AttnTensor{v, (int64_t)(s.hkv * s.tk * s.dh), (int64_t)(s.tk * s.dh), (int64_t)s.dh};
  p.qpos = qp; p.kpos = kp; p.mask = mask;
  return p;
}

void run_attention(Call& cl, const AttShape& s, bool backward, bool scratch,
                   std::vector<void*>& outs) {
  Pool& P = pool();
  const float* q = (const float*)dev_in(cl, 0);
  const float* k = (const float*)dev_in(cl, 1);
  const float* v = (const float*)dev_in(cl, 2);
  const int64_t* qp = (const int64_t*)dev_in(cl, 3);
  const int64_t* kp = (const int64_t*)dev_in(cl, 4);
  const uint8_t* mask = (const uint8_t*)dev_in(cl, 5);
  AttnParams p = attention_params(s, q, k, v, qp, kp, mask);
  p.ws = (float*)P.alloc(attention_workspace_floats(p) * 4);
  const size_t rows = s.n * s.hq * s.tq;
  float* m = (float*)P.alloc(rows * 4);
  float* l = (float*)P.alloc(rows * 4);
  const int64_t qsb = s.hq * s.tq * s.dh, qsh = s.tq * s.dh, kvsb = s.hkv * s.tk * s.dh,
                kvsh = s.tk * s.dh;
  if (!backward) {
    float* o = (float*)dev_out(cl, 0, scratch);
    outs = {o};
    attention_forward(p, AttnOut{o, qsb, qsh, (int64_t)s.dh}, m, l, P.stream);
    return;
  }
  const float* dout = (const float*)dev_in(cl, 6);
  float* o = (float*)P.alloc(rows * s.dh * 4);
  const bool prepared = attention_forward(p, AttnOut{o, qsb, qsh, (int64_t)s.dh}, m, l, P.stream);
  float* dq = (float*)dev_out(cl, 0, scratch);
  float* dk = (float*)dev_out(cl, 1, scratch);
  float* dv = (float*)dev_out(cl, 2, scratch);
  outs = {dq, dk, dv};
  float* delta = (float*)P.alloc(rows * 4);
  p.ws_ready = prepared ? 1 : 0;  // the forward above prepared Q/K/V in p.ws
  attention_backward(p, AttnTensor{o, qsb, qsh, (int64_t)s.dh}, nullptr,
                     AttnTensor{dout, qsb, qsh, (int64_t)s.dh}, m, l, delta,
                     AttnOut{dq, qsb, qsh, (int64_t)s.dh}, AttnOut{dk, kvsb, kvsh, (int64_t)s.dh},
                     AttnOut{dv, kvsb, kvsh, (int64_t)s.dh}, P.stream);
}

// ---- RoPE ----

struct RopeShape {
  uint64_t n, h, t, dh;
};

int32_t rope_checks(const et_kernel_call_v1* c, bool backward, Call& cl, RopeShape& s,
                    et_kernel_error* e) {
  const char* op = backward ? "rope.backward" : "rope.forward";
  int32_t r = common_request(c, "kernel.rope", op, e);
  if (r) return r;
  uint64_t d[4];
  if (!text_is(c->request->operation, op) || !request_shape(c, 4, d))
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "RoPE request is outside this provider's capabilities");
  s = RopeShape{d[0], d[1], d[2], d[3]};
  if (s.dh < 2 || s.dh % 2 != 0)
    return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "RoPE requires an even head dimension of at least two");
  const Spec x{"f32", 4, {s.n, s.h, s.t, s.dh}};
  const Spec ins[3] = {x, {"i64", 2, {s.n, s.t}}, {"f32", 1, {s.dh / 2}}};
  r = check_tables(c, op, 3, 1, ins, &x, &cl, e);
  if (r) return r;
  auto pos = host_copy<int64_t>(cl, 1);
  bool ok = inputs_finite(cl, {0});
  for (uint64_t b = 0; ok && b < s.n; b++) {
    int64_t prev = -1;
    for (uint64_t i = 0; i < s.t; i++) {
      const int64_t p = pos[b * s.t + i];
      if (p < 0 || p > INT64_C(16777215) || p <= prev) { ok = false; break; }
      prev = p;
    }
  }
  if (!ok)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "RoPE inputs or positions are outside the finite exact domain");
  auto inv = host_copy<float>(cl, 2);
  for (float f : inv)
    if (!isfinite(f) || f <= 0.0f)
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                  "RoPE inverse frequencies must be positive and finite");
  return 0;
}

void run_rope(Call& cl, const RopeShape& s, bool backward, bool scratch, std::vector<void*>& outs) {
  Pool& P = pool();
  auto pos = host_copy<int64_t>(cl, 1);
  auto inv = host_copy<float>(cl, 2);
  const uint64_t half = s.dh / 2;
  std::vector<float> ct(s.n * s.t * half), st(s.n * s.t * half);
  for (uint64_t r = 0; r < s.n * s.t; r++)
    for (uint64_t i = 0; i < half; i++) {
      volatile float angle = (float)pos[r] * inv[i];
      ct[r * half + i] = cosf(angle);
      st[r * half + i] = sinf(angle);
    }
  float* dct = (float*)P.alloc(ct.size() * 4);
  float* dst = (float*)P.alloc(st.size() * 4);
  cudaMemcpyAsync(dct, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice, P.stream);
  cudaMemcpyAsync(dst, st.data(), st.size() * 4, cudaMemcpyHostToDevice, P.stream);
  const float* x = (const float*)dev_in(cl, 0);
  float* y = (float*)dev_out(cl, 0, scratch);
  outs = {y};
  rope_apply(x, y, dct, dst, s.n, s.h, s.t, s.dh, backward ? 1 : 0, P.stream);
  // the host tables must outlive the asynchronous copies
  cudaStreamSynchronize(P.stream);
}

int32_t a2_validate(const et_kernel_call_v1* c, et_kernel_error* e) {
  if (c == nullptr || c->request == nullptr || c->request->operation == nullptr)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, "a2.provider",
                "call, request, and operation are required");
  const char* opn = c->request->operation;
  Call cl;
  std::vector<void*> outs;
  Pool& P = pool();
  P.reset();
  if (text_is(opn, "causal-attention.forward") || text_is(opn, "causal-attention.backward")) {
    const bool bwd = text_is(opn, "causal-attention.backward");
    AttShape s;
    int32_t r = attention_checks(c, bwd, cl, s, e);
    if (r) return r;
    run_attention(cl, s, bwd, true, outs);
    for (size_t i = 0; i < outs.size(); i++)
      if (!device_finite((const float*)outs[i], cl.out[i]->byte_length / 4))
        return preflight_fail(e, opn);
  } else if (text_is(opn, "rope.forward") || text_is(opn, "rope.backward")) {
    const bool bwd = text_is(opn, "rope.backward");
    RopeShape s;
    int32_t r = rope_checks(c, bwd, cl, s, e);
    if (r) return r;
    run_rope(cl, s, bwd, true, outs);
    if (!device_finite((const float*)outs[0], cl.out[0]->byte_length / 4))
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                  "RoPE output would be nonfinite");
  } else {
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, "a2.provider",
                "operation is outside this provider's capabilities");
  }
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

void a2_invoke(const et_kernel_call_v1* c) {
  const char* opn = c->request->operation;
  Call cl;
  std::vector<void*> outs;
  pool().reset();
  et_kernel_error e;
  if (text_is(opn, "causal-attention.forward") || text_is(opn, "causal-attention.backward")) {
    const bool bwd = text_is(opn, "causal-attention.backward");
    AttShape s;
    if (attention_checks(c, bwd, cl, s, &e)) return;
    run_attention(cl, s, bwd, false, outs);
  } else {
    const bool bwd = text_is(opn, "rope.backward");
    RopeShape s;
    if (rope_checks(c, bwd, cl, s, &e)) return;
    run_rope(cl, s, bwd, false, outs);
  }
  finish(cl, outs);
}

// ============================================================== N2 / N3K

enum NOp {
  OP_EMB_F, OP_EMB_B, OP_LIN_F, OP_LIN_FN, OP_LIN_B, OP_LIN_BN, OP_LN_F, OP_LN_B, OP_GELU_F,
  OP_GELU_B, OP_RELU_F, OP_RELU_B, OP_RES_F, OP_RES_B, OP_NONE
};

NOp n2_kind(const char* o) {
  static const char* names[] = {"embedding.forward", "embedding.backward", "linear.forward",
                                "linear.forward-no-bias", "linear.backward",
                                "linear.backward-no-bias", "layer-norm.forward",
                                "layer-norm.backward", "gelu.forward", "gelu.backward",
                                "relu.forward", "relu.backward", "residual.forward",
                                "residual.backward"};
  for (int i = 0; i < OP_NONE; i++)
    if (text_is(o, names[i])) return (NOp)i;
  return OP_NONE;
}

const char* n2_capability(NOp k) {
  switch (k) {
    case OP_EMB_F: return "kernel.embedding-forward";
    case OP_EMB_B: return "kernel.embedding-backward";
    case OP_LIN_F: case OP_LIN_FN: case OP_LIN_B: case OP_LIN_BN: return "kernel.matmul";
    case OP_LN_F: case OP_LN_B: return "kernel.norm";
    case OP_GELU_F: case OP_GELU_B: case OP_RELU_F: case OP_RELU_B: return "kernel.activation";
    case OP_RES_F: case OP_RES_B: return "kernel.residual";
    default: return "";
  }
}

struct NPlan {
  NOp kind = OP_NONE;
  uint64_t d[4] = {0, 0, 0, 0};
  bool n3k = false;
};

int32_t n2_checks(const et_kernel_call_v1* c, bool n3k, Call& cl, NPlan& pl, et_kernel_error* e) {
  if (c == nullptr || c->request == nullptr || c->request->operation == nullptr)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT,
                n3k ? "n3k.provider" : "n2.provider", "call, request, and operation are required");
  const char* opn = c->request->operation;
  pl.n3k = n3k;
  if (n3k) {
    pl.kind = text_is(opn, "n3k.linear.forward-no-bias")    ? OP_LIN_FN
              : text_is(opn, "n3k.linear.backward-no-bias") ? OP_LIN_BN
                                                            : OP_NONE;
  } else {
    pl.kind = n2_kind(opn);
  }
  const char* cap = n3k ? "n3k.linear" : n2_capability(pl.kind);
  if (pl.kind == OP_NONE)
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                "operation is outside this provider's capabilities");
  int32_t r = common_request(c, cap, opn, e);
  if (r) return r;
  const bool four = pl.kind <= OP_LIN_BN;
  if (!request_shape(c, four ? 4 : 3, pl.d))
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                "request shape is outside this provider's capabilities");
  const uint64_t* d = pl.d;
  std::vector<Spec> ins, outs;
  switch (pl.kind) {
    case OP_EMB_F:
      ins = {{"i64", 2, {d[0], d[1]}}, {"f32", 2, {d[2], d[3]}}};
      outs = {{"f32", 3, {d[0], d[1], d[3]}}};
      break;
    case OP_EMB_B:
      ins = {{"i64", 2, {d[0], d[1]}}, {"f32", 3, {d[0], d[1], d[3]}}};
      outs = {{"f32", 2, {d[2], d[3]}}};
      break;
    case OP_LIN_F: case OP_LIN_FN:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 2, {d[3], d[2]}}};
      if (pl.kind == OP_LIN_F) ins.push_back({"f32", 1, {d[3]}});
      outs = {{"f32", 3, {d[0], d[1], d[3]}}};
      break;
    case OP_LIN_B: case OP_LIN_BN:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 2, {d[3], d[2]}},
             {"f32", 3, {d[0], d[1], d[3]}}};
      outs = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 2, {d[3], d[2]}}};
      if (pl.kind == OP_LIN_B) outs.push_back({"f32", 1, {d[3]}});
      break;
    case OP_LN_F:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 1, {d[2]}}, {"f32", 1, {d[2]}}, {"f32", 0, {}}};
      outs = {{"f32", 3, {d[0], d[1], d[2]}}};
      break;
    case OP_LN_B:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 1, {d[2]}}, {"f32", 0, {}},
             {"f32", 3, {d[0], d[1], d[2]}}};
      outs = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 1, {d[2]}}, {"f32", 1, {d[2]}}};
      break;
    case OP_GELU_F: case OP_RELU_F:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}};
      outs = ins;
      break;
    case OP_GELU_B: case OP_RELU_B:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 3, {d[0], d[1], d[2]}}};
      outs = {{"f32", 3, {d[0], d[1], d[2]}}};
      break;
    case OP_RES_F:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 3, {d[0], d[1], d[2]}}};
      outs = {{"f32", 3, {d[0], d[1], d[2]}}};
      break;
    case OP_RES_B:
      ins = {{"f32", 3, {d[0], d[1], d[2]}}};
      outs = {{"f32", 3, {d[0], d[1], d[2]}}, {"f32", 3, {d[0], d[1], d[2]}}};
      break;
    default: break;
  }
  r = check_tables(c, opn, ins.size(), outs.size(), ins.data(), outs.data(), &cl, e);
  if (r) return r;
  // floating inputs finite; ids in range
  for (size_t i = 0; i < cl.in.size(); i++) {
    if (text_is(cl.in[i]->dtype, "f32")) {
      if (!inputs_finite(cl, {i}))
        return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                    "floating input is nonfinite");
    } else {
      auto ids = host_copy<int64_t>(cl, i);
      for (int64_t id : ids)
        if (id < 0 || (uint64_t)id >= d[2])
          return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                      "embedding ID is outside the signed exact vocabulary range");
    }
  }
  if (pl.kind == OP_LN_F || pl.kind == OP_LN_B) {
    auto eps = host_copy<float>(cl, pl.kind == OP_LN_F ? 3 : 2);
    if (eps.empty() || !(eps[0] > 0.0f))
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                  "LayerNorm epsilon must be finite and greater than zero");
  }
  return 0;
}

// A GEMM operand as the contraction mode wants it: the tensor itself (TF32,
// FFMA), its TF32 hi/lo pair (3xTF32), or its binary16 hi/lo pair scaled by
// 2^exp with exp from the tensor's own max |x| (split-f16; amax 2^exp below
// 2^15, so no binary16 overflow).
struct Operand {
  const float* hi;
  const float* lo;
  const int* exp;
};
Operand make_pair(const float* x, size_t n, bool f16) {
  Pool& P = pool();
  if (f16) {
    uint16_t* h = (uint16_t*)P.alloc(n * 2);
    uint16_t* l = (uint16_t*)P.alloc(n * 2);
    unsigned* amax = (unsigned*)P.alloc(sizeof(unsigned));
    int* ex = (int*)P.alloc(sizeof(int));
    cudaMemsetAsync(amax, 0, sizeof(unsigned), P.stream);
    cudaMemsetAsync(ex, 0, sizeof(int), P.stream);
    abs_max(x, n, amax, P.stream);
    scale_from_amax(amax, ex, 1, 15, 0, P.stream);
    split_f16(x, nullptr, n, h, l, ex, nullptr, P.stream);
    return Operand{(const float*)h, (const float*)l, ex};
  }
  if (g_precision != ET_B200_PRECISION_TF32X3 && g_precision != ET_B200_PRECISION_F16X3)
    return Operand{x, nullptr, nullptr};
  float* h = (float*)P.alloc(n * 4);
  float* l = (float*)P.alloc(n * 4);
  split_tf32(x, h, l, n, P.stream);
  return Operand{h, l, nullptr};
}
// Split-f16 takes the linear ops whose leading dimensions keep binary16 rows
// 16-byte aligned; the others run 3xTF32.
int linear_precision(bool f16) {
  return f16 ? (int)ET_B200_PRECISION_F16X3
             : (g_precision == ET_B200_PRECISION_F16X3 ? (int)ET_B200_PRECISION_TF32X3
                                                       : (int)g_precision);
}
void set_operands(GemmArgs& g, const Operand& a, const Operand& b) {
  g.A = a.hi; g.A_lo = a.lo; g.exp_a = a.exp;
  g.B = b.hi; g.B_lo = b.lo; g.exp_b = b.exp;
  g.f16 = a.exp != nullptr;
}

void run_n2(Call& cl, const NPlan& pl, bool scratch, std::vector<void*>& outs) {
  Pool& P = pool();
  cudaStream_t s = P.stream;
  const uint64_t* d = pl.d;
  const size_t rows = d[0] * d[1];
  for (size_t i = 0; i < cl.out.size(); i++) outs.push_back(dev_out(cl, i, scratch));
  switch (pl.kind) {
    case OP_EMB_F:
      embedding_forward((const int64_t*)dev_in(cl, 0), (const float*)dev_in(cl, 1),
                        (float*)outs[0], rows, d[2], d[3], P.flag + 1, s);
      break;
    case OP_EMB_B: {
      void* scratch_sort = P.alloc(embedding_scratch_bytes(rows, d[2]));
      embedding_backward((const int64_t*)dev_in(cl, 0), (const float*)dev_in(cl, 1), nullptr,
                         (float*)outs[0], rows, d[2], d[3], scratch_sort, s);
      break;
    }
    case OP_LIN_F: case OP_LIN_FN: {
      const float *x = (const float*)dev_in(cl, 0), *w = (const float*)dev_in(cl, 1);
      const float* b = pl.kind == OP_LIN_F ? (const float*)dev_in(cl, 2) : nullptr;
      const bool f16 = g_precision == ET_B200_PRECISION_F16X3 && d[2] % 8 == 0;
      const Operand xo = make_pair(x, rows * d[2], f16), wo = make_pair(w, d[3] * d[2], f16);
      GemmArgs g{};
      g.M = (int)rows; g.N = (int)d[3]; g.K = (int)d[2];
      set_operands(g, xo, wo);
      g.lda = d[2]; g.a_kmajor = true;
      g.ldb = d[2]; g.b_kmajor = true;
      g.C = (float*)outs[0]; g.ldc = d[3]; g.bias = b; g.accumulate = false;
      g.chunk_ws_floats = gemm_chunk_ws_floats();
      g.chunk_ws = (float*)P.alloc(g.chunk_ws_floats * 4);
      gemm(g, linear_precision(f16), s);
      break;
    }
    case OP_LIN_B: case OP_LIN_BN: {
      const float *x = (const float*)dev_in(cl, 0), *w = (const float*)dev_in(cl, 1),
                  *dy = (const float*)dev_in(cl, 2);
      const bool f16 = g_precision == ET_B200_PRECISION_F16X3 && d[2] % 8 == 0 && d[3] % 8 == 0;
      const Operand xo = make_pair(x, rows * d[2], f16), wo = make_pair(w, d[3] * d[2], f16),
                    go = make_pair(dy, rows * d[3], f16);
      GemmArgs g{};
      g.M = (int)rows; g.N = (int)d[2]; g.K = (int)d[3];
      set_operands(g, go, wo);
      g.lda = d[3]; g.a_kmajor = true;
      g.ldb = d[2]; g.b_kmajor = false;
      g.C = (float*)outs[0]; g.ldc = d[2];
      g.chunk_ws_floats = gemm_chunk_ws_floats();
      g.chunk_ws = (float*)P.alloc(g.chunk_ws_floats * 4);
      gemm(g, linear_precision(f16), s);
      GemmArgs w2{};
      w2.M = (int)d[3]; w2.N = (int)d[2]; w2.K = (int)rows;
      set_operands(w2, go, xo);
      w2.lda = d[3]; w2.a_kmajor = false;
      w2.ldb = d[2]; w2.b_kmajor = false;
      w2.C = (float*)outs[1]; w2.ldc = d[2];
      w2.chunk_ws = g.chunk_ws;  // (same stream, after the dX GEMM)
      w2.chunk_ws_floats = g.chunk_ws_floats;
      gemm(w2, linear_precision(f16), s);
      if (pl.kind == OP_LIN_B) {
        float* ws = (float*)P.alloc(colsum_workspace_floats(rows, d[3]) * 4);
        column_sum(dy, (float*)outs[2], rows, d[3], ws, s);
      }
      break;
    }
    case OP_LN_F: {
      const float* x = (const float*)dev_in(cl, 0);
      auto eps = host_copy<float>(cl, 3);
      layer_norm_forward(x, (const float*)dev_in(cl, 1), (const float*)dev_in(cl, 2), eps[0],
                         (float*)outs[0], nullptr, nullptr, rows, d[2], s);
      break;
    }
    case OP_LN_B: {
      const float* x = (const float*)dev_in(cl, 0);
      const float* gamma = (const float*)dev_in(cl, 1);
      auto eps = host_copy<float>(cl, 2);
      const float* dy = (const float*)dev_in(cl, 3);
      float* mean = (float*)P.alloc(rows * 4);
      float* rstd = (float*)P.alloc(rows * 4);
      float* tmp = (float*)P.alloc(rows * d[2] * 4);
      float* ones = (float*)P.alloc(d[2] * 4);
      float* zeros = (float*)P.alloc(d[2] * 4);
      std::vector<float> one(d[2], 1.0f);
      cudaMemcpyAsync(ones, one.data(), d[2] * 4, cudaMemcpyHostToDevice, s);
      cudaMemsetAsync(zeros, 0, d[2] * 4, s);
      layer_norm_forward(x, ones, zeros, eps[0], tmp, mean, rstd, rows, d[2], s);
      float* ws = (float*)P.alloc(ln_workspace_floats(rows, d[2]) * 4);
      layer_norm_backward(x, gamma, mean, rstd, dy, (float*)outs[0], 0, (float*)outs[1],
                          (float*)outs[2], ws, rows, d[2], s);
      cudaStreamSynchronize(s);  // `one` is a host temporary
      break;
    }
    case OP_GELU_F:
      gelu_forward((const float*)dev_in(cl, 0), (float*)outs[0], rows * d[2], s);
      break;
    case OP_GELU_B:
      gelu_backward((const float*)dev_in(cl, 0), (const float*)dev_in(cl, 1), (float*)outs[0],
                    rows * d[2], s);
      break;
    case OP_RELU_F:
      relu_forward((const float*)dev_in(cl, 0), (float*)outs[0], rows * d[2], s);
      break;
    case OP_RELU_B:
      relu_backward((const float*)dev_in(cl, 0), (const float*)dev_in(cl, 1), (float*)outs[0],
                    rows * d[2], s);
      break;
    case OP_RES_F:
      add_tensors((const float*)dev_in(cl, 0), (const float*)dev_in(cl, 1), (float*)outs[0],
                  rows * d[2], s);
      break;
    case OP_RES_B: {
      const float* dy = (const float*)dev_in(cl, 0);
      copy_tensor(dy, (float*)outs[0], rows * d[2], s);
      copy_tensor(dy, (float*)outs[1], rows * d[2], s);
      break;
    }
    default: break;
  }
}

int32_t n_validate(const et_kernel_call_v1* c, et_kernel_error* e, bool n3k) {
  Call cl;
  NPlan pl;
  pool().reset();
  int32_t r = n2_checks(c, n3k, cl, pl, e);
  if (r) return r;
  std::vector<void*> outs;
  run_n2(cl, pl, true, outs);
  for (size_t i = 0; i < outs.size(); i++)
    if (!device_finite((const float*)outs[i], cl.out[i]->byte_length / 4))
      return preflight_fail(e, c->request->operation);
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

void n_invoke(const et_kernel_call_v1* c, bool n3k) {
  Call cl;
  NPlan pl;
  et_kernel_error e;
  pool().reset();
  if (n2_checks(c, n3k, cl, pl, &e)) return;
  std::vector<void*> outs;
  run_n2(cl, pl, false, outs);
  finish(cl, outs);
}

int32_t n2_validate(const et_kernel_call_v1* c, et_kernel_error* e) { return n_validate(c, e, false); }
void n2_invoke(const et_kernel_call_v1* c) { n_invoke(c, false); }
int32_t n3k_validate(const et_kernel_call_v1* c, et_kernel_error* e) { return n_validate(c, e, true); }
void n3k_invoke(const et_kernel_call_v1* c) { n_invoke(c, true); }

// ============================================================== L2

int32_t l2_checks(const et_kernel_call_v1* c, Call& cl, bool& backward, et_kernel_error* e) {
  if (c == nullptr || c->request == nullptr || c->request->operation == nullptr)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT,
                "indexed-cross-entropy", "call, request, and operation are required");
  const char* opn = c->request->operation;
  const bool fwd = text_is(opn, "indexed-cross-entropy.forward");
  backward = text_is(opn, "indexed-cross-entropy.backward");
  uint64_t d[3];
  if ((!fwd && !backward) || !request_shape(c, 3, d))
    return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_PROVIDER_REJECTED,
                "indexed-cross-entropy", "operation or request shape is invalid");
  int32_t r = common_request(c, "kernel.indexed-cross-entropy", opn, e);
  if (r) return r;
  const Spec logits{"f32", 3, {d[0], d[1], d[2]}}, rows{"f32", 2, {d[0], d[1]}};
  const Spec ins[3] = {logits, {"i64", 2, {d[0], d[1]}}, rows};
  const Spec outs[1] = {backward ? logits : rows};
  r = check_tables(c, opn, backward ? 3 : 2, 1, ins, outs, &cl, e);
  if (r) return r;
  auto targets = host_copy<int64_t>(cl, 1);
  for (int64_t t : targets)
    if (t < 0 || (uint64_t)t >= d[2])
      return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                  "target index is outside the vocabulary");
  if (!inputs_finite(cl, {0}))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                "logits must be finite f32 values");
  if (backward && !inputs_finite(cl, {2}))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, opn,
                "upstream gradients must be finite f32 values");
  return 0;
}

void run_l2(Call& cl, bool backward, bool scratch, std::vector<void*>& outs) {
  Pool& P = pool();
  const uint64_t* d = cl.call->request->shape;
  const size_t rows = d[0] * d[1];
  const float* logits = (const float*)dev_in(cl, 0);
  const int64_t* targets = (const int64_t*)dev_in(cl, 1);
  float* out = (float*)dev_out(cl, 0, scratch);
  outs = {out};
  if (backward)
    ce_fused(logits, out, targets, (const float*)dev_in(cl, 2), 0.0f, nullptr, rows, d[2],
             P.flag + 1, P.stream);
  else
    ce_fused(logits, nullptr, targets, nullptr, 0.0f, out, rows, d[2], P.flag + 1, P.stream);
}

int32_t l2_validate(const et_kernel_call_v1* c, et_kernel_error* e) {
  Call cl;
  bool backward = false;
  pool().reset();
  int32_t r = l2_checks(c, cl, backward, e);
  if (r) return r;
  std::vector<void*> outs;
  run_l2(cl, backward, true, outs);
  if (!device_finite((const float*)outs[0], cl.out[0]->byte_length / 4))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED,
                c->request->operation,
                backward ? "logit gradient is not representable as finite f32"
                         : "per-token loss is not representable as finite f32");
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

void l2_invoke(const et_kernel_call_v1* c) {
  Call cl;
  bool backward = false;
  et_kernel_error e;
  pool().reset();
  if (l2_checks(c, cl, backward, &e)) return;
  std::vector<void*> outs;
  run_l2(cl, backward, false, outs);
  finish(cl, outs);
}

// ============================================================== descriptors

#define UNBOUNDED {1u, 0u, 1u, {0}}
const et_kernel_dimension_range_v1 dims6[6] = {UNBOUNDED, UNBOUNDED, UNBOUNDED,
                                               UNBOUNDED, UNBOUNDED, UNBOUNDED};
#undef UNBOUNDED
const et_kernel_shape_range_v1 rank3[1] = {{3u, dims6}};
const et_kernel_shape_range_v1 rank4[1] = {{4u, dims6}};
const et_kernel_shape_range_v1 rank6[1] = {{6u, dims6}};
const et_kernel_dimension_range_v1 l2_dims[3] = {{1u, 1664510u, 0u, {0}},
                                                 {1u, 1664510u, 0u, {0}},
                                                 {1u, 1664510u, 0u, {0}}};
const et_kernel_shape_range_v1 l2_rank3[1] = {{3u, l2_dims}};

const char* const f32_only[] = {"f32"};
const char* const devices[] = {"cpu", "cuda"};
const char* const att_ops[] = {"causal-attention.backward", "causal-attention.forward"};
const char* const rope_ops[] = {"rope.backward", "rope.forward"};
const char* const act_ops[] = {"gelu.backward", "gelu.forward", "relu.backward", "relu.forward"};
const char* const embf_ops[] = {"embedding.forward"};
const char* const embb_ops[] = {"embedding.backward"};
const char* const mm_ops[] = {"linear.backward", "linear.backward-no-bias", "linear.forward",
                              "linear.forward-no-bias"};
const char* const norm_ops[] = {"layer-norm.backward", "layer-norm.forward"};
const char* const res_ops[] = {"residual.backward", "residual.forward"};
const char* const n3k_ops[] = {"n3k.linear.backward-no-bias", "n3k.linear.forward-no-bias"};
const char* const l2_ops[] = {"indexed-cross-entropy.backward", "indexed-cross-entropy.forward"};

#define CAP(name, ops, ranges, impl)                                                        \
  {sizeof(et_kernel_capability_v1), name, ET_KERNEL_CAPABILITY_VERIFIED, impl, "1.0",       \
   "B200:sm100a-f32-v1", 1u, {0}, sizeof(ops) / sizeof(ops[0]), ops, 1, f32_only, 2, devices, \
   1, ranges}

const et_kernel_capability_v1 a2_caps[] = {
    CAP("kernel.causal-attention", att_ops, rank6, "a2.b200-sm100a"),
    CAP("kernel.rope", rope_ops, rank4, "a2.b200-sm100a"),
};
const et_kernel_capability_v1 n2_caps[] = {
    CAP("kernel.activation", act_ops, rank3, "n2.b200-sm100a"),
    CAP("kernel.embedding-backward", embb_ops, rank4, "n2.b200-sm100a"),
    CAP("kernel.embedding-forward", embf_ops, rank4, "n2.b200-sm100a"),
    CAP("kernel.matmul", mm_ops, rank4, "n2.b200-sm100a"),
    CAP("kernel.norm", norm_ops, rank3, "n2.b200-sm100a"),
    CAP("kernel.residual", res_ops, rank3, "n2.b200-sm100a"),
};
const et_kernel_capability_v1 n3k_caps[] = {
    CAP("n3k.linear", n3k_ops, rank4, "n3k.b200-sm100a"),
};
const et_kernel_capability_v1 l2_caps[] = {
    CAP("kernel.indexed-cross-entropy", l2_ops, l2_rank3, "l2.b200-sm100a"),
};
#undef CAP

#define PROVIDER(caps, nm, val, inv)                                                          \
  {sizeof(et_kernel_provider_v1), ET_KERNEL_ABI_MAJOR, ET_KERNEL_ABI_MINOR, 0u, nm, "1.0",    \
   "B200:sm100a-f32-v1", sizeof(caps) / sizeof(caps[0]), sizeof(et_kernel_capability_v1),     \
   sizeof(caps), caps, val, inv}

const et_kernel_provider_v1 a2_provider = PROVIDER(a2_caps, "a2.b200-sm100a", a2_validate, a2_invoke);
const et_kernel_provider_v1 n2_provider = PROVIDER(n2_caps, "n2.b200-sm100a", n2_validate, n2_invoke);
const et_kernel_provider_v1 n3k_provider =
    PROVIDER(n3k_caps, "n3k.b200-sm100a", n3k_validate, n3k_invoke);
const et_kernel_provider_v1 l2_provider = PROVIDER(l2_caps, "l2.b200-sm100a", l2_validate, l2_invoke);

// ---- one provider for every capability ---------------------------------------------
// A K1 runtime takes exactly one provider from its resolver
// (native/kernel_abi.c:764-840); the composite lists the four providers'
// capabilities, sorted by name, and hands each call to the provider owning
// its capability.
const et_kernel_capability_v1 all_caps[] = {
    n2_caps[0],   // kernel.activation
    a2_caps[0],   // kernel.causal-attention
    n2_caps[1],   // kernel.embedding-backward
    n2_caps[2],   // kernel.embedding-forward
    l2_caps[0],   // kernel.indexed-cross-entropy
    n2_caps[3],   // kernel.matmul
    n2_caps[4],   // kernel.norm
    n2_caps[5],   // kernel.residual
    a2_caps[1],   // kernel.rope
    n3k_caps[0],  // n3k.linear
};

const et_kernel_provider_v1* owner_of(const et_kernel_call_v1* c) {
  if (c == nullptr || c->capability == nullptr) return nullptr;
  for (const et_kernel_provider_v1* p : {&a2_provider, &n2_provider, &n3k_provider, &l2_provider})
    for (size_t i = 0; i < p->capability_count; i++)
      if (strcmp(static_cast<const et_kernel_capability_v1*>(p->capabilities)[i].name,
                 c->capability) == 0)
        return p;
  return nullptr;
}
int32_t all_validate(const et_kernel_call_v1* c, et_kernel_error* e) {
  const et_kernel_provider_v1* p = owner_of(c);
  if (p == nullptr)
    return fail(e, ET_KERNEL_ERROR_UNSUPPORTED, ET_KERNEL_CODE_PROVIDER_REJECTED,
                "b200-dispatch", "capability is not provided");
  return p->validate_call(c, e);
}
void all_invoke(const et_kernel_call_v1* c) {
  const et_kernel_provider_v1* p = owner_of(c);
  if (p != nullptr) p->invoke_call(c);
}
const et_kernel_provider_v1 all_provider =
    PROVIDER(all_caps, "b200.sm100a", all_validate, all_invoke);
#undef PROVIDER

// The fixed resolver's private context (its address is the token).
const unsigned char k2_resolver_sentinel = 0x62u;

bool same_text(const char* a, const char* b) { return a != nullptr && strcmp(a, b) == 0; }

}  // namespace

extern "C" {

const et_kernel_provider_v1* et_a2_kernel_provider_v1(void) { return &a2_provider; }
const et_kernel_provider_v1* et_n2_kernel_provider_v1(void) { return &n2_provider; }
const et_kernel_provider_v1* et_n3k_kernel_provider_v1(void) { return &n3k_provider; }
const et_kernel_provider_v1* et_l2_indexed_cross_entropy_provider_v1(void) { return &l2_provider; }
const et_kernel_provider_v1* et_b200_kernel_provider_v1(void) { return &all_provider; }

const void* et_b200_k2_resolver_context_v1(void) { return &k2_resolver_sentinel; }

const et_kernel_provider_v1* et_b200_k2_resolver_v1(void* context, const char* symbol) {
  if (context != &k2_resolver_sentinel || !same_text(symbol, "eshkol_transformer_kernel_provider_v1"))
    return nullptr;
  return &all_provider;
}

int32_t et_b200_k2_audit_provider_v1(const et_kernel_provider_v1* p) {
  if (p == nullptr) return ET_B200_K2_PROVIDER_ABSENT;
  if (p->struct_size != sizeof(et_kernel_provider_v1) || p->abi_major != ET_KERNEL_ABI_MAJOR ||
      p->abi_minor != ET_KERNEL_ABI_MINOR || p->required_features != 0u ||
      !same_text(p->version, all_provider.version))
    return ET_B200_K2_PROVIDER_VERSION_MISMATCH;
  const size_t n = sizeof(all_caps) / sizeof(all_caps[0]);
  bool exact = same_text(p->name, all_provider.name) &&
               same_text(p->evidence, all_provider.evidence) && p->capability_count == n &&
               p->capability_stride == sizeof(et_kernel_capability_v1) &&
               p->capability_bytes == sizeof(all_caps) && p->capabilities != nullptr &&
               p->validate_call == all_provider.validate_call &&
               p->invoke_call == all_provider.invoke_call;
  for (size_t i = 0; exact && i < n; i++) {
    const et_kernel_capability_v1& a = static_cast<const et_kernel_capability_v1*>(p->capabilities)[i];
    const et_kernel_capability_v1& b = all_caps[i];
    exact = a.struct_size == b.struct_size && same_text(a.name, b.name) && a.status == b.status &&
            same_text(a.implementation, b.implementation) && same_text(a.version, b.version) &&
            same_text(a.evidence, b.evidence) && a.deterministic == b.deterministic &&
            a.operation_count == b.operation_count && a.dtype_count == b.dtype_count &&
            a.device_count == b.device_count && a.shape_range_count == b.shape_range_count;
    for (size_t k = 0; exact && k < b.operation_count; k++)
      exact = same_text(a.operations[k], b.operations[k]);
    for (size_t k = 0; exact && k < b.device_count; k++)
      exact = same_text(a.devices[k], b.devices[k]);
  }
  return exact ? ET_B200_K2_PROVIDER_EXACT : ET_B200_K2_PROVIDER_METADATA_MISMATCH;
}

int32_t et_l2_indexed_cross_entropy_abi_major_v1(void) { return 1; }
int32_t et_l2_indexed_cross_entropy_abi_minor_v1(void) { return 0; }

// Contraction mode of the K1 matmul / n3k.linear providers (process-wide).
int32_t et_b200_k1_precision_v1(uint32_t precision) {
  if (precision > ET_B200_PRECISION_F16X3) return ET_KERNEL_ERROR_INVALID_ARGUMENT;
  g_precision = precision;
  return 0;
}

}  // extern "C"
