// A2 KV cache on the device: transactional append of post-RoPE K/V into
// HBM-resident storage, with the reference's handle, lease and error
// semantics (native/a2_kv_cache.c:394-880, ABI
// include/eshkol_transformer/a2_kv_cache.h:42-147).
//
// Storage K, V f32 [layers, batch, kv_heads, capacity, head_dimension] and the
// committed key-keep mask u8 [batch, capacity] live in device memory of the
// GPU that was current at create; committed lengths i64 [batch] are kept on
// the host (admission checks) and mirrored on the device (views).  A
// transaction snapshots the append counts, derives the effective lengths and
// mask on the device, copies each staged layer's first counts[n] positions of
// [batch, kv_heads, append_width, head_dimension] into the tail at the old
// length, and on abort scrubs every staged slot back to +0.  Views and read
// borrows hand out device ("cuda") tensor views of the storage; they feed the
// device attention provider without a copy (cached decoding: Tq = the new
// tokens, Tk = capacity, the key-keep mask broadcast over the queries).
//
// Every call completes its device work before returning (one private stream
// per cache, synchronised), like the reference's synchronous CPU copies.
// Sources may be "cpu" (host, staged through a per-transaction device buffer)
// or "cuda" views; append counts are "cpu" (they are needed on the host).
// Handle, slot and alias checks restate the reference's rules with the same
// error categories and codes; host-memory span checks apply to host data,
// and device data is checked against the live caches' device storage.
#include <math.h>

#include <algorithm>
#include <mutex>
#include <unordered_set>
#include <vector>

#include "eshkol_b200/et_b200.h"
#include "ops.cuh"

namespace {

constexpr uint64_t kCacheMagic = 0x42324b5643414348ull;
constexpr uint64_t kTxnMagic = 0x42324b565452414eull;
constexpr uint64_t kViewMagic = 0x42324b5656494557ull;
constexpr uint64_t kBorrowMagic = 0x42324b56424f5252ull;

}  // namespace

struct et_a2_kv_cache {
  uint64_t magic;
  int device;
  cudaStream_t stream;
  size_t layers, batch, kv_heads, capacity, head_dimension;
  size_t layer_elements, total_elements;
  float* keys;             // device
  float* values;           // device
  int64_t* lengths_dev;    // device [batch], committed
  uint8_t* mask_dev;       // device [batch, capacity], committed
  std::vector<int64_t> lengths;  // host copy of the committed lengths
  et_a2_kv_cache_transaction* active_transaction;
  et_a2_kv_cache_read_borrow* active_borrow;
};

struct et_a2_kv_cache_transaction {
  uint64_t magic;
  et_a2_kv_cache* cache;
  size_t append_width;
  std::vector<int64_t> counts;
  int64_t* counts_dev;      // device [batch]
  int64_t* old_lengths_dev; // device [batch]
  int64_t* lengths_dev;     // device [batch], effective
  uint8_t* mask_dev;        // device [batch, capacity], effective
  float* staging;           // device copy of host sources (K then V), lazily allocated
  std::vector<uint8_t> staged;
  et_a2_kv_cache_transaction_view* active_view;
};

struct et_a2_kv_cache_transaction_view {
  uint64_t magic;
  et_a2_kv_cache_transaction* transaction;
  size_t layer;
  uint64_t tensor_shape[4], lengths_shape[1], mask_shape[2];
  et_kernel_tensor_view_v1 keys, values, lengths, key_keep_mask;
};

struct et_a2_kv_cache_read_borrow {
  uint64_t magic;
  et_a2_kv_cache* cache;
  uint64_t tensor_shape[4], lengths_shape[1], mask_shape[2];
  std::vector<et_kernel_tensor_view_v1> keys, values;
  et_kernel_tensor_view_v1 lengths, key_keep_mask;
};

namespace {

std::mutex g_mu;
std::unordered_set<const void*> g_caches, g_txns, g_views, g_borrows;

// ---- device work --------------------------------------------------------------------

// dst[(n, h, old[n] + a)] = src[(n, h, a)] for a < counts[n] (one thread per
// element of the [batch, kv_heads, width, dim] source); with src == nullptr
// the destination slots are set to +0 instead (abort).
__global__ void kv_copy_kernel(float* __restrict__ dk, float* __restrict__ dv,
                               const float* __restrict__ sk, const float* __restrict__ sv,
                               const int64_t* __restrict__ counts,
                               const int64_t* __restrict__ old_len, int64_t batch,
                               int64_t heads, int64_t width, int64_t capacity, int64_t dim) {
  const int64_t total = batch * heads * width * dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = i % dim;
    const int64_t a = (i / dim) % width;
    const int64_t h = (i / (dim * width)) % heads;
    const int64_t n = i / (dim * width * heads);
    if (a >= counts[n]) continue;
    const int64_t dst = ((n * heads + h) * capacity + old_len[n] + a) * dim + d;
    dk[dst] = sk != nullptr ? sk[i] : 0.0f;
    dv[dst] = sv != nullptr ? sv[i] : 0.0f;
  }
}

// mask[n, c] = c < lengths[n]
__global__ void kv_mask_kernel(uint8_t* __restrict__ mask, const int64_t* __restrict__ lengths,
                               int64_t batch, int64_t capacity) {
  const int64_t total = batch * capacity;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    mask[i] = (i % capacity) < lengths[i / capacity] ? 1u : 0u;
}

unsigned grid_of(int64_t total) {
  const int64_t want = (total + 255) / 256;
  const int64_t cap = (int64_t)etb::sm_count() * 8;
  return (unsigned)std::max<int64_t>(1, std::min(want, cap));
}

// Runs on the cache's device; restores the caller's device.
struct DeviceScope {
  int previous = 0;
  explicit DeviceScope(int device) {
    cudaGetDevice(&previous);
    if (previous != device) cudaSetDevice(device);
  }
  ~DeviceScope() {
    int now = 0;
    cudaGetDevice(&now);
    if (now != previous) cudaSetDevice(previous);
  }
};

// ---- validation (restating native/a2_kv_cache.c:97-357) -----------------------------

bool overlaps(const void* a, size_t an, const void* b, size_t bn) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return an != 0 && bn != 0 && x < y + bn && y < x + an;
}
bool span_fits(const void* p, size_t n) {
  return p != nullptr && reinterpret_cast<uintptr_t>(p) <= UINTPTR_MAX - n;
}
bool mul_size(size_t a, size_t b, size_t* out) {
  if (a != 0 && b > SIZE_MAX / a) return false;
  *out = a * b;
  return true;
}

// Host-side objects owned by this library (handles and the descriptors they
// hand out): a caller span overlapping one of them is rejected.
bool live_host_overlap(const void* p, size_t n) {
  for (const void* c : g_caches)
    if (overlaps(p, n, c, sizeof(et_a2_kv_cache))) return true;
  for (const void* t : g_txns)
    if (overlaps(p, n, t, sizeof(et_a2_kv_cache_transaction))) return true;
  for (const void* v : g_views)
    if (overlaps(p, n, v, sizeof(et_a2_kv_cache_transaction_view))) return true;
  for (const void* b : g_borrows) {
    const auto* r = static_cast<const et_a2_kv_cache_read_borrow*>(b);
    if (overlaps(p, n, b, sizeof(*r))) return true;
    if (!r->keys.empty() &&
        (overlaps(p, n, r->keys.data(), r->keys.size() * sizeof(et_kernel_tensor_view_v1)) ||
         overlaps(p, n, r->values.data(), r->values.size() * sizeof(et_kernel_tensor_view_v1))))
      return true;
  }
  return false;
}
// Device storage of the live caches (and their open transactions).
bool live_device_overlap(const void* p, size_t n) {
  for (const void* cv : g_caches) {
    const auto* c = static_cast<const et_a2_kv_cache*>(cv);
    const size_t bytes = c->total_elements * sizeof(float);
    if (overlaps(p, n, c->keys, bytes) || overlaps(p, n, c->values, bytes) ||
        overlaps(p, n, c->lengths_dev, c->batch * sizeof(int64_t)) ||
        overlaps(p, n, c->mask_dev, c->batch * c->capacity))
      return true;
  }
  for (const void* tv : g_txns) {
    const auto* t = static_cast<const et_a2_kv_cache_transaction*>(tv);
    if (overlaps(p, n, t->lengths_dev, t->cache->batch * sizeof(int64_t)) ||
        overlaps(p, n, t->mask_dev, t->cache->batch * t->cache->capacity))
      return true;
  }
  return false;
}

int32_t raw_reject() { return (int32_t)ET_KERNEL_ERROR_INVALID_ARGUMENT; }

bool error_writable(const et_kernel_error* e) {
  return e == nullptr || (span_fits(e, sizeof(*e)) && !live_host_overlap(e, sizeof(*e)));
}

int32_t fail(et_kernel_error* e, et_kernel_error_category category, et_kernel_error_code code,
             const char* operation, const char* message) {
  if (!error_writable(e)) return raw_reject();
  if (e != nullptr) {
    memset(e, 0, sizeof(*e));
    e->category = category;
    e->code = code;
    snprintf(e->operation, sizeof(e->operation), "%s", operation);
    snprintf(e->message, sizeof(e->message), "%s", message);
  }
  return (int32_t)category;
}

int32_t ok(et_kernel_error* e) {
  if (e != nullptr) memset(e, 0, sizeof(*e));
  return 0;
}

int32_t cuda_fail(et_kernel_error* e, const char* op, cudaError_t st) {
  char text[160];
  snprintf(text, sizeof(text), "CUDA: %s", cudaGetErrorString(st));
  return fail(e, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_ALLOCATION_FAILED, op, text);
}

int output_slot_ok(const void* slot, et_kernel_error* e, const char* op) {
  if (slot == nullptr)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                "output slot is null");
  if (e != nullptr && overlaps(slot, sizeof(void*), e, sizeof(*e))) return raw_reject();
  if (!span_fits(slot, sizeof(void*)) || reinterpret_cast<uintptr_t>(slot) % alignof(void*) != 0 ||
      live_host_overlap(slot, sizeof(void*)))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                "output slot aliases live or error storage");
  return 0;
}

// 1: exact match; 0: other text; -1: the text runs into the error record.
int exact_symbol(const char* s, const char* expected, const et_kernel_error* e) {
  if (s == nullptr) return 0;
  const size_t n = strlen(expected);
  for (size_t i = 0; i <= ET_KERNEL_MAX_SYMBOL_BYTES; i++) {
    if (e != nullptr && overlaps(s + i, 1, e, sizeof(*e))) return -1;
    if (s[i] == '\0') return i == n ? 1 : 0;
    if (i >= n || s[i] != expected[i]) {
      // keep scanning to the terminator for the error-overlap rule
      for (size_t k = i + 1; k <= ET_KERNEL_MAX_SYMBOL_BYTES; k++) {
        if (e != nullptr && overlaps(s + k, 1, e, sizeof(*e))) return -1;
        if (s[k] == '\0') return 0;
      }
      return 0;
    }
  }
  return 0;
}

enum class Where { kCpu, kCuda, kEither };

// Checks a dense zero-offset view of `dtype`, `shape` on the allowed device;
// sets *on_device for a "cuda" view.
int32_t validate_view(const et_kernel_tensor_view_v1* v, const char* dtype, size_t rank,
                      const size_t* shape, size_t elem, Where where, bool* on_device,
                      et_kernel_error* e, const char* op) {
  if (v == nullptr)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                "tensor view is null");
  if (!span_fits(v, sizeof(*v)) || (e != nullptr && overlaps(v, sizeof(*v), e, sizeof(*e))))
    return raw_reject();
  if (live_host_overlap(v, sizeof(*v)))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor descriptor aliases live A2 cache storage");
  if (v->struct_size < ET_KERNEL_TENSOR_VIEW_V1_0_SIZE)
    return fail(e, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_INVALID_STRUCT_SIZE, op,
                "tensor view struct size is not v1.0");
  int r = exact_symbol(v->dtype, dtype, e);
  if (r < 0) return raw_reject();
  if (r == 0)
    return fail(e, ET_KERNEL_ERROR_DTYPE_MISMATCH, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor dtype mismatch");
  const int cpu = exact_symbol(v->device, "cpu", e);
  const int cuda = exact_symbol(v->device, "cuda", e);
  if (cpu < 0 || cuda < 0) return raw_reject();
  const bool device_ok = (where == Where::kCpu && cpu == 1) ||
                         (where == Where::kCuda && cuda == 1) ||
                         (where == Where::kEither && (cpu == 1 || cuda == 1));
  if (!device_ok)
    return fail(e, ET_KERNEL_ERROR_DEVICE_MISMATCH, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor device mismatch");
  *on_device = cuda == 1;
  if (v->layout != ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR || v->offset_bytes != 0u)
    return fail(e, ET_KERNEL_ERROR_NONCONTIGUOUS, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor must be dense row-major with zero offset");
  if (v->rank != rank || v->shape == nullptr)
    return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "tensor rank mismatch");
  if (!span_fits(v->shape, rank * sizeof(*v->shape)) ||
      (e != nullptr && overlaps(v->shape, rank * sizeof(*v->shape), e, sizeof(*e))))
    return raw_reject();
  if (live_host_overlap(v->shape, rank * sizeof(*v->shape)))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor shape aliases live A2 cache storage");
  size_t elements = 1, bytes = 0;
  for (size_t i = 0; i < rank; i++) {
    if (v->shape[i] != shape[i])
      return fail(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                  "tensor shape mismatch");
    if (!mul_size(elements, shape[i], &elements))
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INTEGER_OVERFLOW, op,
                  "tensor element count overflows size_t");
  }
  if (!mul_size(elements, elem, &bytes))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INTEGER_OVERFLOW, op,
                "tensor byte length overflows size_t");
  if (v->byte_length != bytes || v->data == nullptr || !span_fits(v->data, bytes) ||
      reinterpret_cast<uintptr_t>(v->data) % elem != 0)
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor data span or alignment is invalid");
  if (*on_device) {
    if (live_device_overlap(v->data, bytes))
      return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                  "borrowed tensor aliases live A2 cache storage");
    return 0;
  }
  if (e != nullptr && overlaps(v->data, bytes, e, sizeof(*e))) return raw_reject();
  if (overlaps(v->data, bytes, v, sizeof(*v)) ||
      overlaps(v->data, bytes, v->shape, rank * sizeof(*v->shape)))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "tensor data aliases its descriptor metadata");
  if (live_host_overlap(v->data, bytes))
    return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "borrowed tensor aliases live A2 cache storage");
  return 0;
}

et_a2_kv_cache* find_cache(const void* h) {
  return g_caches.count(h) ? const_cast<et_a2_kv_cache*>(static_cast<const et_a2_kv_cache*>(h))
                           : nullptr;
}
et_a2_kv_cache_transaction* find_txn(const void* h) {
  return g_txns.count(h) ? const_cast<et_a2_kv_cache_transaction*>(
                               static_cast<const et_a2_kv_cache_transaction*>(h))
                         : nullptr;
}
et_a2_kv_cache_transaction_view* find_view(const void* h) {
  return g_views.count(h) ? const_cast<et_a2_kv_cache_transaction_view*>(
                                static_cast<const et_a2_kv_cache_transaction_view*>(h))
                          : nullptr;
}
et_a2_kv_cache_read_borrow* find_borrow(const void* h) {
  return g_borrows.count(h) ? const_cast<et_a2_kv_cache_read_borrow*>(
                                  static_cast<const et_a2_kv_cache_read_borrow*>(h))
                            : nullptr;
}

// Device descriptors of layer `layer` with the given lengths / mask storage.
void fill_views(const et_a2_kv_cache* c, size_t layer, const int64_t* lengths,
                const uint8_t* mask, uint64_t ts[4], uint64_t ls[1], uint64_t ms[2],
                et_kernel_tensor_view_v1* k, et_kernel_tensor_view_v1* v,
                et_kernel_tensor_view_v1* l, et_kernel_tensor_view_v1* m) {
  const size_t layer_bytes = c->layer_elements * sizeof(float);
  ts[0] = c->batch; ts[1] = c->kv_heads; ts[2] = c->capacity; ts[3] = c->head_dimension;
  ls[0] = c->batch;
  ms[0] = c->batch; ms[1] = c->capacity;
  *k = et_kernel_tensor_view_v1{sizeof(*k), c->keys + layer * c->layer_elements, layer_bytes,
                                "f32", "cuda", ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR, 0u, 4u, ts};
  *v = et_kernel_tensor_view_v1{sizeof(*v), c->values + layer * c->layer_elements, layer_bytes,
                                "f32", "cuda", ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR, 0u, 4u, ts};
  *l = et_kernel_tensor_view_v1{sizeof(*l), const_cast<int64_t*>(lengths),
                                c->batch * sizeof(int64_t), "i64", "cuda",
                                ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR, 0u, 1u, ls};
  *m = et_kernel_tensor_view_v1{sizeof(*m), const_cast<uint8_t*>(mask), c->batch * c->capacity,
                                "bool", "cuda", ET_KERNEL_LAYOUT_DENSE_ROW_MAJOR, 0u, 2u, ms};
}

void free_txn(et_a2_kv_cache_transaction* t) {
  t->cache->active_transaction = nullptr;
  g_txns.erase(t);
  t->magic = 0;
  cudaFree(t->counts_dev);
  cudaFree(t->old_lengths_dev);
  cudaFree(t->lengths_dev);
  cudaFree(t->mask_dev);
  cudaFree(t->staging);
  delete t;
}

}  // namespace

extern "C" {

int32_t et_a2_kv_cache_abi_major_v1(void) { return 1; }
int32_t et_a2_kv_cache_abi_minor_v1(void) { return 0; }

int32_t et_a2_kv_cache_abi_require_v1(uint32_t major, uint32_t minimum_minor,
                                      et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!error_writable(error)) return raw_reject();
  const char* op = "a2-kv-cache.abi-require";
  if (major != 1u)
    return fail(error, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_ABI_MAJOR_MISMATCH, op,
                "requested ABI major does not match supported major 1");
  if (minimum_minor > 0u)
    return fail(error, ET_KERNEL_ERROR_VERSION_MISMATCH, ET_KERNEL_CODE_UNKNOWN_REQUIRED_FEATURE,
                op, "requested minimum ABI minor exceeds supported minor 0");
  return ok(error);
}

int32_t et_a2_kv_cache_create_v1(uint64_t layers, uint64_t batch, uint64_t kv_heads,
                                 uint64_t capacity, uint64_t head_dimension,
                                 et_a2_kv_cache** out, et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.create";
  if (!error_writable(error)) return raw_reject();
  if (int r = output_slot_ok(out, error, op)) return r;
  if (*out != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "output slot must contain NULL");
  if (layers == 0 || batch == 0 || kv_heads == 0 || capacity == 0 || head_dimension == 0 ||
      layers > SIZE_MAX || batch > SIZE_MAX || kv_heads > SIZE_MAX || capacity > SIZE_MAX ||
      head_dimension > SIZE_MAX)
    return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "all cache dimensions must be positive and representable");
  size_t elements = (size_t)layers, bytes = 0, mask_bytes = 0;
  if (!mul_size(elements, (size_t)batch, &elements) ||
      !mul_size(elements, (size_t)kv_heads, &elements) ||
      !mul_size(elements, (size_t)capacity, &elements) ||
      !mul_size(elements, (size_t)head_dimension, &elements) ||
      !mul_size(elements, sizeof(float), &bytes) ||
      !mul_size((size_t)batch, (size_t)capacity, &mask_bytes) ||
      (size_t)batch > SIZE_MAX / sizeof(int64_t))
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INTEGER_OVERFLOW, op,
                "cache size overflows size_t");
  auto* c = new et_a2_kv_cache{};
  cudaGetDevice(&c->device);
  c->layers = (size_t)layers; c->batch = (size_t)batch; c->kv_heads = (size_t)kv_heads;
  c->capacity = (size_t)capacity; c->head_dimension = (size_t)head_dimension;
  c->total_elements = elements;
  c->layer_elements = elements / c->layers;
  c->lengths.assign(c->batch, 0);
  cudaError_t st = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (st == cudaSuccess) st = cudaMalloc(&c->keys, bytes);
  if (st == cudaSuccess) st = cudaMalloc(&c->values, bytes);
  if (st == cudaSuccess) st = cudaMalloc(&c->lengths_dev, c->batch * sizeof(int64_t));
  if (st == cudaSuccess) st = cudaMalloc(&c->mask_dev, mask_bytes);
  if (st == cudaSuccess) st = cudaMemsetAsync(c->keys, 0, bytes, c->stream);
  if (st == cudaSuccess) st = cudaMemsetAsync(c->values, 0, bytes, c->stream);
  if (st == cudaSuccess) st = cudaMemsetAsync(c->lengths_dev, 0, c->batch * sizeof(int64_t), c->stream);
  if (st == cudaSuccess) st = cudaMemsetAsync(c->mask_dev, 0, mask_bytes, c->stream);
  if (st == cudaSuccess) st = cudaStreamSynchronize(c->stream);
  if (st != cudaSuccess) {
    cudaFree(c->keys); cudaFree(c->values); cudaFree(c->lengths_dev); cudaFree(c->mask_dev);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    cudaGetLastError();
    return fail(error, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_ALLOCATION_FAILED, op,
                "cache allocation failed");
  }
  c->magic = kCacheMagic;
  g_caches.insert(c);
  *out = c;
  return ok(error);
}

int32_t et_a2_kv_cache_destroy_v1(et_a2_kv_cache** slot, et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.destroy";
  if (!error_writable(error)) return raw_reject();
  if (int r = output_slot_ok(slot, error, op)) return r;
  et_a2_kv_cache* c = find_cache(*slot);
  if (c == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "cache handle is invalid");
  if (c->active_transaction != nullptr || c->active_borrow != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "cache has a live lease");
  g_caches.erase(c);
  c->magic = 0;
  {
    DeviceScope scope(c->device);
    cudaStreamSynchronize(c->stream);
    cudaFree(c->keys); cudaFree(c->values); cudaFree(c->lengths_dev); cudaFree(c->mask_dev);
    cudaStreamDestroy(c->stream);
  }
  delete c;
  *slot = nullptr;
  return ok(error);
}

int32_t et_a2_kv_cache_transaction_begin_v1(et_a2_kv_cache* handle, uint64_t width,
                                            const et_kernel_tensor_view_v1* counts_view,
                                            et_a2_kv_cache_transaction** out,
                                            et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.transaction-begin";
  if (!error_writable(error)) return raw_reject();
  et_a2_kv_cache* c = find_cache(handle);
  if (int r = output_slot_ok(out, error, op)) return r;
  if (*out != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "output slot must contain NULL");
  if (c == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "cache handle is invalid");
  if (c->active_transaction != nullptr || c->active_borrow != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "cache already has a live lease");
  if (width == 0 || width > SIZE_MAX)
    return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "append width must be positive");
  const size_t shape[1] = {c->batch};
  bool dev = false;
  if (int r = validate_view(counts_view, "i64", 1, shape, sizeof(int64_t), Where::kCpu, &dev,
                            error, op))
    return r;
  if (overlaps(out, sizeof(*out), counts_view, sizeof(*counts_view)) ||
      overlaps(out, sizeof(*out), counts_view->shape, sizeof(*counts_view->shape)) ||
      overlaps(out, sizeof(*out), counts_view->data, counts_view->byte_length))
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                "transaction output aliases append-count input");
  const int64_t* counts = static_cast<const int64_t*>(counts_view->data);
  bool any = false;
  for (size_t i = 0; i < c->batch; i++) {
    if (counts[i] < 0)
      return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                  "append count is negative");
    const uint64_t count = (uint64_t)counts[i];
    if (count > width)
      return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                  "append count exceeds width");
    if ((uint64_t)c->lengths[i] > UINT64_MAX - count ||
        (uint64_t)c->lengths[i] + count > c->capacity)
      return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INTEGER_OVERFLOW, op,
                  "append exceeds cache capacity");
    any = any || count != 0;
  }
  if (!any)
    return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "at least one append count must be positive");
  auto* t = new et_a2_kv_cache_transaction{};
  t->cache = c;
  t->append_width = (size_t)width;
  t->counts.assign(counts, counts + c->batch);
  t->staged.assign(c->layers, 0);
  std::vector<int64_t> effective(c->batch);
  for (size_t i = 0; i < c->batch; i++) effective[i] = c->lengths[i] + counts[i];
  DeviceScope scope(c->device);
  const size_t lb = c->batch * sizeof(int64_t);
  cudaError_t st = cudaMalloc(&t->counts_dev, lb);
  if (st == cudaSuccess) st = cudaMalloc(&t->old_lengths_dev, lb);
  if (st == cudaSuccess) st = cudaMalloc(&t->lengths_dev, lb);
  if (st == cudaSuccess) st = cudaMalloc(&t->mask_dev, c->batch * c->capacity);
  if (st == cudaSuccess)
    st = cudaMemcpyAsync(t->counts_dev, t->counts.data(), lb, cudaMemcpyHostToDevice, c->stream);
  if (st == cudaSuccess)
    st = cudaMemcpyAsync(t->old_lengths_dev, c->lengths.data(), lb, cudaMemcpyHostToDevice,
                         c->stream);
  if (st == cudaSuccess)
    st = cudaMemcpyAsync(t->lengths_dev, effective.data(), lb, cudaMemcpyHostToDevice, c->stream);
  if (st == cudaSuccess) {
    const int64_t total = (int64_t)(c->batch * c->capacity);
    kv_mask_kernel<<<grid_of(total), 256, 0, c->stream>>>(t->mask_dev, t->lengths_dev,
                                                         (int64_t)c->batch,
                                                         (int64_t)c->capacity);
    etb::count_launch();
    st = cudaStreamSynchronize(c->stream);  // the host vectors are copied from
  }
  if (st == cudaSuccess) st = cudaGetLastError();
  if (st != cudaSuccess) {
    cudaFree(t->counts_dev); cudaFree(t->old_lengths_dev); cudaFree(t->lengths_dev);
    cudaFree(t->mask_dev);
    delete t;
    cudaGetLastError();
    return fail(error, ET_KERNEL_ERROR_INTERNAL, ET_KERNEL_CODE_ALLOCATION_FAILED, op,
                "transaction allocation failed");
  }
  t->magic = kTxnMagic;
  g_txns.insert(t);
  c->active_transaction = t;
  *out = t;
  return ok(error);
}

int32_t et_a2_kv_cache_transaction_stage_layer_v1(et_a2_kv_cache_transaction* handle,
                                                  uint64_t layer,
                                                  const et_kernel_tensor_view_v1* keys,
                                                  const et_kernel_tensor_view_v1* values,
                                                  et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.stage-layer";
  if (!error_writable(error)) return raw_reject();
  et_a2_kv_cache_transaction* t = find_txn(handle);
  if (t == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "transaction handle is invalid");
  et_a2_kv_cache* c = t->cache;
  if (t->active_view != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "transaction view is live");
  if (layer >= c->layers)
    return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "layer is out of range");
  if (t->staged[layer])
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_DUPLICATE_ENTRY, op,
                "layer was already staged");
  const size_t shape[4] = {c->batch, c->kv_heads, t->append_width, c->head_dimension};
  bool kdev = false, vdev = false;
  if (int r = validate_view(keys, "f32", 4, shape, sizeof(float), Where::kEither, &kdev, error,
                            op))
    return r;
  if (int r = validate_view(values, "f32", 4, shape, sizeof(float), Where::kEither, &vdev, error,
                            op))
    return r;
  const size_t bytes = keys->byte_length;
  if ((kdev == vdev && overlaps(keys->data, bytes, values->data, bytes)) ||
      overlaps(keys, sizeof(*keys), values, sizeof(*values)) ||
      (!kdev && (overlaps(keys->data, bytes, values, sizeof(*values)) ||
                 overlaps(keys->data, bytes, values->shape, 4 * sizeof(*values->shape)))) ||
      (!vdev && (overlaps(values->data, bytes, keys, sizeof(*keys)) ||
                 overlaps(values->data, bytes, keys->shape, 4 * sizeof(*keys->shape)))))
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                "key and value sources alias");
  DeviceScope scope(c->device);
  const size_t n = bytes / sizeof(float);
  const float* sk = static_cast<const float*>(keys->data);
  const float* sv = static_cast<const float*>(values->data);
  // every source element, padding included, must be finite
  if (!kdev)
    for (size_t i = 0; i < n; i++)
      if (!isfinite(sk[i]))
        return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                    "key and value sources must be finite f32");
  if (!vdev)
    for (size_t i = 0; i < n; i++)
      if (!isfinite(sv[i]))
        return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                    "key and value sources must be finite f32");
  cudaError_t st = cudaSuccess;
  if (kdev || vdev) {
    // Device sources are read like a CPU call reads host memory: once every
    // kernel and copy already enqueued on this device, on any stream, has
    // finished (the caller may have produced them on its own stream just
    // before this call; the cache's stream is not ordered after it).
    st = cudaDeviceSynchronize();
    // then a device finite check (one flag word in the staging area)
    if (st == cudaSuccess && t->staging == nullptr) st = cudaMalloc(&t->staging, 2 * bytes + 16);
    int* flag = t->staging ? reinterpret_cast<int*>(t->staging + 2 * n) : nullptr;
    int bad = 0;
    if (st == cudaSuccess) st = cudaMemsetAsync(flag, 0, sizeof(int), c->stream);
    if (st == cudaSuccess && kdev) etb::check_finite(sk, n, flag, c->stream);
    if (st == cudaSuccess && vdev) etb::check_finite(sv, n, flag, c->stream);
    if (st == cudaSuccess)
      st = cudaMemcpyAsync(&bad, flag, sizeof(int), cudaMemcpyDeviceToHost, c->stream);
    if (st == cudaSuccess) st = cudaStreamSynchronize(c->stream);
    if (st != cudaSuccess) return cuda_fail(error, op, st);
    if (bad)
      return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                  "key and value sources must be finite f32");
  }
  if ((!kdev || !vdev) && t->staging == nullptr) st = cudaMalloc(&t->staging, 2 * bytes + 16);
  if (st != cudaSuccess) return cuda_fail(error, op, st);
  const float* dk = sk;
  const float* dv = sv;
  if (!kdev) {
    st = cudaMemcpyAsync(t->staging, sk, bytes, cudaMemcpyHostToDevice, c->stream);
    dk = t->staging;
  }
  if (st == cudaSuccess && !vdev) {
    st = cudaMemcpyAsync(t->staging + n, sv, bytes, cudaMemcpyHostToDevice, c->stream);
    dv = t->staging + n;
  }
  if (st == cudaSuccess) {
    const int64_t total = (int64_t)n;
    kv_copy_kernel<<<grid_of(total), 256, 0, c->stream>>>(
        c->keys + layer * c->layer_elements, c->values + layer * c->layer_elements, dk, dv,
        t->counts_dev, t->old_lengths_dev, (int64_t)c->batch, (int64_t)c->kv_heads,
        (int64_t)t->append_width, (int64_t)c->capacity, (int64_t)c->head_dimension);
    etb::count_launch();
    st = cudaStreamSynchronize(c->stream);  // sources are only borrowed for this call
  }
  if (st == cudaSuccess) st = cudaGetLastError();
  if (st != cudaSuccess) return cuda_fail(error, op, st);
  t->staged[layer] = 1;
  return ok(error);
}

int32_t et_a2_kv_cache_transaction_view_begin_v1(et_a2_kv_cache_transaction* handle,
                                                 uint64_t layer,
                                                 et_a2_kv_cache_transaction_view** out,
                                                 et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.transaction-view-begin";
  if (!error_writable(error)) return raw_reject();
  et_a2_kv_cache_transaction* t = find_txn(handle);
  if (int r = output_slot_ok(out, error, op)) return r;
  if (*out != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "output slot must contain NULL");
  if (t == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "transaction handle is invalid");
  if (t->active_view != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "transaction view is already live");
  if (layer >= t->cache->layers || !t->staged[layer])
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "layer is not staged");
  auto* v = new et_a2_kv_cache_transaction_view{};
  v->magic = kViewMagic;
  v->transaction = t;
  v->layer = (size_t)layer;
  fill_views(t->cache, v->layer, t->lengths_dev, t->mask_dev, v->tensor_shape, v->lengths_shape,
             v->mask_shape, &v->keys, &v->values, &v->lengths, &v->key_keep_mask);
  g_views.insert(v);
  t->active_view = v;
  *out = v;
  return ok(error);
}

namespace {
int descriptor_slots_ok(const void* a, const void* b, const void* c, const void* d,
                        et_kernel_error* e, const char* op) {
  if (int r = output_slot_ok(a, e, op)) return r;
  if (int r = output_slot_ok(b, e, op)) return r;
  if (int r = output_slot_ok(c, e, op)) return r;
  if (int r = output_slot_ok(d, e, op)) return r;
  const void* s[4] = {a, b, c, d};
  for (int i = 0; i < 4; i++)
    for (int j = i + 1; j < 4; j++)
      if (overlaps(s[i], sizeof(void*), s[j], sizeof(void*)))
        return fail(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_ALIASING_OUTPUT, op,
                    "output slots alias");
  return 0;
}
}  // namespace

int32_t et_a2_kv_cache_transaction_view_tensors_v1(
    const et_a2_kv_cache_transaction_view* handle, const et_kernel_tensor_view_v1** keys,
    const et_kernel_tensor_view_v1** values, const et_kernel_tensor_view_v1** lengths,
    const et_kernel_tensor_view_v1** key_keep_mask, et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.transaction-view-tensors";
  if (!error_writable(error)) return raw_reject();
  et_a2_kv_cache_transaction_view* v = find_view(handle);
  if (int r = descriptor_slots_ok(keys, values, lengths, key_keep_mask, error, op)) return r;
  if (*keys != nullptr || *values != nullptr || *lengths != nullptr || *key_keep_mask != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "output slots must contain NULL");
  if (v == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "view handle is invalid");
  *keys = &v->keys;
  *values = &v->values;
  *lengths = &v->lengths;
  *key_keep_mask = &v->key_keep_mask;
  return ok(error);
}

int32_t et_a2_kv_cache_transaction_view_end_v1(et_a2_kv_cache_transaction_view** slot,
                                               et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.transaction-view-end";
  if (!error_writable(error)) return raw_reject();
  if (int r = output_slot_ok(slot, error, op)) return r;
  et_a2_kv_cache_transaction_view* v = find_view(*slot);
  if (v == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "view handle is invalid");
  v->transaction->active_view = nullptr;
  g_views.erase(v);
  v->magic = 0;
  delete v;
  *slot = nullptr;
  return ok(error);
}

int32_t et_a2_kv_cache_transaction_commit_v1(et_a2_kv_cache_transaction** slot,
                                             et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.transaction-commit";
  if (!error_writable(error)) return raw_reject();
  if (int r = output_slot_ok(slot, error, op)) return r;
  et_a2_kv_cache_transaction* t = find_txn(*slot);
  if (t == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "transaction handle is invalid");
  if (t->active_view != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "transaction view is live");
  for (size_t i = 0; i < t->cache->layers; i++)
    if (!t->staged[i])
      return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                  "not every layer is staged");
  et_a2_kv_cache* c = t->cache;
  DeviceScope scope(c->device);
  cudaError_t st = cudaMemcpyAsync(c->lengths_dev, t->lengths_dev, c->batch * sizeof(int64_t),
                                   cudaMemcpyDeviceToDevice, c->stream);
  if (st == cudaSuccess)
    st = cudaMemcpyAsync(c->mask_dev, t->mask_dev, c->batch * c->capacity,
                         cudaMemcpyDeviceToDevice, c->stream);
  if (st == cudaSuccess) st = cudaStreamSynchronize(c->stream);
  if (st != cudaSuccess) return cuda_fail(error, op, st);
  for (size_t i = 0; i < c->batch; i++) c->lengths[i] += t->counts[i];
  free_txn(t);
  *slot = nullptr;
  return ok(error);
}

int32_t et_a2_kv_cache_transaction_abort_v1(et_a2_kv_cache_transaction** slot,
                                            et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.transaction-abort";
  if (!error_writable(error)) return raw_reject();
  if (int r = output_slot_ok(slot, error, op)) return r;
  et_a2_kv_cache_transaction* t = find_txn(*slot);
  if (t == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "transaction handle is invalid");
  if (t->active_view != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "transaction view is live");
  et_a2_kv_cache* c = t->cache;
  DeviceScope scope(c->device);
  // every staged append slot back to +0
  const int64_t total =
      (int64_t)(c->batch * c->kv_heads * t->append_width * c->head_dimension);
  for (size_t l = 0; l < c->layers; l++) {
    if (!t->staged[l]) continue;
    kv_copy_kernel<<<grid_of(total), 256, 0, c->stream>>>(
        c->keys + l * c->layer_elements, c->values + l * c->layer_elements, nullptr, nullptr,
        t->counts_dev, t->old_lengths_dev, (int64_t)c->batch, (int64_t)c->kv_heads,
        (int64_t)t->append_width, (int64_t)c->capacity, (int64_t)c->head_dimension);
    etb::count_launch();
  }
  cudaError_t st = cudaStreamSynchronize(c->stream);
  if (st == cudaSuccess) st = cudaGetLastError();
  if (st != cudaSuccess) return cuda_fail(error, op, st);
  free_txn(t);
  *slot = nullptr;
  return ok(error);
}

int32_t et_a2_kv_cache_read_borrow_begin_v1(et_a2_kv_cache* handle,
                                            et_a2_kv_cache_read_borrow** out,
                                            et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.read-borrow-begin";
  if (!error_writable(error)) return raw_reject();
  et_a2_kv_cache* c = find_cache(handle);
  if (int r = output_slot_ok(out, error, op)) return r;
  if (*out != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "output slot must contain NULL");
  if (c == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "cache handle is invalid");
  if (c->active_transaction != nullptr || c->active_borrow != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                "cache already has a live lease");
  auto* b = new et_a2_kv_cache_read_borrow{};
  b->magic = kBorrowMagic;
  b->cache = c;
  b->keys.resize(c->layers);
  b->values.resize(c->layers);
  for (size_t l = 0; l < c->layers; l++)
    fill_views(c, l, c->lengths_dev, c->mask_dev, b->tensor_shape, b->lengths_shape,
               b->mask_shape, &b->keys[l], &b->values[l], &b->lengths, &b->key_keep_mask);
  g_borrows.insert(b);
  c->active_borrow = b;
  *out = b;
  return ok(error);
}

int32_t et_a2_kv_cache_read_borrow_layer_v1(et_a2_kv_cache_read_borrow* handle, uint64_t layer,
                                            const et_kernel_tensor_view_v1** keys,
                                            const et_kernel_tensor_view_v1** values,
                                            const et_kernel_tensor_view_v1** lengths,
                                            const et_kernel_tensor_view_v1** key_keep_mask,
                                            et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.read-borrow-layer";
  if (!error_writable(error)) return raw_reject();
  et_a2_kv_cache_read_borrow* b = find_borrow(handle);
  if (int r = descriptor_slots_ok(keys, values, lengths, key_keep_mask, error, op)) return r;
  if (*keys != nullptr || *values != nullptr || *lengths != nullptr || *key_keep_mask != nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "output slots must contain NULL");
  if (b == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "read borrow handle is invalid");
  if (layer >= b->cache->layers)
    return fail(error, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                "layer is out of range");
  *keys = &b->keys[layer];
  *values = &b->values[layer];
  *lengths = &b->lengths;
  *key_keep_mask = &b->key_keep_mask;
  return ok(error);
}

int32_t et_a2_kv_cache_read_borrow_end_v1(et_a2_kv_cache_read_borrow** slot,
                                          et_kernel_error* error) {
  std::lock_guard<std::mutex> lock(g_mu);
  const char* op = "a2-kv-cache.read-borrow-end";
  if (!error_writable(error)) return raw_reject();
  if (int r = output_slot_ok(slot, error, op)) return r;
  et_a2_kv_cache_read_borrow* b = find_borrow(*slot);
  if (b == nullptr)
    return fail(error, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_INVALID_BUFFER, op,
                "read borrow handle is invalid");
  b->cache->active_borrow = nullptr;
  g_borrows.erase(b);
  b->magic = 0;
  delete b;
  *slot = nullptr;
  return ok(error);
}

}  // extern "C"
