// Library-wide state and small C entry points: ABI version, the launch
// counter, the device check, the device error word and the seeded synthetic
// input generators.
#include <math.h>

#include <mutex>
#include <vector>

#include "ops.cuh"

namespace etb {

std::atomic<uint64_t> g_launches{0};

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 1;
  }
  return cache[dev];
}

// One device word per GPU that bounded device-side waits set when they give
// up (instead of hanging); host entry points read and clear it.
int* device_error_word() {
  static std::mutex mu;
  static std::vector<int*> words;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if ((int)words.size() <= dev) words.resize(dev + 1, nullptr);
  if (words[dev] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) {
      cudaMemset(p, 0, sizeof(int));
      words[dev] = p;
    }
  }
  return words[dev];
}

// ---- synthetic inputs (same definition as the test oracle) ------------------

static uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}
static uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return splitmix64(seed) ^ splitmix64(stream * 0x632be59bd9b4e019ull + 1u);
}
static uint64_t stream_word(uint64_t key, uint64_t counter) {
  return splitmix64(key + counter * 0x9e3779b97f4a7c15ull);
}

}  // namespace etb

extern "C" {

int32_t et_b200_abi_major_v1(void) { return (int32_t)ET_B200_ABI_MAJOR; }
int32_t et_b200_abi_minor_v1(void) { return (int32_t)ET_B200_ABI_MINOR; }

uint64_t et_b200_launch_count_v1(void) { return etb::g_launches.load(); }

int32_t et_b200_device_check_v1(et_kernel_error* error) {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return etb::cuda_error(error, st, "device-check");
  cudaDeviceProp prop;
  st = cudaGetDeviceProperties(&prop, dev);
  if (st != cudaSuccess) return etb::cuda_error(error, st, "device-check");
  if (prop.major != 10 || prop.minor != 0)
    return etb::set_error(error, ET_KERNEL_ERROR_DEVICE_MISMATCH, ET_KERNEL_CODE_PROVIDER_REJECTED,
                          "device-check", "libet_b200 is built for sm_100a (B200) only");
  if (error) memset(error, 0, sizeof(*error));
  return 0;
}

void et_b200_fill_normal_v1(uint64_t seed, uint64_t stream, size_t count, double mean,
                            double stddev, float* out) {
  const uint64_t key = etb::stream_key(seed, stream);
  const double two_pi = 6.283185307179586476925286766559;
  for (size_t i = 0; i < count; i++) {
    const uint64_t a = etb::stream_word(key, 2u * (uint64_t)i);
    const uint64_t b = etb::stream_word(key, 2u * (uint64_t)i + 1u);
    const double u1 = (double)((a >> 11) + 1u) * 0x1p-53;
    const double u2 = (double)(b >> 11) * 0x1p-53;
    const double z = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
    out[i] = (float)(mean + stddev * z);
  }
}

void et_b200_fill_tokens_v1(uint64_t seed, uint64_t stream, size_t count, uint64_t vocabulary,
                            int64_t* out) {
  const uint64_t key = etb::stream_key(seed, stream);
  const uint64_t limit = (UINT64_MAX / vocabulary) * vocabulary;
  for (size_t i = 0; i < count; i++) {
    for (uint64_t attempt = 0;; attempt++) {
      const uint64_t x = etb::stream_word(key, (uint64_t)i | (attempt << 40));
      if (x < limit) {
        out[i] = (int64_t)(x % vocabulary);
        break;
      }
    }
  }
}

}  // extern "C"
