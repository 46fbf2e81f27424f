// Library-wide C ABI helpers: status strings, per-thread CUDA error, device attributes.
#include <atomic>
#include <map>
#include <tuple>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace fdwt {

static thread_local int g_last_cuda_error = 0;
static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

int max_smem_optin() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 48 * 1024;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      v = 48 * 1024;
    cache[dev] = v;
  }
  return cache[dev];
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

int occupancy(const void* kernel, int threads, size_t smem, int* blocks) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t, int>, int> cache;
  int dev = 0;
  FDWT_CUDA(cudaGetDevice(&dev));
  const auto key = std::make_tuple(kernel, threads, smem, dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) {
      *blocks = it->second;
      return FDWT_OK;
    }
  }
  int v = 0;
  FDWT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, threads, smem));
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = v;
  *blocks = v;
  return FDWT_OK;
}

int allow_max_dynamic_smem(const void* kernel) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  FDWT_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return FDWT_OK;
  cudaFuncAttributes fa{};
  FDWT_CUDA(cudaFuncGetAttributes(&fa, kernel));
  FDWT_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 max_smem_optin() - static_cast<int>(fa.sharedSizeBytes)));
  done.insert({kernel, dev});
  return FDWT_OK;
}

}  // namespace fdwt

extern "C" const char* fdwt_status_string(int status) {
  switch (status) {
    case FDWT_OK: return "ok";
    case FDWT_ERR_INVALID: return "invalid argument";
    case FDWT_ERR_UNSUPPORTED: return "unsupported configuration";
    case FDWT_ERR_WORKSPACE: return "workspace missing or too small";
    case FDWT_ERR_CUDA: return "CUDA runtime error";
    case FDWT_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the static no-allocation array holds";
    default: return "unknown status";
  }
}

extern "C" int fdwt_last_cuda_error(void) { return fdwt::g_last_cuda_error; }

extern "C" int fdwt_version(void) { return 100; }

extern "C" unsigned long long fdwt_launch_count(void) {
  return fdwt::g_launches.load(std::memory_order_relaxed);
}

namespace {
// One CTA per SM at the largest dynamic shared-memory size, every word set to `word`.
__global__ void fill_shared_kernel(unsigned word, int words) {
  extern __shared__ unsigned fill_smem[];
  volatile unsigned* s = fill_smem;
  for (int i = threadIdx.x; i < words; i += blockDim.x) s[i] = word;
}
std::atomic<int> g_fill_enabled{0};
std::atomic<unsigned> g_fill_word{0u};
}  // namespace

namespace fdwt {
int pre_launch(cudaStream_t stream) {
  if (!g_fill_enabled.load(std::memory_order_relaxed)) return FDWT_OK;
  const int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(fill_shared_kernel));
  if (st != FDWT_OK) return st;
  const int bytes = max_smem_optin();
  fill_shared_kernel<<<2 * sm_count(), 1024, bytes, stream>>>(
      g_fill_word.load(std::memory_order_relaxed), bytes / 4);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return FDWT_ERR_CUDA;
  }
  return FDWT_OK;
}
}  // namespace fdwt

namespace {
// Set (to a nonzero code) by a kernel whose bounded wait on an asynchronous copy ran out.
__device__ int g_device_error;
}  // namespace

namespace fdwt {
// The address is looked up once per device (with that device current) under a lock and kept:
// like every per-device cache of this library it assumes the device's primary context lives
// as long as the process (no cudaDeviceReset between calls).
int* device_error_flag() {
  static std::mutex mu;
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

static std::atomic<unsigned> g_wait_extra_tx{0};
static std::atomic<long long> g_wait_tries{kCopyWaitTries};

CopyWaitTest copy_wait_test() {
  return {g_wait_extra_tx.load(std::memory_order_relaxed),
          g_wait_tries.load(std::memory_order_relaxed)};
}
}  // namespace fdwt

static std::atomic<int> g_cwt_tile_test{0};
int fdwt::cwt_tile_test() { return g_cwt_tile_test.load(std::memory_order_relaxed); }

extern "C" void fdwt_set_cwt_tile_test(int t_len) {
  g_cwt_tile_test.store(t_len > 0 ? t_len : 0, std::memory_order_relaxed);
}

extern "C" void fdwt_set_copy_wait_test(unsigned extra_tx_bytes, long long tries) {
  fdwt::g_wait_extra_tx.store(extra_tx_bytes, std::memory_order_relaxed);
  fdwt::g_wait_tries.store(tries > 0 ? tries : fdwt::kCopyWaitTries, std::memory_order_relaxed);
}

extern "C" int fdwt_device_error(int* code) {
  if (code == nullptr) return FDWT_ERR_INVALID;
  int v = 0;
  FDWT_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  if (v != 0) {
    const int zero = 0;
    FDWT_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  }
  *code = v;
  return FDWT_OK;
}

extern "C" void fdwt_set_shared_memory_fill(int enable, unsigned int word) {
  g_fill_word.store(word, std::memory_order_relaxed);
  g_fill_enabled.store(enable != 0, std::memory_order_relaxed);
}
