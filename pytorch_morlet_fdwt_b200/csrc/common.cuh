// Shared helpers of the sm_100a wavelet kernels: status handling, element types, boundary
// index maps, padded shared-memory indexing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fdwt_b200.h"

namespace fdwt {

// ------------------------------------------------------------------------------ status
void set_cuda_error(cudaError_t e);
// Every kernel launch of the library is counted (fdwt_launch_count()).
void count_launch();

#define FDWT_CUDA(call)                 \
  do {                                  \
    cudaError_t e_ = (call);            \
    if (e_ != cudaSuccess) {            \
      ::fdwt::set_cuda_error(e_);       \
      return FDWT_ERR_CUDA;             \
    }                                   \
  } while (0)

#define FDWT_CHECK(cond)                \
  do {                                  \
    if (!(cond)) return FDWT_ERR_INVALID; \
  } while (0)

inline int launch_status() {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return FDWT_ERR_CUDA;
  }
  return FDWT_OK;
}

// Opt-in dynamic shared memory limit of the current device (cached per device).
int max_smem_optin();
int sm_count();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize = device opt-in limit), cached per
// (kernel, device).
int allow_max_dynamic_smem(const void* kernel);
// Resident blocks per SM of `kernel` at `threads` threads and `smem` dynamic shared bytes on
// the current device (cudaOccupancyMaxActiveBlocksPerMultiprocessor, cached per key).
int occupancy(const void* kernel, int threads, size_t smem, int* blocks);
// Called before every kernel launch: runs the shared-memory fill kernel of the test hook
// fdwt_set_shared_memory_fill when it is enabled (FDWT_OK and nothing otherwise).
int pre_launch(cudaStream_t stream);
// Device address of the current device's error word (0: no error).  A kernel whose bounded
// wait on an asynchronous copy runs out stores a nonzero code there and returns early;
// fdwt_device_error() reads and clears it.
int* device_error_flag();
constexpr int kErrCopyTimeout = 1;
// Poll limit of every bounded mbarrier wait of the streaming kernels.
constexpr long long kCopyWaitTries = 1LL << 22;
// Test hook of those waits (fdwt_set_copy_wait_test): `extra_tx` bytes the kernels add to the
// expected transaction count of the copy of global tile 0 (its wait then runs out while every
// issued copy still completes), and the poll limit of the main waits (`tries`).  The wait for
// copies still in flight after a timeout polls max(tries, 2^20) times.  {0, kCopyWaitTries}
// unless a test set them.
struct CopyWaitTest {
  unsigned extra_tx;
  long long tries;
};
CopyWaitTest copy_wait_test();
// Test hook of the Morlet kernels (fdwt_set_cwt_tile_test): when > 0, the forward and backward
// passes run on time tiles of that many positions even where whole rows would fit.
int cwt_tile_test();

// ------------------------------------------------------------------------------ types
template <typename T> struct AccOf { using type = float; };
template <> struct AccOf<double> { using type = double; };

template <typename T> __device__ __forceinline__ typename AccOf<T>::type to_acc(T v) {
  return static_cast<typename AccOf<T>::type>(v);
}
template <> __device__ __forceinline__ float to_acc<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_acc<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_acc(typename AccOf<T>::type v) {
  return static_cast<T>(v);
}
template <> __device__ __forceinline__ __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// ------------------------------------------------------------------------------ index maps
// Python-style floor division / modulo for signed 64-bit ints.
__host__ __device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b) {
  int64_t q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}
__host__ __device__ __forceinline__ int64_t pos_mod(int64_t a, int64_t b) {
  if (a >= INT32_MIN && a <= INT32_MAX && b <= INT32_MAX) {  // 32-bit: a short sequence
    int32_t r = static_cast<int32_t>(a) % static_cast<int32_t>(b);
    return r < 0 ? r + b : r;
  }
  int64_t r = a % b;
  return r < 0 ? r + b : r;
}

// reflect on a single sample degenerates to a constant (period-1) extension
__host__ __device__ __forceinline__ int normalize_mode(int mode, int64_t n) {
  return (mode == FDWT_MODE_REFLECT && n == 1) ? FDWT_MODE_PERIODIC : mode;
}

__host__ __device__ __forceinline__ int64_t mode_period(int mode, int64_t n) {
  switch (mode) {
    case FDWT_MODE_PERIODIC: return n;
    case FDWT_MODE_SYMMETRIC: return 2 * n;
    case FDWT_MODE_REFLECT: return 2 * n - 2;
    case FDWT_MODE_PERIODIZATION: return n + (n & 1);
    default: return 1;
  }
}

// Map an extended position p onto [0, n) for a (normalized) mode; returns -1 when the
// position is outside the signal in zero mode.
__host__ __device__ __forceinline__ int64_t ext_index(int64_t p, int64_t n, int mode, int64_t P) {
  if (p >= 0 && p < n) return p;
  if (mode == FDWT_MODE_ZERO) return -1;
  // one wrap covers every extended position of signals longer than the filter; the modulo
  // (a long dependent sequence for 64-bit operands) is left to the rare multi-wrap case
  int64_t q = p < 0 ? p + P : (p >= P ? p - P : p);
  if (q < 0 || q >= P) q = pos_mod(p, P);
  switch (mode) {
    case FDWT_MODE_PERIODIC: return q;
    case FDWT_MODE_SYMMETRIC: return q < n ? q : P - 1 - q;
    case FDWT_MODE_REFLECT: return q < n ? q : P - q;
    default: return q < n - 1 ? q : n - 1;  // periodization: odd lengths repeat the last sample
  }
}

// Padded shared-memory index: one spare element after every 2^PS elements, so that lanes
// reading windows spaced 2^PS elements apart hit distinct banks.
template <int PS> __host__ __device__ __forceinline__ int sidx(int e) { return e + (e >> PS); }
template <int PS> __host__ __device__ __forceinline__ int64_t padded_len(int64_t n) {
  return n + (n >> PS) + 1;
}

__host__ __device__ __forceinline__ int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t imax(int64_t a, int64_t b) { return a > b ? a : b; }

inline size_t dtype_size(int dtype) {
  switch (dtype) {
    case FDWT_F32: return 4;
    case FDWT_F64: return 8;
    case FDWT_F16: return 2;
    case FDWT_BF16: return 2;
    default: return 0;
  }
}

}  // namespace fdwt
