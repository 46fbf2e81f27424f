// C ABI of the fused multilevel DWT (kernels in dwt_impl.cuh, instantiated per dtype in
// dwt_f32.cu / dwt_f64.cu / dwt_f16.cu / dwt_bf16.cu).
#include <mutex>

#include "dwt_impl.cuh"

namespace fdwt {
namespace dwtk {
namespace {

template <bool ANA, typename... Args>
int dispatch(int dtype, int LM, Args... args) {
  switch (dtype) {
    case FDWT_F32:
      return ANA ? analysis_dtype<float>(LM, args...) : synthesis_dtype<float>(LM, args...);
    case FDWT_F64:
      return ANA ? analysis_dtype<double>(LM, args...) : synthesis_dtype<double>(LM, args...);
    case FDWT_F16:
      return ANA ? analysis_dtype<__half>(LM, args...) : synthesis_dtype<__half>(LM, args...);
    case FDWT_BF16:
      return ANA ? analysis_dtype<__nv_bfloat16>(LM, args...)
                 : synthesis_dtype<__nv_bfloat16>(LM, args...);
    default: return FDWT_ERR_INVALID;
  }
}

// Level descriptors of an analysis call (finest first); returns FDWT_OK or an error.
int analysis_levels(int64_t n, int levels, const int64_t* coef_len, const int64_t* pad_last,
                    int mode, std::vector<Level>& lv, void* const* out) {
  if (levels < 1 || levels > 4096 || coef_len == nullptr) return FDWT_ERR_INVALID;
  if (mode < 0 || mode > 4) return FDWT_ERR_INVALID;
  int64_t n_in = n;
  for (int k = 0; k < levels; ++k) {
    const int64_t nc = coef_len[k];
    const int64_t pad = pad_last ? pad_last[k] : 0;
    if (n_in < 1 || nc < 0 || pad < 0 || pad > 1) return FDWT_ERR_INVALID;
    Level L{};
    L.n_in = n_in;
    L.n_coef = nc;
    L.a_len = nc + pad;
    L.mode = normalize_mode(mode, n_in);
    L.P = mode_period(L.mode, n_in);
    L.detail = out ? out[levels - k] : nullptr;
    lv.push_back(L);
    n_in = nc + pad;
  }
  return FDWT_OK;
}

int synthesis_levels(int levels, int64_t approx_len, const int64_t* coef_len,
                     const int64_t* out_len, int mode, std::vector<Level>& lv,
                     const void* const* in) {
  if (levels < 1 || levels > 4096 || coef_len == nullptr || out_len == nullptr)
    return FDWT_ERR_INVALID;
  if (mode < 0 || mode > 4) return FDWT_ERR_INVALID;
  // processing order: coarsest level (index levels-1) first
  for (int k = levels - 1; k >= 0; --k) {
    const int64_t nc = coef_len[k], n = out_len[k];
    const int64_t a_in = (k == levels - 1) ? approx_len : out_len[k + 1];
    if (nc < 1 || n < 1 || a_in < nc || a_in > nc + 1) return FDWT_ERR_INVALID;
    Level L{};
    L.n_in = n;
    L.n_coef = nc;
    L.a_len = a_in;
    L.mode = normalize_mode(mode, n);
    L.P = mode_period(L.mode, n);
    L.detail = in ? const_cast<void*>(in[levels - k]) : nullptr;
    lv.push_back(L);
  }
  return FDWT_OK;
}

// Checks the arguments of an analysis call that do not point at device data, as
// fdwt_dwt_analysis does, and stores the workspace its plan needs in *need.
int analysis_need(int dtype, int64_t rows, int64_t n, int levels, const int64_t* coef_len,
                  const int64_t* pad_last, int filter_len, int mode, int off, size_t* need) {
  *need = 0;
  if (rows < 0 || dtype < FDWT_F32 || dtype > FDWT_BF16) return FDWT_ERR_INVALID;
  if (filter_len < 2 || (filter_len & 1)) return FDWT_ERR_INVALID;
  const int LM = pick_lm(filter_len);
  if (LM < 0) return FDWT_ERR_UNSUPPORTED;
  std::vector<Level> lv;
  const int st = analysis_levels(n, levels, coef_len, pad_last, mode, lv, nullptr);
  if (st != FDWT_OK) return st;
  return dispatch<true>(dtype, LM, rows, static_cast<const void*>(nullptr), lv,
                        static_cast<void*>(nullptr), static_cast<const double*>(nullptr),
                        static_cast<const double*>(nullptr), filter_len, off,
                        static_cast<void*>(nullptr), size_t(0),
                        static_cast<cudaStream_t>(nullptr), need);
}

}  // namespace
}  // namespace dwtk
}  // namespace fdwt

using namespace fdwt::dwtk;

extern "C" int fdwt_dwt_analysis(int dtype, int64_t rows, const void* x, int64_t n, int levels,
                                 const int64_t* coef_len, const int64_t* pad_last,
                                 void* const* out, const double* h0, const double* h1,
                                 int filter_len, int mode, int off, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (rows < 0 || out == nullptr || h0 == nullptr || h1 == nullptr) return FDWT_ERR_INVALID;
  if (filter_len < 2 || (filter_len & 1)) return FDWT_ERR_INVALID;
  const int LM = pick_lm(filter_len);
  if (LM < 0) return FDWT_ERR_UNSUPPORTED;
  std::vector<Level> lv;
  int st = analysis_levels(n, levels, coef_len, pad_last, mode, lv, out);
  if (st != FDWT_OK) return st;
  if (rows > 0) {
    if (x == nullptr || out[0] == nullptr) return FDWT_ERR_INVALID;
    for (int k = 1; k <= levels; ++k)
      if (out[k] == nullptr) return FDWT_ERR_INVALID;
  }
  return dispatch<true>(dtype, LM, rows, x, lv, out[0], h0, h1, filter_len, off, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream),
                          static_cast<size_t*>(nullptr));
}

extern "C" size_t fdwt_dwt_analysis_workspace(int dtype, int64_t rows, int64_t n, int levels,
                                              const int64_t* coef_len, const int64_t* pad_last,
                                              int filter_len, int mode, int off) {
  size_t need = 0;
  if (analysis_need(dtype, rows, n, levels, coef_len, pad_last, filter_len, mode, off, &need) !=
      FDWT_OK)
    return 0;
  return need;
}

extern "C" int fdwt_dwt_synthesis(int dtype, int64_t rows, int levels, const void* const* in,
                                  int64_t approx_len, const int64_t* coef_len,
                                  const int64_t* out_len, void* y, const double* h0,
                                  const double* h1, int filter_len, int mode, int off,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || in == nullptr || h0 == nullptr || h1 == nullptr) return FDWT_ERR_INVALID;
  if (filter_len < 2 || (filter_len & 1)) return FDWT_ERR_INVALID;
  const int LM = pick_lm(filter_len);
  if (LM < 0) return FDWT_ERR_UNSUPPORTED;
  std::vector<Level> lv;
  int st = synthesis_levels(levels, approx_len, coef_len, out_len, mode, lv, in);
  if (st != FDWT_OK) return st;
  if (rows > 0 && (in[0] == nullptr || y == nullptr)) return FDWT_ERR_INVALID;
  return dispatch<false>(dtype, LM, rows, in[0], lv, y, h0, h1, filter_len, off, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream),
                          static_cast<size_t*>(nullptr));
}

extern "C" size_t fdwt_dwt_synthesis_workspace(int dtype, int64_t rows, int levels,
                                               int64_t approx_len, const int64_t* coef_len,
                                               const int64_t* out_len, int filter_len, int mode,
                                               int off) {
  const int LM = pick_lm(filter_len);
  if (LM < 0 || rows < 0) return 0;
  std::vector<Level> lv;
  if (synthesis_levels(levels, approx_len, coef_len, out_len, mode, lv, nullptr) != FDWT_OK)
    return 0;
  size_t need = 0;
  dispatch<false>(dtype, LM, rows, static_cast<const void*>(nullptr), lv,
                   static_cast<void*>(nullptr), static_cast<const double*>(nullptr),
                   static_cast<const double*>(nullptr), filter_len, off,
                   static_cast<void*>(nullptr), size_t(0), static_cast<cudaStream_t>(nullptr),
                   &need);
  return need;
}

// ------------------------------------------------------------------------------------------
// Allocation-free analysis.  Some callers cannot allocate device memory once they are running:
// a real-time acquisition loop where cudaMalloc/cudaFree would synchronise the device and stall
// its other streams, or a host application whose own allocator owns the device and whose FFI
// has no way to hand this library a workspace buffer.  fdwt_dwt_analysis_noalloc serves them:
// the workspace that long rows need (the approximation handed from one launch to the next) is
// a fixed array compiled into this file, which every GPU that loads the library holds until
// the process exits.
// ------------------------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // FDWT_NOALLOC_SCRATCH_BYTES
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  In host code the array's name is
// only a host-side stand-in, so the address comes from cudaGetSymbolAddress, looked up once per
// device with that device current (the first call on each device) and cached.
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[kNoAllocMaxDevices] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    fdwt::set_cuda_error(e);
    return FDWT_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return FDWT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      fdwt::set_cuda_error(e);
      return FDWT_ERR_CUDA;
    }
    if (p == nullptr) return FDWT_ERR_CUDA;
    addr[dev] = p;
  }
  *out = addr[dev];
  return FDWT_OK;
}

}  // namespace

extern "C" int fdwt_dwt_analysis_noalloc(int dtype, int64_t rows, const void* x, int64_t n,
                                         int levels, const int64_t* coef_len,
                                         const int64_t* pad_last, void* const* out,
                                         const double* h0, const double* h1, int filter_len,
                                         int mode, int off, void* stream) {
  if (out == nullptr || h0 == nullptr || h1 == nullptr) return FDWT_ERR_INVALID;
  // one validation of the arguments, which also sizes the plan's workspace (it covers every
  // plan the call may take at run time, e.g. the one for an x that is not 16-byte aligned)
  size_t need = 0;
  const int st = analysis_need(dtype, rows, n, levels, coef_len, pad_last, filter_len, mode, off,
                               &need);
  if (st != FDWT_OK) return st;
  if (need > kNoAllocScratchBytes) return FDWT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    const int sc = noalloc_scratch(&scratch);
    if (sc != FDWT_OK) return sc;
  }
  // Every element of a handover region is written by one launch before the next launch reads
  // it, so nothing left in the array by an earlier call needs clearing.
  return fdwt_dwt_analysis(dtype, rows, x, n, levels, coef_len, pad_last, out, h0, h1,
                           filter_len, mode, off, scratch, scratch ? kNoAllocScratchBytes : 0,
                           stream);
}
