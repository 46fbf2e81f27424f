// C ABI of the Morlet CWT pyramid kernels (cwt_impl.cuh).  The computation type follows the
// row type: fp32 rows compute in fp32, fp64 rows in fp64 (fp16/bf16 inputs are upcast to fp32
// by the caller, as the reference does at fdwt/cwt.py:606-607).
#include "cwt_impl.cuh"

using namespace fdwt;
using namespace fdwt::cwtk;

namespace {

template <int EPI>
int dispatch_forward(int dtype, int64_t rows, int64_t n, const void* x, const void* h,
                     const fdwt_morlet_plan* pl, void* y, const void* a, const void* b,
                     void* m, void* l, int64_t dim, int v_pos, double inv_tau,
                     cudaStream_t stream) {
  switch (dtype) {
    case FDWT_F32:
      return run_forward<float, float, EPI>(rows, n, x, h, pl, y, a, b, m, l, dim, v_pos, inv_tau,
                                            stream);
    case FDWT_F64:
      return run_forward<double, double, EPI>(rows, n, x, h, pl, y, a, b, m, l, dim, v_pos,
                                              inv_tau, stream);
    default:
      return FDWT_ERR_UNSUPPORTED;
  }
}

}  // namespace

extern "C" int fdwt_cwt_forward(int dtype, int64_t rows, int64_t n, const void* x,
                                const void* filters, const fdwt_morlet_plan* plan, void* y,
                                void* stream) {
  if (rows < 0) return FDWT_ERR_INVALID;
  if (rows > 0 && (x == nullptr || filters == nullptr || y == nullptr)) return FDWT_ERR_INVALID;
  return dispatch_forward<EPI_STORE>(dtype, rows, n, x, filters, plan, y, nullptr, nullptr,
                                     nullptr, nullptr, 1, 0, 1.0,
                                     static_cast<cudaStream_t>(stream));
}

extern "C" int fdwt_mix_forward(int dtype, int64_t rows, int64_t n, const void* x,
                                const void* filters, const fdwt_morlet_plan* plan, const void* a,
                                const void* b, int64_t dim, void* y, void* stream) {
  if (rows < 0 || dim < 1) return FDWT_ERR_INVALID;
  if (rows > 0 && (x == nullptr || filters == nullptr || y == nullptr || a == nullptr ||
                   b == nullptr))
    return FDWT_ERR_INVALID;
  return dispatch_forward<EPI_MIX>(dtype, rows, n, x, filters, plan, y, a, b, nullptr, nullptr,
                                   dim, 0, 1.0, static_cast<cudaStream_t>(stream));
}

extern "C" int fdwt_specsoftmax_forward(int dtype, int64_t rows, int64_t n, const void* x,
                                        const void* filters, const fdwt_morlet_plan* plan,
                                        const void* v, int v_per_position, int64_t nch,
                                        double inv_tau, void* out, void* m, void* l,
                                        void* stream) {
  if (rows < 0 || nch < 1) return FDWT_ERR_INVALID;
  if (rows > 0 && (x == nullptr || filters == nullptr || v == nullptr || out == nullptr ||
                   m == nullptr || l == nullptr))
    return FDWT_ERR_INVALID;
  if (plan != nullptr && plan->channels != 2) return FDWT_ERR_INVALID;
  return dispatch_forward<EPI_SOFTMAX>(dtype, rows, n, x, filters, plan, out, v, nullptr, m, l,
                                       nch, v_per_position != 0, inv_tau,
                                       static_cast<cudaStream_t>(stream));
}
