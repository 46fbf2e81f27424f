// C ABI of the Morlet CWT pyramid kernels (cwt_impl.cuh, cwt_bwd.cuh, cwt_bwd_tiled.cuh).  The
// computation type follows the row type: fp32 rows compute in fp32, fp64 rows in fp64 (fp16/bf16
// inputs are upcast to fp32 by the caller, as the reference does at fdwt/cwt.py:606-607).  The
// kernels are instantiated per (type, epilogue) in cwt_<type>_<epilogue>.cu (cwt_entry.cuh).
#include "cwt_entry.cuh"

using namespace fdwt;
using namespace fdwt::cwtk;

namespace {

template <int EPI>
int dispatch_forward(int dtype, int64_t rows, int64_t n, const void* x, const void* h,
                     const fdwt_morlet_plan* pl, void* y, const void* a, const void* b,
                     void* m, void* l, int64_t dim, int v_pos, double inv_tau,
                     cudaStream_t stream, int tok = 0, const void* bias = nullptr) {
  switch (dtype) {
    case FDWT_F32:
      return fwd_entry<float, EPI>(rows, n, x, h, pl, y, a, b, m, l, dim, v_pos, inv_tau, stream,
                                   tok, bias);
    case FDWT_F64:
      return fwd_entry<double, EPI>(rows, n, x, h, pl, y, a, b, m, l, dim, v_pos, inv_tau,
                                    stream, tok, bias);
    default:
      return FDWT_ERR_UNSUPPORTED;
  }
}

template <int EPI>
int dispatch_backward(int dtype, int64_t rows, int64_t n, const void* x, const void* h,
                      const fdwt_morlet_plan* pl, const void* a, const void* b, int64_t dim,
                      int v_pos, double inv_tau, const void* g, const void* m, const void* l,
                      const void* out, void* gx, void* gh, void* ga, void* gb, void* gv,
                      bool need_h, void* ws, size_t ws_bytes, cudaStream_t stream,
                      size_t* need) {
  switch (dtype) {
    case FDWT_F32:
      return bwd_entry<float, EPI>(rows, n, x, h, pl, a, b, dim, v_pos, inv_tau, g, m, l, out,
                                   gx, gh, ga, gb, gv, need_h, ws, ws_bytes, stream, need);
    case FDWT_F64:
      return bwd_entry<double, EPI>(rows, n, x, h, pl, a, b, dim, v_pos, inv_tau, g, m, l, out,
                                    gx, gh, ga, gb, gv, need_h, ws, ws_bytes, stream, need);
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

extern "C" size_t fdwt_cwt_backward_workspace(int dtype, int64_t rows, int64_t n,
                                              const fdwt_morlet_plan* plan, int need_gh) {
  size_t need = 0;
  if (rows < 0) return 0;
  if (dispatch_backward<EPI_STORE>(dtype, rows, n, nullptr, nullptr, plan, nullptr, nullptr, 1,
                                   0, 1.0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                   nullptr, nullptr, nullptr, need_gh != 0, nullptr, 0, nullptr,
                                   &need) != FDWT_OK)
    return 0;
  return need;
}

extern "C" int fdwt_cwt_backward(int dtype, int64_t rows, int64_t n, const void* x,
                                 const void* filters, const fdwt_morlet_plan* plan,
                                 const void* gy, void* gx, void* gh, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (rows < 0) return FDWT_ERR_INVALID;
  if (rows > 0 && (filters == nullptr || gy == nullptr || (gh != nullptr && x == nullptr)))
    return FDWT_ERR_INVALID;
  return dispatch_backward<EPI_STORE>(dtype, rows, n, x, filters, plan, nullptr, nullptr, 1, 0,
                                      1.0, gy, nullptr, nullptr, nullptr, gx, gh, nullptr,
                                      nullptr, nullptr, gh != nullptr, workspace,
                                      workspace_bytes, static_cast<cudaStream_t>(stream),
                                      nullptr);
}

extern "C" size_t fdwt_mix_backward_workspace(int dtype, int64_t rows, int64_t n,
                                              const fdwt_morlet_plan* plan, int64_t dim,
                                              int need_gh) {
  size_t need = 0;
  if (rows < 0 || dim < 1) return 0;
  if (dispatch_backward<EPI_MIX>(dtype, rows, n, nullptr, nullptr, plan, nullptr, nullptr, dim,
                                 0, 1.0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                 nullptr, nullptr, nullptr, need_gh != 0, nullptr, 0, nullptr,
                                 &need) != FDWT_OK)
    return 0;
  return need;
}

extern "C" int fdwt_mix_backward(int dtype, int64_t rows, int64_t n, const void* x,
                                 const void* filters, const fdwt_morlet_plan* plan, const void* a,
                                 const void* b, int64_t dim, const void* gy, void* gx, void* gh,
                                 void* ga, void* gb, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  if (rows < 0 || dim < 1) return FDWT_ERR_INVALID;
  if (rows > 0 && (x == nullptr || filters == nullptr || a == nullptr || b == nullptr ||
                   gy == nullptr))
    return FDWT_ERR_INVALID;
  return dispatch_backward<EPI_MIX>(dtype, rows, n, x, filters, plan, a, b, dim, 0, 1.0, gy,
                                    nullptr, nullptr, nullptr, gx, gh, ga, gb, nullptr,
                                    gh != nullptr, workspace, workspace_bytes,
                                    static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" size_t fdwt_specsoftmax_backward_workspace(int dtype, int64_t rows, int64_t n,
                                                      const fdwt_morlet_plan* plan,
                                                      int v_per_position, int64_t nch,
                                                      int need_gh) {
  size_t need = 0;
  if (rows < 0 || nch < 1) return 0;
  if (dispatch_backward<EPI_SOFTMAX>(dtype, rows, n, nullptr, nullptr, plan, nullptr, nullptr,
                                     nch, v_per_position != 0, 1.0, nullptr, nullptr, nullptr,
                                     nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                     need_gh != 0, nullptr, 0, nullptr, &need) != FDWT_OK)
    return 0;
  return need;
}

extern "C" int fdwt_specsoftmax_backward(int dtype, int64_t rows, int64_t n, const void* x,
                                         const void* filters, const fdwt_morlet_plan* plan,
                                         const void* v, int v_per_position, int64_t nch,
                                         double inv_tau, const void* m, const void* l,
                                         const void* out, const void* gout, void* gx, void* gh,
                                         void* gv, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  if (rows < 0 || nch < 1) return FDWT_ERR_INVALID;
  if (rows > 0 && (x == nullptr || filters == nullptr || v == nullptr || m == nullptr ||
                   l == nullptr || out == nullptr || gout == nullptr))
    return FDWT_ERR_INVALID;
  return dispatch_backward<EPI_SOFTMAX>(dtype, rows, n, x, filters, plan, v, nullptr, nch,
                                        v_per_position != 0, inv_tau, gout, m, l, out, gx, gh,
                                        nullptr, nullptr, gv, gh != nullptr, workspace,
                                        workspace_bytes, static_cast<cudaStream_t>(stream),
                                        nullptr);
}

// MorletTokenMixer's layout: x, y, dL/dy and dL/dx are (batch, n, dim) tensors (the reference
// transposes them to (batch, dim, n) rows around morlet_mix, fdwt/layers.py:49-55).
extern "C" int fdwt_mix_tokens_forward(int dtype, int64_t batch, int64_t n, int64_t dim,
                                       const void* x, const void* filters,
                                       const fdwt_morlet_plan* plan, const void* a,
                                       const void* b, const void* bias, void* y, void* stream) {
  if (batch < 0 || dim < 1 || batch > 0x7fffffffLL / dim) return FDWT_ERR_INVALID;
  if (batch > 0 && (x == nullptr || filters == nullptr || y == nullptr || a == nullptr ||
                    b == nullptr))
    return FDWT_ERR_INVALID;
  return dispatch_forward<EPI_MIX>(dtype, batch * dim, n, x, filters, plan, y, a, b, nullptr,
                                   nullptr, dim, 0, 1.0, static_cast<cudaStream_t>(stream), 1,
                                   bias);
}

namespace {
int dispatch_tokens_backward(int dtype, int64_t batch, int64_t n, int64_t dim, const void* x,
                             const void* h, const fdwt_morlet_plan* pl, const void* a,
                             const void* b, const void* gy, void* gx, void* gh, void* ga,
                             void* gb, void* gbias, bool need_h, void* ws, size_t ws_bytes,
                             cudaStream_t stream, size_t* need) {
  switch (dtype) {
    case FDWT_F32:
      return tokens_bwd_entry<float>(batch, n, dim, x, h, pl, a, b, gy, gx, gh, ga, gb, gbias,
                                     need_h, ws, ws_bytes, stream, need);
    case FDWT_F64:
      return tokens_bwd_entry<double>(batch, n, dim, x, h, pl, a, b, gy, gx, gh, ga, gb, gbias,
                                      need_h, ws, ws_bytes, stream, need);
    default:
      return FDWT_ERR_UNSUPPORTED;
  }
}
}  // namespace

extern "C" size_t fdwt_mix_tokens_backward_workspace(int dtype, int64_t batch, int64_t n,
                                                     int64_t dim, const fdwt_morlet_plan* plan,
                                                     int need_gh) {
  size_t need = 0;
  if (check_plan(plan, n) != FDWT_OK) return 0;
  if (dispatch_tokens_backward(dtype, batch, n, dim, nullptr, nullptr, plan, nullptr, nullptr,
                               nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                               need_gh != 0, nullptr, 0, nullptr, &need) != FDWT_OK)
    return 0;
  return need;
}

extern "C" int fdwt_mix_tokens_backward(int dtype, int64_t batch, int64_t n, int64_t dim,
                                        const void* x, const void* filters,
                                        const fdwt_morlet_plan* plan, const void* a,
                                        const void* b, const void* gy, void* gx, void* gh,
                                        void* ga, void* gb, void* gbias, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (batch < 0 || dim < 1) return FDWT_ERR_INVALID;
  if (batch > 0 && (x == nullptr || filters == nullptr || a == nullptr || b == nullptr ||
                    gy == nullptr))
    return FDWT_ERR_INVALID;
  const int st = check_plan(plan, n);
  if (st != FDWT_OK) return st;
  return dispatch_tokens_backward(dtype, batch, n, dim, x, filters, plan, a, b, gy, gx, gh, ga,
                                  gb, gbias, gh != nullptr, workspace, workspace_bytes,
                                  static_cast<cudaStream_t>(stream), nullptr);
}
