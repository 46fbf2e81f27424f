// Per-(type, epilogue) entry points of the Morlet CWT kernels.  cwt.cu (the C ABI) calls these
// declarations; each cwt_<type>_<epilogue>.cu defines one set with FDWT_CWT_INSTANTIATE, so the
// kernels of the six combinations compile as separate units in parallel.
#pragma once

#include "cwt_bwd_tiled.cuh"

namespace fdwt {
namespace cwtk {

template <typename A, int EPI>
int fwd_entry(int64_t rows, int64_t n, const void* x, const void* h, const fdwt_morlet_plan* pl,
              void* y, const void* a, const void* b, void* m, void* l, int64_t dim, int v_pos,
              double inv_tau, cudaStream_t stream, int tok, const void* bias);

template <typename A, int EPI>
int bwd_entry(int64_t rows, int64_t n, const void* x, const void* h, const fdwt_morlet_plan* pl,
              const void* a, const void* b, int64_t dim, int v_pos, double inv_tau,
              const void* g, const void* m, const void* l, const void* out, void* gx, void* gh,
              void* ga, void* gb, void* gv, bool need_h, void* ws, size_t ws_bytes,
              cudaStream_t stream, size_t* need);

template <typename A>
int tokens_bwd_entry(int64_t batch, int64_t n, int64_t dim, const void* x, const void* h,
                     const fdwt_morlet_plan* pl, const void* a, const void* b, const void* gy,
                     void* gx, void* gh, void* ga, void* gb, void* gbias, bool need_h, void* ws,
                     size_t ws_bytes, cudaStream_t stream, size_t* need);

#define FDWT_CWT_INSTANTIATE(T, EPI)                                                           \
  template <>                                                                                 \
  int fwd_entry<T, EPI>(int64_t rows, int64_t n, const void* x, const void* h,                \
                        const fdwt_morlet_plan* pl, void* y, const void* a, const void* b,    \
                        void* m, void* l, int64_t dim, int v_pos, double inv_tau,             \
                        cudaStream_t stream, int tok, const void* bias) {                     \
    return run_forward<T, T, EPI>(rows, n, x, h, pl, y, a, b, m, l, dim, v_pos, inv_tau,      \
                                  stream, tok, bias);                                         \
  }                                                                                           \
  template <>                                                                                 \
  int bwd_entry<T, EPI>(int64_t rows, int64_t n, const void* x, const void* h,                \
                        const fdwt_morlet_plan* pl, const void* a, const void* b,             \
                        int64_t dim, int v_pos, double inv_tau, const void* g, const void* m, \
                        const void* l, const void* out, void* gx, void* gh, void* ga,         \
                        void* gb, void* gv, bool need_h, void* ws, size_t ws_bytes,           \
                        cudaStream_t stream, size_t* need) {                                  \
    return run_backward<T, EPI>(rows, n, x, h, pl, a, b, dim, v_pos, inv_tau, g, m, l, out,   \
                                gx, gh, ga, gb, gv, need_h, ws, ws_bytes, stream, need);      \
  }

#define FDWT_CWT_INSTANTIATE_TOKENS(T)                                                         \
  template <>                                                                                 \
  int tokens_bwd_entry<T>(int64_t batch, int64_t n, int64_t dim, const void* x,               \
                          const void* h, const fdwt_morlet_plan* pl, const void* a,           \
                          const void* b, const void* gy, void* gx, void* gh, void* ga,        \
                          void* gb, void* gbias, bool need_h, void* ws, size_t ws_bytes,      \
                          cudaStream_t stream, size_t* need) {                                \
    return run_mix_tokens_backward<T>(batch, n, dim, x, h, pl, a, b, gy, gx, gh, ga, gb,      \
                                      gbias, need_h, ws, ws_bytes, stream, need);             \
  }

}  // namespace cwtk
}  // namespace fdwt
