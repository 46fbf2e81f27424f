// double instantiation of the Morlet CWT kernels with the softmax epilogue (cwt_entry.cuh).
#include "cwt_entry.cuh"

namespace fdwt {
namespace cwtk {
FDWT_CWT_INSTANTIATE(double, EPI_SOFTMAX)
}  // namespace cwtk
}  // namespace fdwt
