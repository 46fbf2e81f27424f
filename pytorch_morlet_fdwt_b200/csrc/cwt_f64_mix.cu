// double instantiation of the Morlet CWT kernels with the mix epilogue (cwt_entry.cuh).
#include "cwt_entry.cuh"

namespace fdwt {
namespace cwtk {
FDWT_CWT_INSTANTIATE(double, EPI_MIX)
FDWT_CWT_INSTANTIATE_TOKENS(double)
}  // namespace cwtk
}  // namespace fdwt
