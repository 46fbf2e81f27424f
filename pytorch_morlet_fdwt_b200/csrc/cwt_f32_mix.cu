// float instantiation of the Morlet CWT kernels with the mix epilogue (cwt_entry.cuh).
#include "cwt_entry.cuh"

namespace fdwt {
namespace cwtk {
FDWT_CWT_INSTANTIATE(float, EPI_MIX)
FDWT_CWT_INSTANTIATE_TOKENS(float)
}  // namespace cwtk
}  // namespace fdwt
