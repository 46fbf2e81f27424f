// float instantiation of the Morlet CWT kernels with the store epilogue (cwt_entry.cuh).
#include "cwt_entry.cuh"

namespace fdwt {
namespace cwtk {
FDWT_CWT_INSTANTIATE(float, EPI_STORE)
}  // namespace cwtk
}  // namespace fdwt
