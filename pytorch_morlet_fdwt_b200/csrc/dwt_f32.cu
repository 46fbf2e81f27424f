// float instantiations of the fused multilevel DWT kernels (every supported filter length).
#include "dwt_impl.cuh"

namespace fdwt {
namespace dwtk {
FDWT_DWT_INSTANTIATE(float)
}  // namespace dwtk
}  // namespace fdwt
