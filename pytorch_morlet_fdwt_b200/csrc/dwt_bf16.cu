// __nv_bfloat16 instantiations of the fused multilevel DWT kernels (every supported filter length).
#include "dwt_impl.cuh"

namespace fdwt {
namespace dwtk {
FDWT_DWT_INSTANTIATE(__nv_bfloat16)
}  // namespace dwtk
}  // namespace fdwt
