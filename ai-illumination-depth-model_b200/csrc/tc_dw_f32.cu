// Instances of the depthwise -> pointwise tcgen05 kernel (tc_dw_kernel.cuh)
// for f32 storage, unsplit launches.
#include "tc_dw_kernel.cuh"

namespace illumina {
namespace gpu {
namespace tcd {
template cudaError_t launch_all<float, false>(int, int, int, const CUtensorMap &, const CUtensorMap &, const Params &,
                                        size_t, cudaStream_t);
}  // namespace tcd
}  // namespace gpu
}  // namespace illumina
