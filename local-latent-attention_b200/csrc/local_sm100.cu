// Placeholder until the tcgen05 kernels land: every geometry uses SIMT.
#include "sm100.cuh"

namespace llattn {
namespace sm100 {
bool fwd_supported(const Geom&, int) { return false; }
bool bwd_supported(const Geom&, int) { return false; }
cudaError_t launch_local_fwd(const Geom&, const void*, void*, float*, cudaStream_t) {
  return cudaErrorNotSupported;
}
cudaError_t launch_local_bwd(const Geom&, const void*, const void*, const float*, const float*, void*,
                             cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace sm100
}  // namespace llattn
