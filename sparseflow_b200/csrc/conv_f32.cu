// Sparse-conv kernel instantiations for float activations (split per dtype so
// the build compiles them in parallel).
#include "conv_kernel.cuh"

namespace sf {
namespace conv {
sf_status dispatch_f32(int mode, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                       const Plan& pl, cudaStream_t st) {
  return dispatch_x<float>(mode, wdt, K, S, p, ym, grid, pl, st);
}
}  // namespace conv
}  // namespace sf

