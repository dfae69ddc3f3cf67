// Sparse-conv kernel instantiations for __half activations (split per dtype so
// the build compiles them in parallel).
#include "conv_kernel.cuh"

namespace sf {
namespace conv {
sf_status dispatch_f16(int mode, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                       const Plan& pl, cudaStream_t st) {
  return dispatch_x<__half>(mode, wdt, K, S, p, ym, grid, pl, st);
}
}  // namespace conv
}  // namespace sf
