// Sparse-conv kernel instantiations for float activations (split per dtype so
// the build compiles them in parallel).
#include "conv_kernel.cuh"

namespace sf {
namespace conv {
sf_status dispatch_f32(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                       const Plan& pl, cudaStream_t st) {
  return dispatch_x<float>(lif, wdt, K, S, p, ym, grid, pl, st);
}
}  // namespace conv
}  // namespace sf

#ifdef SF_CONV_PHASE_PROFILE
// Instrumented builds only: copies (and clears) the fp32 kernels' phase cycle totals.
extern "C" int sf_debug_conv_phases(unsigned long long* out8) {
  if (cudaMemcpyFromSymbol(out8, sf::conv::g_conv_phase, 64) != cudaSuccess) return 1;
  unsigned long long z[8] = {0};
  return cudaMemcpyToSymbol(sf::conv::g_conv_phase, z, 64) == cudaSuccess ? 0 : 1;
}
#endif
