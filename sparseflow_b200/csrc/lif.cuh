// Multi-step LIF over a convolution's fp32 output, for the fused conv + LIF
// entry point when its convolution runs on the tensor-core kernel.
#pragma once
#include "common.cuh"

namespace sf {

// y: fp32 [T, N, C, HW] preactivations (may equal spikes: each element is
// read before its spike is stored over it); v: fp32 [N, C, HW] state in and
// out; spikes: fp32 [T, N, C, HW]; masks: the spikes' event masks in the
// mask-pass layout, or null. The update and its operation order are those of
// sf_lif_multistep. Every kernel returns at entry unless `gate` is open.
sf_status lif_after_conv(const float* y, float* v, float* spikes, void* masks, int T, int N, int C, int HW,
                         float tau, float v_threshold, float v_reset, int hard_reset, int decay_input,
                         const Gate& gate, cudaStream_t st);

}  // namespace sf
