// Host interface of the tcgen05 3x3 convolution (conv3x3_tc.cu) and of the
// weight section it reads, appended to the gather-packed weights.
#pragma once
#include "common.cuh"

namespace sf {
namespace c3tc {

// Input channels the kernel takes; up to kTcResidentMaxC the weight digits
// of an output block stay in shared memory, above it they stream through a
// ring of stages while the unit's converted input stays resident.
constexpr int kTcMaxC = 512;
constexpr int kTcResidentMaxC = 64;

// Whether sf_pack_weights appends the tensor-core section for this layer.
bool tc3_packs(int Co, int C, int K);
// Bytes of that section: per-channel digit scales [3][ncob * CB] (fp32) and
// the int8 digit image [ncob][9][kcores][3 * CB][16].
size_t tc3_section_bytes(int Co, int C);
// Writes the section from OIHW weights of any supported dtype.
sf_status tc3_pack(const void* w_oihw, int src_dtype, int Co, int C, void* section, cudaStream_t st);
// Whether the kernel can run this shape (shared memory, TMEM, 32-bit
// position decode); run_conv3x3_tc returns SF_ERR_UNSUPPORTED otherwise.
bool tc3_supported(int N, int C, int H, int W, int Co);
// Multi-step LIF applied in the epilogue: the N images are T steps of N / T
// images each (image t * N / T + n), v is the fp32 membrane [N / T, Co, H, W]
// (state in and out) and y receives the spikes instead of the convolution.
struct TcLif {
  int T;
  float* v;
  float tau, v_threshold, v_reset;
  int hard_reset, decay_input;
  // false: only where it pays (streamed weights and at least 2 tiles per SM
  // in one step's plane); true: wherever the membranes can be staged.
  bool always;
};
// Runs the convolution (when `gate` selects it); with `lif`, the fused
// convolution + multi-step LIF.
sf_status run_conv3x3_tc(const void* x, const void* w_gather, int cpl, const void* section, const float* bias,
                         void* y, uint32_t* err, int N, int C, int H, int W, int Co, int xdt, int wdt,
                         cudaStream_t st, const Gate& gate, const TcLif* lif = nullptr);

}  // namespace c3tc
}  // namespace sf
