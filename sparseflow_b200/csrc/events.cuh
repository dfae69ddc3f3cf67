// Spike-event extraction shared by the sparse convolution entry points.
#pragma once
#include "common.cuh"

namespace sf {

struct EventBuffers {
  unsigned long long* masks;  // [image][h][w][nw] nonzero-channel bits
  uint32_t* flags;            // [image] bit 0: a nonzero other than 1.0 occurs
  int nw;                     // 64-bit words per pixel
};

// Workspace bytes for nimg images of C channels and HW pixels: masks, flags,
// and one 256-byte slot for the sampled nonzero count (event_count_word).
size_t event_workspace_bytes(long long nimg, int C, int HW);
uint32_t* event_count_word(void* workspace, long long nimg, int C, int HW);

// Fills `out` (carved from `workspace`) for x (NCHW, nimg images) on `st`;
// the mask kernel runs only when `gate` selects it.
sf_status extract_events(const void* x, int xdt, long long nimg, int C, int HW, void* workspace,
                         size_t workspace_bytes, EventBuffers& out, cudaStream_t st, const Gate& gate);

// Writes to *count the number of nonzeros among `samples` (at most
// kMaxDensitySamples) elements of x (n elements) taken at a fixed stride: a
// memset of the count and one load per thread over samples/256 CTAs.
constexpr int kMaxDensitySamples = 32768;
sf_status sample_nonzeros(const void* x, int xdt, long long n, int samples, uint32_t* count, cudaStream_t st);

}  // namespace sf
