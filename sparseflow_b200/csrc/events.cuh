// Spike-event extraction shared by the sparse convolution entry points.
#pragma once
#include "common.cuh"

namespace sf {

struct EventBuffers {
  unsigned long long* masks;  // [image][h][w][nw] nonzero-channel bits
  uint32_t* flags;            // [image] bit 0: a nonzero other than 1.0 occurs
  int nw;                     // 64-bit words per pixel
};

// Workspace bytes for nimg images of C channels and HW pixels.
size_t event_workspace_bytes(long long nimg, int C, int HW);

// Fills `out` (carved from `workspace`) for x (NCHW, nimg images) on `st`.
sf_status extract_events(const void* x, int xdt, long long nimg, int C, int HW, void* workspace,
                         size_t workspace_bytes, EventBuffers& out, cudaStream_t st);

}  // namespace sf
