// Stage 1 of the sparse convolution: spike-event extraction.
//
// One streaming pass over x (NCHW, images = T*N) writes, for every pixel, a
// bitmask of its nonzero input channels: nw = ceil(C/64) 64-bit words per
// pixel, layout [image][h][w][nw]. For fp32 spikes this is 1/32 of the bytes
// of x, so the convolution stage never has to stage x itself. The pass also
// raises flags[image] when a nonzero value other than 1.0 occurs; only then
// does the convolution read x values (binary spikes need none).
//
// This is the element-granular form of the reference's stage-1 metadata
// (Kernels/_prescan_common.py:32-189 builds per-tile channel-group bits); the
// tile-group metadata itself is produced bit-exactly by prescan.cu.
#include "events.cuh"

namespace sf {
namespace {

constexpr int kEvThreads = 256;

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) EVec {
  T v[VEC];
};

// Each thread owns VEC consecutive pixels of one image and channel word
// blockIdx.y. With FLAT, thread g of the grid takes image g / (HW / VEC), so
// small feature maps (8x8) still fill whole CTAs; otherwise blockIdx.z is
// the image (a CTA never straddles two images; measured 12 % faster for
// 56x56 maps with four channel words).
template <typename XT, int VEC, bool FLAT>
__global__ void __launch_bounds__(kEvThreads) spike_masks_kernel(const XT* __restrict__ x, int C, int HW, int nw,
                                                                 long long nimg,
                                                                 unsigned long long* __restrict__ masks,
                                                                 uint32_t* __restrict__ flags, const Gate gate) {
  if (!gate_open(gate)) return;
  const int word = blockIdx.y;
  const int vpi = HW / VEC;  // vectors per image
  long long img;
  int pix0;
  if constexpr (FLAT) {
    const long long gid = (long long)blockIdx.x * kEvThreads + threadIdx.x;
    if (gid >= nimg * vpi) return;
    img = gid / vpi;
    pix0 = (int)(gid - img * vpi) * VEC;
  } else {
    img = blockIdx.z;
    pix0 = (blockIdx.x * kEvThreads + threadIdx.x) * VEC;
    if (pix0 >= HW) return;
  }
  const int c0 = word * 64;
  const int cn = min(64, C - c0);
  uint32_t lo[VEC], hi[VEC];
  uint32_t bad = 0u;
#pragma unroll
  for (int e = 0; e < VEC; ++e) lo[e] = hi[e] = 0u;
  const XT* src = x + ((size_t)img * C + c0) * HW + pix0;
  int c = 0;
  // Eight channels per step keep eight 16-byte loads in flight per thread.
#pragma unroll 1
  for (; c + 8 <= cn; c += 8) {
    EVec<XT, VEC> r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) r[u] = *reinterpret_cast<const EVec<XT, VEC>*>(src + (size_t)(c + u) * HW);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int cc = c + u;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const uint32_t nz = DT<XT>::nz_bit(r[u].v[e]);
        bad |= nz & DT<XT>::not_one(r[u].v[e]);
        if (cc < 32)
          lo[e] |= nz << cc;
        else
          hi[e] |= nz << (cc - 32);
      }
    }
  }
  for (; c < cn; ++c) {
    const EVec<XT, VEC> r = *reinterpret_cast<const EVec<XT, VEC>*>(src + (size_t)c * HW);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const uint32_t nz = DT<XT>::nz_bit(r.v[e]);
      bad |= nz & DT<XT>::not_one(r.v[e]);
      if (c < 32)
        lo[e] |= nz << c;
      else
        hi[e] |= nz << (c - 32);
    }
  }
  unsigned long long* dst = masks + ((size_t)img * HW + pix0) * nw + word;
#pragma unroll
  for (int e = 0; e < VEC; ++e) dst[(size_t)e * nw] = ((unsigned long long)hi[e] << 32) | lo[e];
  // One atomic per image present in the warp that saw a value other than 0/1.
  const unsigned same = __match_any_sync(__activemask(), img);
  const unsigned any_bad = __ballot_sync(__activemask(), bad != 0u) & same;
  if (any_bad != 0u && (threadIdx.x & 31) == __ffs(same) - 1) atomicOr(&flags[img], 1u);
}

template <typename XT>
sf_status launch(const void* x, int nimg, int C, int HW, unsigned long long* masks, uint32_t* flags,
                 cudaStream_t st, const Gate& gate) {
  const int nw = (C + 63) / 64;
  constexpr int V = 16 / (int)sizeof(XT);
  const bool vec = aligned16(x) && HW % V == 0;
  const int vpi = HW / (vec ? V : 1);
  const XT* xp = static_cast<const XT*>(x);
  if (nw > 65535) return SF_ERR_UNSUPPORTED;
  if (vpi >= kEvThreads && nimg <= 65535) {
    const dim3 grid((vpi + kEvThreads - 1) / kEvThreads, nw, (unsigned)nimg);
    if (vec)
      spike_masks_kernel<XT, V, false><<<grid, kEvThreads, 0, st>>>(xp, C, HW, nw, nimg, masks, flags, gate);
    else
      spike_masks_kernel<XT, 1, false><<<grid, kEvThreads, 0, st>>>(xp, C, HW, nw, nimg, masks, flags, gate);
  } else {
    const long long blocks = ((long long)nimg * vpi + kEvThreads - 1) / kEvThreads;
    if (blocks > 0x7fffffffll) return SF_ERR_UNSUPPORTED;
    const dim3 grid((unsigned)blocks, nw, 1);
    if (vec)
      spike_masks_kernel<XT, V, true><<<grid, kEvThreads, 0, st>>>(xp, C, HW, nw, nimg, masks, flags, gate);
    else
      spike_masks_kernel<XT, 1, true><<<grid, kEvThreads, 0, st>>>(xp, C, HW, nw, nimg, masks, flags, gate);
  }
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

}  // namespace

static size_t event_core_bytes(long long nimg, int C, int HW) {
  const size_t nw = (size_t)(C + 63) / 64;
  const size_t mask_bytes = (size_t)nimg * HW * nw * 8;
  return ((mask_bytes + 255) / 256) * 256 + (((size_t)nimg * 4 + 255) / 256) * 256;
}

size_t event_workspace_bytes(long long nimg, int C, int HW) { return event_core_bytes(nimg, C, HW) + 256; }

uint32_t* event_count_word(void* workspace, long long nimg, int C, int HW) {
  return reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + event_core_bytes(nimg, C, HW));
}

namespace {
template <typename XT>
__global__ void __launch_bounds__(256) sample_nonzeros_kernel(const XT* __restrict__ x, long long n, int samples,
                                                               uint32_t* count) {
  __shared__ uint32_t warp_cnt[8];
  const long long stride = max(1ll, n / samples);
  const int i = blockIdx.x * 256 + threadIdx.x;
  const long long idx = (long long)i * stride;
  uint32_t c = (i < samples && idx < n) ? DT<XT>::nz_bit(x[idx]) : 0u;
  for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) warp_cnt[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < 8; ++w) t += warp_cnt[w];
    if (t) atomicAdd(count, t);
  }
}
}  // namespace

// The samples are scattered over x (one 32-byte sector each), so they are
// spread over many CTAs: one SM issuing all 32768 took 20-28 us.
sf_status sample_nonzeros(const void* x, int xdt, long long n, int samples, uint32_t* count, cudaStream_t st) {
  if (samples <= 0 || samples > kMaxDensitySamples) return SF_ERR_INVALID_ARG;
  if (cudaMemsetAsync(count, 0, 4, st) != cudaSuccess) return SF_ERR_CUDA;
  const unsigned blocks = (unsigned)((samples + 255) / 256);
  switch (xdt) {
    case SF_DTYPE_F32:
      sample_nonzeros_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), n, samples, count);
      break;
    case SF_DTYPE_F16:
      sample_nonzeros_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x), n, samples, count);
      break;
    case SF_DTYPE_BF16:
      sample_nonzeros_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n,
                                                                     samples, count);
      break;
    default: return SF_ERR_INVALID_ARG;
  }
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

sf_status extract_events(const void* x, int xdt, long long nimg, int C, int HW, void* workspace,
                         size_t workspace_bytes, EventBuffers& out, cudaStream_t st, const Gate& gate) {
  if (workspace_bytes < event_workspace_bytes(nimg, C, HW)) return SF_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return SF_ERR_ALIGNMENT;
  const size_t nw = (size_t)(C + 63) / 64;
  out.masks = static_cast<unsigned long long*>(workspace);
  out.flags = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) +
                                          (((size_t)nimg * HW * nw * 8 + 255) / 256) * 256);
  out.nw = (int)nw;
  if (cudaMemsetAsync(out.flags, 0, (size_t)nimg * 4, st) != cudaSuccess) return SF_ERR_CUDA;
  switch (xdt) {
    case SF_DTYPE_F32: return launch<float>(x, (int)nimg, C, HW, out.masks, out.flags, st, gate);
    case SF_DTYPE_F16: return launch<__half>(x, (int)nimg, C, HW, out.masks, out.flags, st, gate);
    case SF_DTYPE_BF16: return launch<__nv_bfloat16>(x, (int)nimg, C, HW, out.masks, out.flags, st, gate);
  }
  return SF_ERR_INVALID_ARG;
}

}  // namespace sf
