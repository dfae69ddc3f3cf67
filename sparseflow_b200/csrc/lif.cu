// Multi-step LIF neuron over [T, numel] (HBM-bound elementwise).
//
// The update is the reference's multi-step LIF (Ops/sparse_fused_conv_lif.py:
// 271-293, spikingjelly LIFNode with step_mode 'm'):
//   decay_input: h = v + (x - (v - v_reset)) / tau
//   otherwise:   h = v - (v - v_reset) / tau + x
//   spike = h >= v_threshold
//   hard reset:  v = spike ? v_reset : h;   soft reset: v = h - spike * v_threshold
// with the same operation order and IEEE division, so spikes equal the
// PyTorch formula bit for bit. A torch LIFNode runs about eight elementwise
// kernels per step and moves v through HBM every step; here each thread owns
// VEC elements, keeps their v in registers across all T steps, and reads x /
// writes spikes once: bytes = T * numel * (|x| + |spike|) + 8 * numel.
#include <cmath>
#include <cstdlib>
#include "common.cuh"
#include "lif.cuh"
#include "policy.cuh"

namespace sf {
namespace {

template <typename T, int V>
struct alignas(sizeof(T) * V) LVec {
  T v[V];
};

struct LifParams {
  float tau, vth, vr;
  int hard, decay_input;
};

__device__ __forceinline__ float lif_update(float& v, float x, const LifParams& q) {
  float h;
  if (q.decay_input)
    h = v + (x - (v - q.vr)) / q.tau;
  else
    h = v - (v - q.vr) / q.tau + x;
  const bool s = h >= q.vth;
  v = q.hard ? (s ? q.vr : h) : (h - (s ? q.vth : 0.f));
  return s ? 1.f : 0.f;
}

// Streaming (evict-first) vector loads and stores: x is read once and the
// spikes are written once, so neither should displace v or other data in L2.
template <typename T, int V>
__device__ __forceinline__ LVec<T, V> ld_stream(const LVec<T, V>* p) {
  if constexpr (sizeof(LVec<T, V>) == 16) {
    const float4 f = __ldcs(reinterpret_cast<const float4*>(p));
    return *reinterpret_cast<const LVec<T, V>*>(&f);
  } else if constexpr (sizeof(LVec<T, V>) == 8) {
    const float2 f = __ldcs(reinterpret_cast<const float2*>(p));
    return *reinterpret_cast<const LVec<T, V>*>(&f);
  } else {
    return *p;
  }
}
template <typename T, int V>
__device__ __forceinline__ void st_stream(LVec<T, V>* p, const LVec<T, V>& v) {
  if constexpr (sizeof(LVec<T, V>) == 16)
    __stcs(reinterpret_cast<float4*>(p), *reinterpret_cast<const float4*>(&v));
  else if constexpr (sizeof(LVec<T, V>) == 8)
    __stcs(reinterpret_cast<float2*>(p), *reinterpret_cast<const float2*>(&v));
  else
    *p = v;
}

// Steps whose x is loaded ahead of their updates: the loads of a group do not
// depend on the membrane state, so all of them are in flight together.
constexpr int kLifPrefetch = 8;

template <typename XT, typename ST, int VEC>
__global__ void __launch_bounds__(256) lif_multistep_kernel(const XT* __restrict__ x, float* __restrict__ v,
                                                            ST* __restrict__ s, long long numel, int T,
                                                            LifParams q, Gate gate) {
  if (!gate_open(gate)) return;
  const long long nvec = numel / VEC;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    LVec<float, VEC> vv = reinterpret_cast<const LVec<float, VEC>*>(v)[i];
    for (int t0 = 0; t0 < T; t0 += kLifPrefetch) {
      LVec<XT, VEC> xb[kLifPrefetch];
#pragma unroll
      for (int k = 0; k < kLifPrefetch; ++k)
        if (t0 + k < T) xb[k] = ld_stream(reinterpret_cast<const LVec<XT, VEC>*>(x + (size_t)(t0 + k) * numel) + i);
#pragma unroll
      for (int k = 0; k < kLifPrefetch; ++k) {
        if (t0 + k < T) {
          LVec<ST, VEC> sv;
#pragma unroll
          for (int e = 0; e < VEC; ++e) sv.v[e] = DT<ST>::from_f(lif_update(vv.v[e], DT<XT>::to_f(xb[k].v[e]), q));
          st_stream(reinterpret_cast<LVec<ST, VEC>*>(s + (size_t)(t0 + k) * numel) + i, sv);
        }
      }
    }
    reinterpret_cast<LVec<float, VEC>*>(v)[i] = vv;
  }
}

template <typename XT, typename ST>
sf_status launch(const void* x, float* v, void* s, long long numel, int T, const LifParams& q, cudaStream_t st,
                 const Gate& gate) {
  const bool vec = numel % 4 == 0 && aligned16(v) && (reinterpret_cast<uintptr_t>(x) % (4 * sizeof(XT))) == 0 &&
                   (reinterpret_cast<uintptr_t>(s) % (4 * sizeof(ST))) == 0;
  const int V = vec ? 4 : 1;
  const long long nvec = numel / V;
  // One vector per thread where the grid allows (no tail of uneven loop trips).
  const long long blocks = std::min<long long>((nvec + 255) / 256, 1ll << 30);
  if (blocks <= 0) return SF_OK;
  if (vec)
    lif_multistep_kernel<XT, ST, 4><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const XT*>(x), v,
                                                                     static_cast<ST*>(s), numel, T, q, gate);
  else
    lif_multistep_kernel<XT, ST, 1><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const XT*>(x), v,
                                                                     static_cast<ST*>(s), numel, T, q, gate);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <typename XT>
sf_status dispatch_s(int sdt, const void* x, float* v, void* s, long long numel, int T, const LifParams& q,
                     cudaStream_t st) {
  const Gate open{nullptr, 0u, 0};
  switch (sdt) {
    case SF_DTYPE_F32: return launch<XT, float>(x, v, s, numel, T, q, st, open);
    case SF_DTYPE_F16: return launch<XT, __half>(x, v, s, numel, T, q, st, open);
    case SF_DTYPE_BF16: return launch<XT, __nv_bfloat16>(x, v, s, numel, T, q, st, open);
  }
  return SF_ERR_INVALID_ARG;
}


// ---------------------------------------------------------------------------
// The same LIF, also writing the spikes' event masks for the next sparse
// convolution (the layout of the mask pass: per image and pixel, bit c % 64
// of 64-bit word c / 64 set iff channel c spiked; written here as 32-bit
// halves). A warp owns 32 consecutive pixels (lane = pixel) x 32 channels of
// one image: every load and store instruction covers one contiguous 128-byte
// row segment (fp32), the 32 membranes stay in registers across all steps,
// and each lane assembles its pixel's half word bit by bit (no ballots).
// ---------------------------------------------------------------------------
constexpr int kEvCh = 32;  // channels per warp (one 32-bit half word)
#ifndef SF_LIF_EV_T
#define SF_LIF_EV_T 4
#endif
#ifndef SF_LIF_EV_G
#define SF_LIF_EV_G 4
#endif
#ifndef SF_LIF_EV_MINB
#define SF_LIF_EV_MINB 4
#endif
constexpr int kEvT = SF_LIF_EV_T;  // steps per load group
constexpr int kEvG = SF_LIF_EV_G;  // channels per load group

// lif_update with x / tau computed as x * (1 / tau): for tau a power of two
// both are the correctly rounded value of the same real number, so the
// results (and spikes) are identical without the division sequence.
__device__ __forceinline__ float lif_update_pow2(float& v, float x, const LifParams& q, float inv_tau) {
  float h;
  if (q.decay_input)
    h = v + __fmul_rn(x - (v - q.vr), inv_tau);
  else
    h = v - __fmul_rn(v - q.vr, inv_tau) + x;
  const bool s = h >= q.vth;
  v = q.hard ? (s ? q.vr : h) : (h - (s ? q.vth : 0.f));
  return s ? 1.f : 0.f;
}

template <typename XT, typename ST, bool POW2>
__global__ void __launch_bounds__(256, SF_LIF_EV_MINB) lif_events_kernel(const XT* __restrict__ x, float* __restrict__ v,
                                                         ST* __restrict__ s, uint32_t* __restrict__ masks, int T,
                                                         int N, int C, int HW, int ncb, int npb, int nw2,
                                                         LifParams q, float inv_tau, Gate gate) {
  if (!gate_open(gate)) return;
  // Membranes of the warp's 32 channels x 32 pixels, [channel][warp][lane]:
  // conflict-free, and no per-channel register file to unroll.
  __shared__ float vs[kEvCh][8][32];
  const int wib = threadIdx.x >> 5;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + wib;
  const int lane = threadIdx.x & 31;
  if (gw >= (long long)N * ncb * npb) return;
  const int pb = (int)(gw % npb);
  const long long rest = gw / npb;
  const int cb = (int)(rest % ncb);
  const int img = (int)(rest / ncb);
  const int p = pb * 32 + lane;
  const bool pix = p < HW;
  const int c0 = cb * kEvCh;
  const int nc = min(kEvCh, C - c0);
  const size_t step = (size_t)N * C * HW;
  const size_t off = ((size_t)img * C + c0) * HW + p;  // channel c0 of this lane's pixel
  // With no sibling block for the upper half word of the last 64-channel word,
  // this warp also writes that half as zero.
  const bool zero_upper = (cb % 2 == 0) && cb + 1 < nw2 && c0 + kEvCh >= C;

  for (int j = 0; j < kEvCh; ++j) vs[j][wib][lane] = (pix && j < nc) ? v[off + j * HW] : 0.f;
  // Steps in groups of kEvT, channels in groups of kEvG: the group's
  // kEvT x kEvG loads are independent of the membrane and all in flight
  // together; each channel then runs through the group's steps.
  for (int t0 = 0; t0 < T; t0 += kEvT) {
    uint32_t word[kEvT];
#pragma unroll
    for (int k = 0; k < kEvT; ++k) word[k] = 0u;
#pragma unroll 1
    for (int g0 = 0; g0 < nc; g0 += kEvG) {
      float xr[kEvT][kEvG];
#pragma unroll
      for (int k = 0; k < kEvT; ++k) {
        const XT* xt = x + (size_t)(t0 + k) * step + off + g0 * HW;
#pragma unroll
        for (int j = 0; j < kEvG; ++j)
          xr[k][j] = (pix && t0 + k < T && g0 + j < nc) ? DT<XT>::to_f(__ldcs(xt + j * HW)) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kEvG; ++j) {
        if (g0 + j < nc) {
          float vv = vs[g0 + j][wib][lane];
#pragma unroll
          for (int k = 0; k < kEvT; ++k) {
            if (t0 + k < T) {
              const float sp = POW2 ? lif_update_pow2(vv, xr[k][j], q, inv_tau) : lif_update(vv, xr[k][j], q);
              word[k] |= (sp != 0.f ? 1u : 0u) << (g0 + j);
              if (pix) __stcs(s + (size_t)(t0 + k) * step + off + (g0 + j) * HW, DT<ST>::from_f(sp));
            }
          }
          vs[g0 + j][wib][lane] = vv;
        }
      }
    }
    if (pix) {
#pragma unroll
      for (int k = 0; k < kEvT; ++k) {
        if (t0 + k < T) {
          uint32_t* mw = masks + ((size_t)((size_t)(t0 + k) * N + img) * HW + p) * nw2;
          mw[cb] = word[k];
          if (zero_upper) mw[cb + 1] = 0u;
        }
      }
    }
  }
  for (int j = 0; j < nc; ++j)
    if (pix) v[off + j * HW] = vs[j][wib][lane];
}

// 1 / tau when tau is a power of two (with a normal reciprocal), else 0.
inline float pow2_reciprocal(float tau) {
  int e = 0;
  const float m = std::frexp(std::fabs(tau), &e);
  if (m != 0.5f || e < -124 || e > 126) return 0.f;
  return 1.f / tau;
}

template <typename XT, typename ST>
sf_status launch_events(const void* x, float* v, void* s, void* masks, int T, int N, int C, int HW,
                        const LifParams& q, cudaStream_t st, const Gate& gate) {
  const int ncb = (C + kEvCh - 1) / kEvCh, npb = (HW + 31) / 32, nw2 = 2 * ((C + 63) / 64);
  const long long warps = (long long)N * ncb * npb;
  const long long blocks = (warps + 7) / 8;
  if (blocks > INT32_MAX) return SF_ERR_UNSUPPORTED;
  const float inv = pow2_reciprocal(q.tau);
  if (inv != 0.f)
    lif_events_kernel<XT, ST, true><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const XT*>(x), v, static_cast<ST*>(s), static_cast<uint32_t*>(masks), T, N, C, HW, ncb, npb,
        nw2, q, inv, gate);
  else
    lif_events_kernel<XT, ST, false><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const XT*>(x), v, static_cast<ST*>(s), static_cast<uint32_t*>(masks), T, N, C, HW, ncb, npb,
        nw2, q, 0.f, gate);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

// Fast path of the event-emitting LIF (C*H*W a multiple of 128, 16-byte
// aligned tensors, an image's spikes at most kBitmapMaxBytes bits/8):
//  1. lif_bitmap_kernel: the streaming sf_lif_multistep kernel plus four warp
//     ballots per step, which pack each warp's 128 consecutive spikes into
//     four 32-bit words of a flat bitmap (bit j % 32 of word j / 32 =
//     element j of the image, j = c*H*W + p). An image's bitmap (C*H*W/8
//     bytes) is never larger than its region of the event-mask buffer
//     (H*W*ceil(C/64)*8 bytes), so it is written at the start of that region.
//  2. bitmap_to_masks_kernel: one CTA per image loads the bitmap into shared
//     memory, synchronises, and overwrites the region with the per-pixel
//     channel masks. Each CTA touches only its own image's region.
// The spikes are read 1/32 as often as by the mask pass over them.
constexpr int kBmPrefetch = 4;  // steps loaded ahead in lif_bitmap_kernel
constexpr int kBitmapMaxBytes = 200 * 1024;  // shared memory of one transpose CTA

__device__ __forceinline__ uint32_t spread_nibbles(uint32_t b) {  // bit j of b (j < 8) -> bit 4j
  b = (b | (b << 12)) & 0x000F000Fu;
  b = (b | (b << 6)) & 0x03030303u;
  b = (b | (b << 3)) & 0x11111111u;
  return b;
}

template <typename XT, typename ST, bool POW2>
__global__ void __launch_bounds__(256, 4) lif_bitmap_kernel(const XT* __restrict__ x, float* __restrict__ v,
                                                         ST* __restrict__ s, uint32_t* __restrict__ masks,
                                                         long long numel, int T, long long img_elems,
                                                         long long region_words, int n_per_step, LifParams q,
                                                         float inv_tau, Gate gate) {
  if (!gate_open(gate)) return;
  constexpr int VEC = 4;
  const long long nvec = numel / VEC;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long wb = ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32; wb < nvec;
       wb += warps * 32) {
    const long long i = wb + lane;
    const bool ok = i < nvec;
    LVec<float, VEC> vv{};
    if (ok) vv = reinterpret_cast<const LVec<float, VEC>*>(v)[i];
    // The warp's 128 elements lie in one image (img_elems % 128 == 0).
    const long long e0 = wb * VEC;
    const long long img_in_step = e0 / img_elems;
    const long long j0 = e0 - img_in_step * img_elems;  // multiple of 128
    for (int t0 = 0; t0 < T; t0 += kBmPrefetch) {
      LVec<XT, VEC> xb[kBmPrefetch];
#pragma unroll
      for (int k = 0; k < kBmPrefetch; ++k)
        if (ok && t0 + k < T)
          xb[k] = ld_stream(reinterpret_cast<const LVec<XT, VEC>*>(x + (size_t)(t0 + k) * numel) + i);
#pragma unroll
      for (int k = 0; k < kBmPrefetch; ++k) {
        if (t0 + k < T) {
          LVec<ST, VEC> sv;
          uint32_t b[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float xe = DT<XT>::to_f(xb[k].v[e]);
            const float sp =
                ok ? (POW2 ? lif_update_pow2(vv.v[e], xe, q, inv_tau) : lif_update(vv.v[e], xe, q)) : 0.f;
            sv.v[e] = DT<ST>::from_f(sp);
            b[e] = __ballot_sync(0xffffffffu, sp != 0.f);  // bit l: element 4l + e of the warp's 128
          }
          if (ok) st_stream(reinterpret_cast<LVec<ST, VEC>*>(s + (size_t)(t0 + k) * numel) + i, sv);
          if (lane < 4) {
            // Word `lane` covers elements 32*lane .. +31 = lanes 8*lane .. +7.
            uint32_t w = 0u;
#pragma unroll
            for (int e = 0; e < VEC; ++e) w |= spread_nibbles((b[e] >> (8 * lane)) & 0xffu) << e;
            const long long img = (long long)(t0 + k) * n_per_step + img_in_step;
            masks[img * region_words + (j0 >> 5) + lane] = w;
          }
        }
      }
    }
    if (ok) reinterpret_cast<LVec<float, VEC>*>(v)[i] = vv;
  }
}

// 32x32 bit-matrix transpose across a warp: lane r holds row r (bit c =
// element (r, c)); afterwards lane c holds column c (bit r = element (r, c)).
// Each stage swaps the off-diagonal blocks of size s.
__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x, int lane) {
  const uint32_t m[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const int sh = 16 >> k;
    const uint32_t y = __shfl_xor_sync(0xffffffffu, x, sh);
    x = (lane & sh) ? ((x & ~m[k]) | ((y >> sh) & m[k])) : ((x & m[k]) | ((y & m[k]) << sh));
  }
  return x;
}

// One CTA per image: bitmap (start of the image's region) -> shared memory ->
// per-pixel channel masks over the same region. A warp item is 32 pixels x
// 32 channels: lane = channel reads its 32-pixel window of the bitmap, the
// warp transposes, lane = pixel writes that 32-channel half word.
__global__ void __launch_bounds__(512) bitmap_to_masks_kernel(uint32_t* __restrict__ masks, int C, int HW,
                                                              long long region_words, int nw, Gate gate) {
  if (!gate_open(gate)) return;
  extern __shared__ uint32_t bm[];
  uint32_t* reg = masks + (size_t)blockIdx.x * region_words;
  const int nbits_words = (int)(((long long)C * HW) >> 5);
#pragma unroll 8
  for (int k = threadIdx.x; k < nbits_words; k += blockDim.x) bm[k] = __ldcs(reg + k);
  if (threadIdx.x == 0) bm[nbits_words] = 0u;  // the last window's upper neighbour
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int ngroups = (HW + 31) / 32, nhalves = 2 * nw;
  for (int item = warp; item < ngroups * nhalves; item += nwarps) {
    const int g = item / nhalves, hb = item - g * nhalves;
    const int c = hb * 32 + lane, p0 = g * 32;
    uint32_t row = 0u;
    if (c < C) {
      const int bit = c * HW + p0;
      row = __funnelshift_r(bm[bit >> 5], bm[(bit >> 5) + 1], bit & 31);
      const int np = HW - p0;
      if (np < 32) row &= (1u << np) - 1u;  // pixels past the row belong to the next channel
    }
    const uint32_t col = warp_transpose32(row, lane);
    if (p0 + lane < HW) reg[(size_t)(p0 + lane) * nhalves + hb] = col;
  }
}

template <typename XT, typename ST>
bool launch_events_bitmap(const void* x, float* v, void* s, void* masks, int T, int N, int C, int HW,
                          const LifParams& q, cudaStream_t st, const Gate& gate, sf_status* status) {
  const long long img_elems = (long long)C * HW;
  const long long bitmap_bytes = img_elems / 8;
  if (img_elems % 128 != 0 || bitmap_bytes > kBitmapMaxBytes) return false;
  if (!aligned16(v) || !aligned16(x) || (reinterpret_cast<uintptr_t>(s) % (4 * sizeof(ST))) != 0 ||
      (reinterpret_cast<uintptr_t>(masks) & 15u) != 0)
    return false;
  const int nw = (C + 63) / 64;
  const long long region_words = (long long)HW * nw * 2;  // 32-bit words per image
  const long long numel = (long long)N * C * HW;
  const long long nvec = numel / 4;
  const long long blocks = std::min<long long>((nvec + 255) / 256, 1ll << 30);
  const float inv = pow2_reciprocal(q.tau);
  if (inv != 0.f)
    lif_bitmap_kernel<XT, ST, true><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const XT*>(x), v, static_cast<ST*>(s), static_cast<uint32_t*>(masks), numel, T, img_elems,
        region_words, N, q, inv, gate);
  else
    lif_bitmap_kernel<XT, ST, false><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const XT*>(x), v, static_cast<ST*>(s), static_cast<uint32_t*>(masks), numel, T, img_elems,
        region_words, N, q, 0.f, gate);
  if (cudaGetLastError() != cudaSuccess) {
    *status = SF_ERR_CUDA;
    return true;
  }
  const int smem = (int)bitmap_bytes + 4;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(bitmap_to_masks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    *status = SF_ERR_CUDA;
    return true;
  }
  const long long images = (long long)T * N;
  if (images > INT32_MAX) {
    *status = SF_ERR_UNSUPPORTED;
    return true;
  }
  bitmap_to_masks_kernel<<<(unsigned)images, 512, smem, st>>>(static_cast<uint32_t*>(masks), C, HW, region_words,
                                                              nw, gate);
  *status = cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
  return true;
}

template <typename XT, typename ST>
sf_status launch_events_any(const void* x, float* v, void* s, void* m, int T, int N, int C, int HW,
                            const LifParams& q, cudaStream_t st, const Gate& gate = Gate{nullptr, 0u, 0}) {
  sf_status status = SF_OK;
  if (policy(SF_POLICY_LIF_EVENTS_GENERAL) == 0 &&
      launch_events_bitmap<XT, ST>(x, v, s, m, T, N, C, HW, q, st, gate, &status))
    return status;
  return launch_events<XT, ST>(x, v, s, m, T, N, C, HW, q, st, gate);
}

template <typename XT>
sf_status dispatch_events_s(int sdt, const void* x, float* v, void* s, void* m, int T, int N, int C, int HW,
                            const LifParams& q, cudaStream_t st) {
  switch (sdt) {
    case SF_DTYPE_F32: return launch_events_any<XT, float>(x, v, s, m, T, N, C, HW, q, st);
    case SF_DTYPE_F16: return launch_events_any<XT, __half>(x, v, s, m, T, N, C, HW, q, st);
    case SF_DTYPE_BF16: return launch_events_any<XT, __nv_bfloat16>(x, v, s, m, T, N, C, HW, q, st);
  }
  return SF_ERR_INVALID_ARG;
}
}  // namespace

sf_status lif_after_conv(const float* y, float* v, float* spikes, void* masks, int T, int N, int C, int HW,
                         float tau, float v_threshold, float v_reset, int hard_reset, int decay_input,
                         const Gate& gate, cudaStream_t st) {
  LifParams q;
  q.tau = tau;
  q.vth = v_threshold;
  q.vr = hard_reset ? v_reset : 0.f;
  q.hard = hard_reset;
  q.decay_input = decay_input;
  if (masks) return launch_events_any<float, float>(y, v, spikes, masks, T, N, C, HW, q, st, gate);
  return launch<float, float>(y, v, spikes, (long long)N * C * HW, T, q, st, gate);
}

}  // namespace sf

using namespace sf;

extern "C" sf_status sf_lif_multistep(const void* x, float* v_inout, void* spikes_out, const sf_lif_ms_desc* d,
                                      void* stream) {
  if (!d || !x || !v_inout || !spikes_out) return SF_ERR_INVALID_ARG;
  if (d->numel < 0 || d->t_steps < 0 || !(d->tau != 0.f)) return SF_ERR_INVALID_ARG;
  if (dtype_size(d->x_dtype) == 0 || dtype_size(d->s_dtype) == 0) return SF_ERR_INVALID_ARG;
  if (d->numel == 0 || d->t_steps == 0) return SF_OK;
  LifParams q;
  q.tau = d->tau;
  q.vth = d->v_threshold;
  q.vr = d->hard_reset ? d->v_reset : 0.f;
  q.hard = d->hard_reset;
  q.decay_input = d->decay_input;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (d->x_dtype) {
    case SF_DTYPE_F32: return dispatch_s<float>(d->s_dtype, x, v_inout, spikes_out, d->numel, d->t_steps, q, st);
    case SF_DTYPE_F16: return dispatch_s<__half>(d->s_dtype, x, v_inout, spikes_out, d->numel, d->t_steps, q, st);
    case SF_DTYPE_BF16:
      return dispatch_s<__nv_bfloat16>(d->s_dtype, x, v_inout, spikes_out, d->numel, d->t_steps, q, st);
  }
  return SF_ERR_INVALID_ARG;
}

extern "C" sf_status sf_lif_multistep_events(const void* x, float* v_inout, void* spikes_out, void* spike_masks_out,
                                             const sf_lif_ms_desc* d, int32_t n, int32_t c, int32_t h, int32_t w,
                                             void* stream) {
  if (!d || !x || !v_inout || !spikes_out || !spike_masks_out) return SF_ERR_INVALID_ARG;
  if (n < 0 || c < 0 || h < 0 || w < 0 || d->t_steps < 0 || !(d->tau != 0.f)) return SF_ERR_INVALID_ARG;
  if ((long long)n * c * h * w != d->numel) return SF_ERR_INVALID_ARG;
  if (dtype_size(d->x_dtype) == 0 || dtype_size(d->s_dtype) == 0) return SF_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(spike_masks_out) & 7u) != 0) return SF_ERR_ALIGNMENT;
  if ((long long)h * w * 32 > INT32_MAX) return SF_ERR_UNSUPPORTED;  // channel offsets in 32-bit
  if (d->numel == 0 || d->t_steps == 0) return SF_OK;
  LifParams q;
  q.tau = d->tau;
  q.vth = d->v_threshold;
  q.vr = d->hard_reset ? d->v_reset : 0.f;
  q.hard = d->hard_reset;
  q.decay_input = d->decay_input;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T = d->t_steps, HW = h * w;
  switch (d->x_dtype) {
    case SF_DTYPE_F32:
      return dispatch_events_s<float>(d->s_dtype, x, v_inout, spikes_out, spike_masks_out, T, n, c, HW, q, st);
    case SF_DTYPE_F16:
      return dispatch_events_s<__half>(d->s_dtype, x, v_inout, spikes_out, spike_masks_out, T, n, c, HW, q, st);
    case SF_DTYPE_BF16:
      return dispatch_events_s<__nv_bfloat16>(d->s_dtype, x, v_inout, spikes_out, spike_masks_out, T, n, c, HW, q,
                                              st);
  }
  return SF_ERR_INVALID_ARG;
}

// ---------------------------------------------------------------------------
// Bounded-wait self test (diagnostics): an mbarrier that never completes.
// ---------------------------------------------------------------------------
namespace sf {
namespace {
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, uint32_t* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none is ever made
    fence_mbar_init();
    *out = mbar_wait_ns(&bar, 0u, limit_ns) ? 1u : 2u;  // 2: gave up, as it must
  }
}
}  // namespace
}  // namespace sf

extern "C" sf_status sf_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* d = nullptr;
  uint32_t h = 0;
  if (cudaMallocAsync(reinterpret_cast<void**>(&d), 4, st) != cudaSuccess) return SF_ERR_CUDA;
  sf::bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns, d);
  const bool ok = cudaGetLastError() == cudaSuccess &&
                  cudaMemcpyAsync(&h, d, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
                  cudaFreeAsync(d, st) == cudaSuccess && cudaStreamSynchronize(st) == cudaSuccess;
  if (!ok) return SF_ERR_CUDA;
  return h == 2u ? SF_ERR_DEVICE_TIMEOUT : (h == 1u ? SF_OK : SF_ERR_CUDA);
}
