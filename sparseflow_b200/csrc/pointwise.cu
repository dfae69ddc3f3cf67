// Sparse 1x1 convolution in one pass (stride 1 or 2, no padding).
//
// The reference's default 1x1 path (Kernels/conv2d.py:364-560,
// _fused_prescan_compute_conv1x1_persistent) builds each tile's group mask
// inline and then dots the active groups. Here a 1x1 output pixel reads one
// input pixel, so there is no halo and no reason to write channel masks to
// HBM first: each CTA turns the x it reads straight into shared-memory masks
// and gathers from them, so x is read from HBM exactly once and y written
// once (the three-by-three path needs a separate mask pass because every
// input pixel feeds nine outputs in different units).
//
// It serves 1x1 stride 2 (the ResNet downsample, which the two-stage path
// does not take). For stride 1 the two stages measured faster on the C2 cell
// (0.54 vs 0.74 ms): both are instruction-issue bound, and this kernel's
// serial load -> gather phases per unit overlap only across CTAs.
//
// Persistent CTAs of 256 threads, several per SM. A unit is (output-channel
// block, image, run of 128 output pixels in row-major order); a CTA takes a
// contiguous range of units, so it loads each weight block into shared memory
// once. Per unit:
//   A. mask build: item (group of VEC output pixels, 32-channel word) loads
//      32 channels of VEC pixels (VEC = 4 -> one 16- or 8-byte load per
//      channel for stride 1) and writes one 32-bit nonzero-channel mask per
//      pixel; the CTA also learns whether any value is neither 0 nor 1.
//   B. gather: warp w owns 8-pixel segments; lane = output channel (CPL
//      slices of 32). For every set bit (ascending channel) it adds the
//      weight vector (binary spikes) or x * weights (FMA, x re-read through
//      L1/L2) into register accumulators; fixed order, no atomics.
//   C. bias and sector-complete stores of the 8 x 32*CPL tile.
#include "conv_kernel.cuh"

namespace sf {
namespace pw {
namespace {

using conv::store_slice;
using conv::WVec;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMinBlocks = 4;   // CTAs per SM the register budget is sized for (2: 1.03 ms, 4: 0.74 ms on C2)
constexpr int kTilePix = 128;   // output pixels per unit (64 measured slower)
constexpr int kR = 8;          // output pixels per warp segment
constexpr int kSegs = kTilePix / kR;


struct PwParams {
  const void* x;
  const void* wp;
  const float* bias;
  void* y;
  int N, C, H, W, Co, Ho, Wo, S;
  int nwords;            // ceil(C / 32)
  int tiles_per_img;     // ceil(Ho*Wo / 128)
  int ncob;              // output-channel blocks of 32*CPL
  long long n_units;
  long long units_per_cta;
  uint32_t w_block_bytes;
};

template <typename T, int V>
struct alignas(sizeof(T) * V) PVec {
  T v[V];
};

template <typename XT, typename WT, int CPL, int VEC>
__global__ void __launch_bounds__(kThreads, kMinBlocks) pointwise_conv_kernel(const PwParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  WT* wsm = reinterpret_cast<WT*>(smem);
  uint32_t* masks = reinterpret_cast<uint32_t*>(smem + ((p.w_block_bytes + 127) / 128) * 128);  // [128][nwords]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const XT* __restrict__ x = static_cast<const XT*>(p.x);
  const int HW = p.H * p.W, HWo = p.Ho * p.Wo;
  const long long u0 = (long long)blockIdx.x * p.units_per_cta;
  const long long u1 = min(p.n_units, u0 + p.units_per_cta);
  const long long upc = (long long)p.N * p.tiles_per_img;  // units per channel block
  int cur_cob = -1;

  for (long long u = u0; u < u1; ++u) {
    const int cob = (int)(u / upc);
    const long long rest = u - (long long)cob * upc;
    const int img = (int)(rest / p.tiles_per_img);
    const int q0 = (int)(rest - (long long)img * p.tiles_per_img) * kTilePix;  // first output pixel
    const int nq = min(kTilePix, HWo - q0);

    __syncthreads();  // previous unit's gather is done with masks (and weights)
    if (cob != cur_cob) {
      // Weight block -> shared memory (16-byte copies; packed blocks are 16-byte multiples).
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const char*>(p.wp) +
                                                        (size_t)cob * p.w_block_bytes);
      uint4* dst = reinterpret_cast<uint4*>(wsm);
      for (uint32_t i = tid; i < p.w_block_bytes / 16; i += kThreads) dst[i] = src[i];
      cur_cob = cob;
    }

    // A. Masks.
    const XT* ximg = x + (size_t)img * p.C * HW;
    uint32_t odd = 0u;
    const int items = (kTilePix / VEC) * p.nwords;
    for (int it = tid; it < items; it += kThreads) {
      const int g = it % (kTilePix / VEC);
      const int wd = it / (kTilePix / VEC);
      const int ql = g * VEC;  // first local pixel of the group
      const int c0 = wd * 32;
      const int cn = min(32, p.C - c0);
      uint32_t m[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) m[e] = 0u;
      if (ql < nq) {
        if constexpr (VEC > 1) {
          // Stride 1, HW % VEC == 0, 16-byte aligned rows: VEC pixels are contiguous.
          const XT* src = ximg + (size_t)c0 * HW + (q0 + ql);
          if (ql + VEC <= nq) {
#pragma unroll 8
            for (int c = 0; c < cn; ++c) {
              const PVec<XT, VEC> r = *reinterpret_cast<const PVec<XT, VEC>*>(src + (size_t)c * HW);
#pragma unroll
              for (int e = 0; e < VEC; ++e) {
                m[e] |= DT<XT>::nz_bit(r.v[e]) << c;
                odd |= DT<XT>::nz_bit(r.v[e]) & DT<XT>::not_one(r.v[e]);
              }
            }
          } else {
            for (int c = 0; c < cn; ++c)
#pragma unroll
              for (int e = 0; e < VEC; ++e)
                if (ql + e < nq) {
                  const XT v = src[(size_t)c * HW + e];
                  m[e] |= DT<XT>::nz_bit(v) << c;
                  odd |= DT<XT>::nz_bit(v) & DT<XT>::not_one(v);
                }
          }
        } else {
          const int q = q0 + ql;
          const int oh = q / p.Wo, ow = q - oh * p.Wo;
          const XT* src = ximg + (size_t)c0 * HW + (size_t)(oh * p.S) * p.W + ow * p.S;
#pragma unroll 8
          for (int c = 0; c < cn; ++c) {
            const XT v = src[(size_t)c * HW];
            m[0] |= DT<XT>::nz_bit(v) << c;
            odd |= DT<XT>::nz_bit(v) & DT<XT>::not_one(v);
          }
        }
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) masks[(ql + e) * p.nwords + wd] = m[e];
    }
    const bool binary = __syncthreads_or(odd != 0u) == 0;

    // B + C. Gather and store, one 8-pixel segment per warp at a time.
    const WT* wl = wsm + lane * CPL;
    for (int sg = warp; sg < kSegs; sg += kWarps) {
      const int ql0 = sg * kR;
      if (ql0 >= nq) break;
      float acc[kR][CPL];
#pragma unroll
      for (int i = 0; i < kR; ++i)
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[i][j] = 0.f;
#pragma unroll
      for (int i = 0; i < kR; ++i) {
        const int ql = ql0 + i;
        if (ql >= nq) break;
        const uint32_t* mrow = masks + ql * p.nwords;
        int q = q0 + ql, ipix = q;
        if (p.S != 1) {
          const int oh = q / p.Wo, ow = q - oh * p.Wo;
          ipix = oh * p.S * p.W + ow * p.S;
        }
        for (int wd = 0; wd < p.nwords; ++wd) {
          uint32_t m = mrow[wd];
          while (m) {
            const int ci = wd * 32 + __ffs(m) - 1;
            m &= m - 1u;
            float w[CPL];
            WVec<WT, CPL, true>::ld(wl + (size_t)ci * (32 * CPL), w);
            if (binary) {
#pragma unroll
              for (int j = 0; j < CPL; ++j) acc[i][j] += w[j];
            } else {
              const float xv = DT<XT>::to_f(__ldg(ximg + (size_t)ci * HW + ipix));
#pragma unroll
              for (int j = 0; j < CPL; ++j) acc[i][j] = fmaf(xv, w[j], acc[i][j]);
            }
          }
        }
      }
      const int nvalid = min(kR, nq - ql0);
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int co0 = (cob * CPL + j) * 32;
        const int co = co0 + lane;
        const float b = (p.bias != nullptr && co < p.Co) ? __ldg(p.bias + co) : 0.f;
        float out[kR];
#pragma unroll
        for (int i = 0; i < kR; ++i) out[i] = acc[i][j] + b;
        XT* ybase = static_cast<XT*>(p.y) + ((size_t)img * p.Co + co0) * HWo + q0 + ql0;
        store_slice<XT, kR>(ybase, HWo, p.Co - co0, lane, nvalid, out);
      }
    }
  }
}

template <typename XT, typename WT, int CPL, int VEC>
sf_status launch(const PwParams& p, size_t smem, cudaStream_t st) {
  auto kern = pointwise_conv_kernel<XT, WT, CPL, VEC>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SF_ERR_CUDA;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess || per_sm < 1)
    return SF_ERR_UNSUPPORTED;
  PwParams q = p;
  const long long ctas = std::min<long long>(q.n_units, (long long)per_sm * num_sms_current_device());
  q.units_per_cta = (q.n_units + ctas - 1) / ctas;
  const long long grid = (q.n_units + q.units_per_cta - 1) / q.units_per_cta;
  kern<<<(unsigned)grid, kThreads, smem, st>>>(q);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <typename XT, typename WT>
sf_status dispatch_cpl(int cpl, bool vec, const PwParams& p, size_t smem, cudaStream_t st) {
  if (vec) {
    if (cpl == 1) return launch<XT, WT, 1, 4>(p, smem, st);
    if (cpl == 2) return launch<XT, WT, 2, 4>(p, smem, st);
    return launch<XT, WT, 4, 4>(p, smem, st);
  }
  if (cpl == 1) return launch<XT, WT, 1, 1>(p, smem, st);
  if (cpl == 2) return launch<XT, WT, 2, 1>(p, smem, st);
  return launch<XT, WT, 4, 1>(p, smem, st);
}

template <typename XT>
sf_status dispatch_w(int wdt, int cpl, bool vec, const PwParams& p, size_t smem, cudaStream_t st) {
  if (wdt == SF_DTYPE_F32) return dispatch_cpl<XT, float>(cpl, vec, p, smem, st);
  if (wdt == SF_DTYPE_BF16) return dispatch_cpl<XT, __nv_bfloat16>(cpl, vec, p, smem, st);
  return SF_ERR_UNSUPPORTED;
}

}  // namespace

// One-pass sparse 1x1 convolution (padding 0, stride 1 or 2). Returns
// SF_ERR_UNSUPPORTED for shapes it does not take (the caller then uses the
// two-stage path).
sf_status run_pointwise(const void* x, const void* w_packed, const float* bias, void* y, int N, int C, int H,
                        int W, int Co, int Ho, int Wo, int S, int xdt, int wdt, cudaStream_t st) {
  if (S != 1 && S != 2) return SF_ERR_UNSUPPORTED;
  const int wsz = (int)dtype_size(wdt);
  const int cpl = conv::weight_block_cpl(C, 1, Co, wsz);
  const size_t wblock = (size_t)C * 32 * cpl * wsz;
  const int nwords = (C + 31) / 32;
  const size_t smem = ((wblock + 127) / 128) * 128 + (size_t)kTilePix * nwords * 4;
  if (smem > 200 * 1024) return SF_ERR_UNSUPPORTED;
  PwParams p;
  p.x = x;
  p.wp = w_packed;
  p.bias = bias;
  p.y = y;
  p.N = N; p.C = C; p.H = H; p.W = W; p.Co = Co; p.Ho = Ho; p.Wo = Wo; p.S = S;
  p.nwords = nwords;
  p.tiles_per_img = (Ho * Wo + kTilePix - 1) / kTilePix;
  p.ncob = conv::weight_blocks(Co, cpl);
  p.n_units = (long long)p.ncob * N * p.tiles_per_img;
  p.units_per_cta = 0;
  p.w_block_bytes = (uint32_t)wblock;
  const int esz = (int)dtype_size(xdt);
  const bool vec = S == 1 && (H * W) % 4 == 0 && (reinterpret_cast<uintptr_t>(x) % (4 * esz)) == 0;
  switch (xdt) {
    case SF_DTYPE_F32: return dispatch_w<float>(wdt, cpl, vec, p, smem, st);
    case SF_DTYPE_F16: return dispatch_w<__half>(wdt, cpl, vec, p, smem, st);
    case SF_DTYPE_BF16: return dispatch_w<__nv_bfloat16>(wdt, cpl, vec, p, smem, st);
  }
  return SF_ERR_INVALID_ARG;
}

}  // namespace pw
}  // namespace sf
