// Stage 2: gather-style sparse convolution, and the same kernel with a fused
// (BN-folded) bias + LIF epilogue run over all T steps.
//
// Reference semantics: Kernels/conv2d.py:563-886 (3x3 s1/s2) and :236-460
// (1x1) compute y = conv2d(x, w) + bias over active (tile, channel-group)
// blocks; Ops/sparse_conv2d.py:819-834 (F.conv2d) is the exact result they
// approximate. Ops/sparse_fused_conv_lif.py:271-293 defines the LIF update.
//
// B200 design (one persistent CTA per SM, 16 warps):
//   * A work unit is (image, band of TH output rows, block of up to 128 output
//     channels). Its input rows (band + halo) are contiguous per channel in
//     NCHW, so each channel's rows arrive with ONE cp.async.bulk (TMA engine)
//     into a shared-memory stage; 32 channels form a chunk; 2-4 chunk stages
//     are in flight, so HBM streams while the SM computes.
//   * Per chunk, every halo pixel gets a 32-bit mask of its nonzero channels
//     (element-level sparsity: exact zeros are skipped, so results are exact).
//   * Gather: each warp owns up to PPW output pixels; lanes own output
//     channels (lane, lane+32, ...). For every tap and every set mask bit (in
//     ascending channel order) the warp broadcasts x and FMAs a coalesced
//     weight row into register accumulators. No atomics, deterministic order.
//   * Epilogue: accumulators (+bias, or the LIF update with v held in
//     registers across all T steps) are transposed through shared memory and
//     written back as whole NCHW rows.
#pragma once
#include <algorithm>
#include "common.cuh"

namespace sf {
namespace conv {


constexpr int kNWarps = 32;
constexpr int kThreads = kNWarps * 32;
constexpr int kCC = 16;  // channels per chunk (one mask bit each)
constexpr int kMaxStages = 4;
constexpr int kSmemLimit = 227 * 1024;
// Shared memory the planner aims to stay under, so that the L1 share of the
// SM's 256 KB keeps the packed weights of a layer resident.
constexpr int kSmemBudget = 96 * 1024;


struct ConvParams {
  const void* x;
  const void* wp;
  const float* bias;
  void* y;  // conv output or spikes
  float* v; // LIF membrane state [N, Co, Ho, Wo]
  uint32_t* err;
  float tau, vth, vreset;
  int hard_reset, decay_input;
  int T, N, C, H, W, Co, Ho, Wo, P;
  int Co_pad;
  int TH, nbands, ncob, n_units;
  int th_in;
  int slot_elems;
  int nchunks;
  int nstage;
  int os;
  int out_off, mask_off, e0_off, bar_off;  // byte offsets in dynamic smem
};

template <typename WT>
__device__ __forceinline__ float ldw(const WT* p);
template <>
__device__ __forceinline__ float ldw<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float ldw<__nv_bfloat16>(const __nv_bfloat16* p) {
  const unsigned short b = __ldg(reinterpret_cast<const unsigned short*>(p));
  return __uint_as_float((uint32_t)b << 16);
}

template <int K, int S, int CPL, int PPW, typename XT, typename WT, bool LIF>
__global__ void __launch_bounds__(kThreads, 1) sparse_conv_kernel(const ConvParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int KK = K * K;
  constexpr int COB = 32 * CPL;
  constexpr int ESZ = (int)sizeof(XT);
  // Pixel slots per warp written back per epilogue pass (bounds out_s).
  constexpr int IPASS = (CPL == 4) ? 1 : 2;

  XT* stages = reinterpret_cast<XT*>(smem);
  float* out_s = reinterpret_cast<float*>(smem + p.out_off);
  uint32_t* masks = reinterpret_cast<uint32_t*>(smem + p.mask_off);
  uint8_t* e0tab = smem + p.e0_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const XT* __restrict__ x = static_cast<const XT*>(p.x);
  const WT* __restrict__ wp = static_cast<const WT*>(p.wp);
  const int T = LIF ? p.T : 1;
  const int chunks_per_unit = T * p.nchunks;
  const int stage_elems = kCC * p.slot_elems;

  // Warp 0 is the producer: lane ci issues the bulk copy of channel ci of a
  // chunk after lane 0 has armed the stage's mbarrier with the total bytes.
  auto issue = [&](int g) {
    const int ul = g / chunks_per_unit;
    const int u = blockIdx.x + ul * gridDim.x;
    if (u >= p.n_units) return;
    const int rem = g - ul * chunks_per_unit;
    const int t = rem / p.nchunks;
    const int k = rem - t * p.nchunks;
    const int nb = u / p.ncob;
    const int band = nb % p.nbands;
    const int n = nb / p.nbands;
    const int r0 = band * p.TH;
    const int ihs = r0 * S - p.P;
    const int ih_lo = max(0, ihs);
    const int ih_hi = min(p.H, ihs + p.th_in);
    const int c0 = k * kCC;
    const int cc = min(kCC, p.C - c0);
    const int s = g % p.nstage;
    const size_t img = (size_t)(LIF ? t * p.N + n : n);
    const int ci = lane;
    size_t a0 = 0;
    uint32_t bytes = 0;
    if (ci < cc) {
      const size_t start = ((img * p.C + c0 + ci) * p.H + ih_lo) * (size_t)p.W * ESZ;
      const size_t end = start + (size_t)(ih_hi - ih_lo) * p.W * ESZ;
      a0 = start & ~(size_t)15;
      bytes = (uint32_t)(((end + 15) & ~(size_t)15) - a0);
      e0tab[s * kCC + ci] = (uint8_t)((start - a0) / ESZ);
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
    if (lane == 0) mbar_arrive_expect_tx(&bars[s], total);
    __syncwarp();
    if (ci < cc)
      bulk_g2s(stages + (size_t)s * stage_elems + (size_t)ci * p.slot_elems,
               reinterpret_cast<const char*>(x) + a0, bytes, &bars[s]);
  };

  if (tid == 0) {
    for (int s = 0; s < p.nstage; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    for (int g = 0; g < p.nstage; ++g) issue(g);
  }

  float acc[PPW][CPL];
  float vreg[LIF ? PPW : 1][LIF ? CPL : 1];
  int g = 0;

  for (int ul = 0;; ++ul) {
    const int u = blockIdx.x + ul * gridDim.x;
    if (u >= p.n_units) break;
    const int cob = u % p.ncob;
    const int nb = u / p.ncob;
    const int band = nb % p.nbands;
    const int n = nb / p.nbands;
    const int r0 = band * p.TH;
    const int rows_out = min(p.TH, p.Ho - r0);
    const int npix = rows_out * p.Wo;
    const int ihs = r0 * S - p.P;
    const int ih_lo = max(0, ihs);
    const int ih_hi = min(p.H, ihs + p.th_in);
    const int co_base = cob * COB;
    const size_t hw_out = (size_t)p.Ho * p.Wo;

    if (LIF) {
      // v[n, co, band pixels] -> out_s (coalesced) -> registers, one pass of
      // IPASS pixel slots per warp at a time.
#pragma unroll
      for (int i0 = 0; i0 < PPW; i0 += IPASS) {
        const int pbase = i0 * kNWarps;
        const int pcnt = min(IPASS * kNWarps, npix - pbase);
        for (int idx = tid; idx < COB * pcnt; idx += kThreads) {
          const int col = idx / pcnt, pp = idx - col * pcnt;
          const int co = co_base + col;
          out_s[col * p.os + pp] =
              (co < p.Co) ? p.v[((size_t)n * p.Co + co) * hw_out + (size_t)r0 * p.Wo + pbase + pp] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int ii = 0; ii < IPASS; ++ii) {
          const int pix = warp + (i0 + ii) * kNWarps;
#pragma unroll
          for (int j = 0; j < CPL; ++j)
            vreg[i0 + ii][j] = (pix < npix) ? out_s[(j * 32 + lane) * p.os + warp + ii * kNWarps] : 0.f;
        }
        __syncthreads();
      }
    }

    for (int t = 0; t < T; ++t) {
#pragma unroll
      for (int i = 0; i < PPW; ++i)
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[i][j] = 0.f;

      for (int k = 0; k < p.nchunks; ++k, ++g) {
        const int s = g % p.nstage;
        const uint32_t parity = (uint32_t)((g / p.nstage) & 1);
        const bool ok = mbar_wait_bounded(&bars[s], parity);
        if (__syncthreads_or(!ok)) {
          if (tid == 0) atomicExch(p.err, 1u);
          return;
        }
        const XT* st = stages + (size_t)s * stage_elems;
        const uint8_t* e0 = e0tab + s * kCC;
        const int c0 = k * kCC;
        const int cc = min(kCC, p.C - c0);

        // Per-halo-pixel nonzero-channel masks: four lanes per pixel, four
        // channels each, combined with shuffles.
        const int mtotal = p.th_in * p.W * 4;
        for (int base = 0; base < mtotal; base += kThreads) {
          const int it = base + tid;  // every lane iterates, so the shuffles below see full warps
          const int q = it >> 2, part = it & 3;
          const int hl = q / p.W;
          const int iw = q - hl * p.W;
          const int ih = ihs + hl;
          uint32_t m = 0;
          if (it < mtotal && ih >= ih_lo && ih < ih_hi) {
            const int off = (ih - ih_lo) * p.W + iw;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int ci = part * 4 + u;
              if (ci < cc) m |= (uint32_t)DT<XT>::nonzero(st[ci * p.slot_elems + e0[ci] + off]) << ci;
            }
          }
          m |= __shfl_xor_sync(0xffffffffu, m, 1);
          m |= __shfl_xor_sync(0xffffffffu, m, 2);
          if (part == 0 && it < mtotal) masks[q] = m;
        }
        __syncthreads();

        // Gather.
        const WT* wchunk = wp + (size_t)c0 * KK * p.Co_pad + co_base + lane;
#pragma unroll
        for (int i = 0; i < PPW; ++i) {
          const int pix = warp + i * kNWarps;
          if (pix < npix) {
            const int r = pix / p.Wo;
            const int oc = pix - r * p.Wo;
#pragma unroll
            for (int kh = 0; kh < K; ++kh) {
              const int hl = r * S + kh;
              const int rowoff = (hl + ihs - ih_lo) * p.W;
#pragma unroll
              for (int kw = 0; kw < K; ++kw) {
                const int iw = oc * S + kw - p.P;
                if (iw < 0 || iw >= p.W) continue;
                uint32_t m = masks[hl * p.W + iw];
                while (m) {
                  const int ci = __ffs(m) - 1;
                  m &= m - 1;
                  const float xv = DT<XT>::to_f(st[ci * p.slot_elems + e0[ci] + rowoff + iw]);
                  const WT* wrow = wchunk + ((size_t)ci * KK + kh * K + kw) * p.Co_pad;
#pragma unroll
                  for (int j = 0; j < CPL; ++j) acc[i][j] = fmaf(xv, ldw<WT>(wrow + j * 32), acc[i][j]);
                }
              }
            }
          }
        }
        __syncthreads();
        if (warp == 0) {
          fence_proxy_async_smem();
          issue(g + p.nstage);
        }
      }

      // Epilogue for (unit, t), in passes of IPASS pixel slots per warp.
      {
        XT* y = static_cast<XT*>(p.y);
        const size_t img = (size_t)(LIF ? t * p.N + n : n);
#pragma unroll
        for (int i0 = 0; i0 < PPW; i0 += IPASS) {
          const int pbase = i0 * kNWarps;
          if (pbase < npix) {
#pragma unroll
            for (int ii = 0; ii < IPASS; ++ii) {
              const int i = i0 + ii;
              const int pix = warp + i * kNWarps;
              if (pix < npix) {
#pragma unroll
                for (int j = 0; j < CPL; ++j) {
                  const int col = j * 32 + lane;
                  const int co = co_base + col;
                  const float b = (p.bias != nullptr && co < p.Co) ? __ldg(p.bias + co) : 0.f;
                  float val = acc[i][j] + b;
                  if (LIF) {
                    const float vp = vreg[i][j];
                    const float vr = p.hard_reset ? p.vreset : 0.f;
                    float vt;
                    if (p.decay_input)
                      vt = vp + (val - (vp - vr)) / p.tau;
                    else
                      vt = vp - (vp - vr) / p.tau + val;
                    const bool spk = vt >= p.vth;
                    vreg[i][j] = p.hard_reset ? (spk ? p.vreset : vt) : (vt - (spk ? p.vth : 0.f));
                    val = spk ? 1.f : 0.f;
                  }
                  out_s[col * p.os + warp + ii * kNWarps] = val;
                }
              }
            }
          }
          __syncthreads();
          const int pcnt = min(IPASS * kNWarps, npix - pbase);
          for (int idx = tid; idx < COB * pcnt; idx += kThreads) {
            const int col = idx / pcnt, pp = idx - col * pcnt;
            const int co = co_base + col;
            if (co < p.Co)
              y[(img * p.Co + co) * hw_out + (size_t)r0 * p.Wo + pbase + pp] = DT<XT>::from_f(out_s[col * p.os + pp]);
          }
          __syncthreads();
        }
      }
    }

    if (LIF) {
#pragma unroll
      for (int i0 = 0; i0 < PPW; i0 += IPASS) {
        const int pbase = i0 * kNWarps;
#pragma unroll
        for (int ii = 0; ii < IPASS; ++ii) {
          const int pix = warp + (i0 + ii) * kNWarps;
          if (pix < npix) {
#pragma unroll
            for (int j = 0; j < CPL; ++j) out_s[(j * 32 + lane) * p.os + warp + ii * kNWarps] = vreg[i0 + ii][j];
          }
        }
        __syncthreads();
        const int pcnt = min(IPASS * kNWarps, npix - pbase);
        for (int idx = tid; idx < COB * pcnt; idx += kThreads) {
          const int col = idx / pcnt, pp = idx - col * pcnt;
          const int co = co_base + col;
          if (co < p.Co) p.v[((size_t)n * p.Co + co) * hw_out + (size_t)r0 * p.Wo + pbase + pp] = out_s[col * p.os + pp];
        }
        __syncthreads();
      }
    }
  }
}

struct Plan {
  int CPL, PPW, TH, th_in, nstage, slot_elems, os;
  int out_off, mask_off, e0_off, bar_off, smem;
};

template <int K, int S, int CPL, int PPW, typename XT, typename WT, bool LIF>
sf_status launch_conv(const ConvParams& p, int smem, cudaStream_t st) {
  auto kern = sparse_conv_kernel<K, S, CPL, PPW, XT, WT, LIF>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return SF_ERR_CUDA;
  // Prefer L1 over shared memory: the driver still grants the dynamic shared
  // memory the launch needs, and the rest of the SM's array caches weights.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 0) != cudaSuccess)
    return SF_ERR_CUDA;
  const int grid = std::max(1, std::min(p.n_units, num_sms_current_device()));
  kern<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <int K, int S, typename XT, typename WT, bool LIF>
sf_status dispatch_cpl(const ConvParams& p, const Plan& pl, cudaStream_t st) {
  if (pl.CPL == 1) return launch_conv<K, S, 1, 8, XT, WT, LIF>(p, pl.smem, st);
  if (pl.CPL == 2) return launch_conv<K, S, 2, 8, XT, WT, LIF>(p, pl.smem, st);
  if constexpr (LIF) return launch_conv<K, S, 4, 4, XT, WT, LIF>(p, pl.smem, st);
  else return launch_conv<K, S, 4, 8, XT, WT, LIF>(p, pl.smem, st);
}

template <typename XT, typename WT, bool LIF>
sf_status dispatch_geom(int K, int S, const ConvParams& p, const Plan& pl, cudaStream_t st) {
  if (K == 3 && S == 1) return dispatch_cpl<3, 1, XT, WT, LIF>(p, pl, st);
  if constexpr (!LIF) {
    if (K == 3 && S == 2) return dispatch_cpl<3, 2, XT, WT, LIF>(p, pl, st);
  }
  if (K == 1 && S == 1) return dispatch_cpl<1, 1, XT, WT, LIF>(p, pl, st);
  return SF_ERR_UNSUPPORTED;
}

// Per input dtype: launches the kernel instantiation matching (LIF, weight
// dtype, kernel/stride, channels per lane). Defined in conv_<dtype>.cu.
sf_status dispatch_f32(bool lif, int wdt, int K, int S, const ConvParams& p, const Plan& pl, cudaStream_t st);
sf_status dispatch_f16(bool lif, int wdt, int K, int S, const ConvParams& p, const Plan& pl, cudaStream_t st);
sf_status dispatch_bf16(bool lif, int wdt, int K, int S, const ConvParams& p, const Plan& pl, cudaStream_t st);

template <typename XT>
sf_status dispatch_x(bool lif, int wdt, int K, int S, const ConvParams& p, const Plan& pl, cudaStream_t st) {
  if (lif) {
    if (wdt == SF_DTYPE_F32) return dispatch_geom<XT, float, true>(K, S, p, pl, st);
    if (wdt == SF_DTYPE_BF16) return dispatch_geom<XT, __nv_bfloat16, true>(K, S, p, pl, st);
  } else {
    if (wdt == SF_DTYPE_F32) return dispatch_geom<XT, float, false>(K, S, p, pl, st);
    if (wdt == SF_DTYPE_BF16) return dispatch_geom<XT, __nv_bfloat16, false>(K, S, p, pl, st);
  }
  return SF_ERR_UNSUPPORTED;
}

}  // namespace conv
}  // namespace sf
