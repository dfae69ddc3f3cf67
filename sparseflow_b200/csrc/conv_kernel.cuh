// Stage 2: gather-style sparse convolution, and the same kernel with a fused
// (BN-folded) bias + LIF epilogue run over all T steps.
//
// Reference semantics: Kernels/conv2d.py:563-886 (3x3 s1/s2) and :236-460
// (1x1) compute y = conv2d(x, w) + bias over active (tile, channel-group)
// blocks; Ops/sparse_conv2d.py:819-834 (F.conv2d) is the exact result they
// approximate. Ops/sparse_fused_conv_lif.py:271-293 defines the LIF update.
//
// B200 design (one persistent CTA of 32 warps per SM):
//   * A work unit is (image, band of TH output rows, block of up to 128 output
//     channels). Its input rows (band + halo) are contiguous per channel in
//     NCHW, so each channel's rows arrive with ONE cp.async.bulk (TMA engine)
//     into a shared-memory stage; cc <= 64 channels form a chunk and 2-4
//     chunk stages are in flight, so HBM streams while the SM computes.
//   * Per chunk every halo pixel gets a 64-bit mask of its nonzero channels
//     (element-level sparsity: exact zeros are skipped, so results are exact).
//     Mask rows carry zero columns on both sides, so taps need no bounds
//     checks. The CTA also learns whether every nonzero of the chunk is 1.0
//     (binary spikes); then the gather adds weight rows without reading x.
//   * Gather: each warp owns a segment of R output pixels of one row; lanes own
//     CPL consecutive output channels. The warp walks the K x ((R-1)S+K) input
//     masks of its segment once; each set bit (ascending channel) is one input
//     event, which feeds up to K taps of the segment with vector weight loads
//     into register accumulators (tap/pixel pairing is resolved at compile
//     time). No atomics, fixed order: bit-identical run to run.
//   * Epilogue: bias (or the LIF update with v held in registers across all T
//     steps), then every lane writes its channels' R-pixel row runs straight
//     to NCHW memory with 16-byte stores.
#pragma once
#include <algorithm>
#include <type_traits>
#include "common.cuh"

namespace sf {
namespace conv {

constexpr int kNWarps = 32;
constexpr int kThreads = kNWarps * 32;
constexpr int kCtasPerSm = 1;
constexpr int kCC = 64;  // max channels per chunk (one mask bit each); p.cc <= kCC is used
constexpr int kMaxStages = 4;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kMaskPadR = 16;  // zero mask columns right of each row (>= (R-1)*S + K - 2)

// Optional phase timing (builds with -DSF_CONV_PHASE_PROFILE only): thread 0
// of every CTA adds the clock cycles it spent in each phase to g_conv_phase.
#ifdef SF_CONV_PHASE_PROFILE
__device__ unsigned long long g_conv_phase[8];
#define SF_PHASE(i)                                   \
  do {                                                \
    if (threadIdx.x == 0) {                           \
      const long long t1_ = clock64();                \
      atomicAdd(&g_conv_phase[i], (unsigned long long)(t1_ - ph_t0)); \
      ph_t0 = t1_;                                    \
    }                                                 \
  } while (0)
#else
#define SF_PHASE(i) \
  do {              \
  } while (0)
#endif

struct ConvParams {
  const void* x;
  const void* wp;
  const float* bias;
  void* y;   // conv output or spikes
  float* v;  // LIF membrane state [N, Co, Ho, Wo]
  uint32_t* err;
  float tau, vth, vreset;
  int hard_reset, decay_input;
  int T, N, C, H, W, Co, Ho, Wo, P;
  int Co_pad;
  int TH, nbands, ncob, n_units, tpr;  // tpr: row segments per output row
  int th_in, Wp;
  int slot_elems;
  int cc;  // channels per chunk
  int nchunks;
  int nstage;
  int use_tmap;         // 1: one 4-D tensor copy per chunk; 0: one bulk copy per channel
  uint32_t box_bytes;   // bytes of one tensor copy
  int mask_off, cb_off, bar_off;  // byte offsets in dynamic smem
};

struct Plan {
  int CPL, R, TH, th_in, nstage, slot_elems, cc, use_tmap;
  int mask_off, cb_off, bar_off, smem;
};

// Per-stage table layout in shared memory: kCC channel base offsets, then
// a uniform flag and the uniform base (element index of channel 0, halo row 0).
constexpr int kCbStride = kCC + 2;

template <typename WT, int CPL>
struct WVec;
template <>
struct WVec<float, 1> {
  static __device__ __forceinline__ void ld(const float* p, float (&w)[1]) { w[0] = __ldg(p); }
};
template <>
struct WVec<float, 2> {
  static __device__ __forceinline__ void ld(const float* p, float (&w)[2]) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(p));
    w[0] = v.x;
    w[1] = v.y;
  }
};
template <>
struct WVec<float, 4> {
  static __device__ __forceinline__ void ld(const float* p, float (&w)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
};
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
template <>
struct WVec<__nv_bfloat16, 1> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&w)[1]) {
    w[0] = __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p)) << 16);
  }
};
template <>
struct WVec<__nv_bfloat16, 2> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&w)[2]) {
    const uint32_t u = __ldg(reinterpret_cast<const unsigned int*>(p));
    w[0] = bf16_lo(u);
    w[1] = bf16_hi(u);
  }
};
template <>
struct WVec<__nv_bfloat16, 4> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&w)[4]) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = bf16_lo(u.x);
    w[1] = bf16_hi(u.x);
    w[2] = bf16_lo(u.y);
    w[3] = bf16_hi(u.y);
  }
};

template <typename XT>
__device__ __forceinline__ bool is_zero_or_one(XT v) {
  const float f = DT<XT>::to_f(v);
  return f == 0.0f || f == 1.0f;
}

// Row run of R values to global memory: 16-byte stores when the whole run is
// valid and aligned, element stores otherwise.
template <typename T, int R>
__device__ __forceinline__ void store_run(T* dst, const float (&v)[R], int nvalid) {
  constexpr int BYTES = R * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
    if (nvalid == R && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      union {
        T e[R];
        uint4 q[BYTES / 16];
      } u;
#pragma unroll
      for (int j = 0; j < R; ++j) u.e[j] = DT<T>::from_f(v[j]);
#pragma unroll
      for (int q = 0; q < BYTES / 16; ++q) reinterpret_cast<uint4*>(dst)[q] = u.q[q];
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < R; ++j)
    if (j < nvalid) dst[j] = DT<T>::from_f(v[j]);
}

template <int R>
__device__ __forceinline__ void load_run(const float* src, float (&v)[R], int nvalid) {
  if constexpr (R % 4 == 0) {
    if (nvalid == R && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
#pragma unroll
      for (int q = 0; q < R / 4; ++q) {
        const float4 f = reinterpret_cast<const float4*>(src)[q];
        v[4 * q] = f.x;
        v[4 * q + 1] = f.y;
        v[4 * q + 2] = f.z;
        v[4 * q + 3] = f.w;
      }
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < R; ++j) v[j] = (j < nvalid) ? src[j] : 0.f;
}

template <int K, int S, int CPL, int R, typename XT, typename WT, bool LIF>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    sparse_conv_kernel(const ConvParams p, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int KK = K * K;
  constexpr int COB = 32 * CPL;
  constexpr int ESZ = (int)sizeof(XT);
  constexpr int QN = (R - 1) * S + K;  // input columns a row segment reads
  static_assert(QN - 2 <= kMaskPadR, "mask padding too small");

  XT* stages = reinterpret_cast<XT*>(smem);
  unsigned long long* masks = reinterpret_cast<unsigned long long*>(smem + p.mask_off);
  int* cbtab = reinterpret_cast<int*>(smem + p.cb_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const XT* __restrict__ x = static_cast<const XT*>(p.x);
  const WT* __restrict__ wp = static_cast<const WT*>(p.wp);
  const int T = LIF ? p.T : 1;
  const int chunks_per_unit = T * p.nchunks;
  const int stage_elems = p.cc * p.slot_elems;
  const int Wp = p.Wp;

  // Warp 0 is the producer: lanes issue the bulk copies (two channels each)
  // of a chunk after lane 0 has armed the stage's mbarrier with the total.
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
    const int c0 = k * p.cc;
    const int cc = min(p.cc, p.C - c0);
    const int s = g % p.nstage;
    const int img = LIF ? t * p.N + n : n;
    int* cbs = cbtab + s * kCbStride;
    if (p.use_tmap) {
      // One tensor copy: box (W, th_in rows from ihs, cc channels, 1 image);
      // rows above/below the image and channels past C arrive as zeros.
      if (lane == 0) {
        cbs[kCC] = 1;
        cbs[kCC + 1] = 0;
        mbar_arrive_expect_tx(&bars[s], p.box_bytes);
        tma_load_4d(stages + (size_t)s * stage_elems, &tmap, 0, ihs, c0, img, &bars[s]);
      }
      return;
    }
    size_t a0[2] = {0, 0};
    uint32_t bytes[2] = {0, 0};
    int e0[2] = {-1, -1};
    const int row_shift = (ih_lo - ihs) * p.W;  // element offset of halo row 0 from the copied rows
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ci = lane + 32 * h;
      if (ci < cc) {
        const size_t start = (((size_t)img * p.C + c0 + ci) * p.H + ih_lo) * (size_t)p.W * ESZ;
        const size_t end = start + (size_t)(ih_hi - ih_lo) * p.W * ESZ;
        a0[h] = start & ~(size_t)15;
        bytes[h] = (uint32_t)(((end + 15) & ~(size_t)15) - a0[h]);
        e0[h] = (int)((start - a0[h]) / ESZ);
        cbs[ci] = ci * p.slot_elems + e0[h] - row_shift;
      }
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, bytes[0] + bytes[1]);
    const int e0_first = __shfl_sync(0xffffffffu, e0[0], 0);
    const bool uniform =
        __all_sync(0xffffffffu, (e0[0] < 0 || e0[0] == e0_first) && (e0[1] < 0 || e0[1] == e0_first));
    if (lane == 0) {
      cbs[kCC] = uniform ? 1 : 0;
      cbs[kCC + 1] = e0_first - row_shift;
      mbar_arrive_expect_tx(&bars[s], total);
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ci = lane + 32 * h;
      if (ci < cc)
        bulk_g2s(stages + (size_t)s * stage_elems + (size_t)ci * p.slot_elems,
                 reinterpret_cast<const char*>(x) + a0[h], bytes[h], &bars[s]);
    }
  };

  // The mask array starts zero; its padding columns are never written again.
  for (int i = tid; i < p.th_in * Wp; i += kThreads) masks[i] = 0ull;
  if (tid == 0) {
    for (int s = 0; s < p.nstage; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    for (int g = 0; g < p.nstage; ++g) issue(g);
  }

  const bool vec_masks = (ESZ == 4) && (p.W % 4 == 0);
#ifdef SF_CONV_PHASE_PROFILE
  long long ph_t0 = clock64();
#endif
  float acc[R][CPL];
  float vreg[LIF ? R : 1][LIF ? CPL : 1];
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
    const int ihs = r0 * S - p.P;
    const int ih_lo = max(0, ihs);
    const int ih_hi = min(p.H, ihs + p.th_in);
    const int co_base = cob * COB;
    const size_t hw_out = (size_t)p.Ho * p.Wo;

    // This warp's row segment.
    const int tr = warp / p.tpr;
    const int seg0 = (warp - tr * p.tpr) * R;
    const bool active = tr < rows_out;
    const int nvalid = min(R, p.Wo - seg0);
    const int orow = r0 + tr;
    const int hl0 = tr * S;
    const int mbase = hl0 * Wp + seg0 * S - p.P + 1;
    const int xbase = hl0 * p.W + seg0 * S - p.P;

    if (LIF && active) {
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int co = co_base + lane * CPL + j;
        float tmp[R];
        if (co < p.Co) {
          load_run<R>(p.v + ((size_t)n * p.Co + co) * hw_out + (size_t)orow * p.Wo + seg0, tmp, nvalid);
        } else {
#pragma unroll
          for (int i = 0; i < R; ++i) tmp[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < R; ++i) vreg[i][j] = tmp[i];
      }
    }

    for (int t = 0; t < T; ++t) {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[i][j] = 0.f;

      for (int k = 0; k < p.nchunks; ++k, ++g) {
        const int s = g % p.nstage;
        const uint32_t parity = (uint32_t)((g / p.nstage) & 1);
        SF_PHASE(4);
        const bool ok = mbar_wait_bounded(&bars[s], parity);
        if (__syncthreads_or(!ok)) {
          if (tid == 0) atomicExch(p.err, 1u);
          return;
        }
        SF_PHASE(0);
        const XT* st = stages + (size_t)s * stage_elems;
        const int* cb = cbtab + s * kCbStride;
        const bool uni = cb[kCC] != 0;
        const int u0 = cb[kCC + 1];
        const int c0 = k * p.cc;
        const int cc = min(p.cc, p.C - c0);

        // Nonzero-channel masks of the halo pixels and whether every nonzero
        // of the chunk is exactly 1.
        bool binary = true;
        if (vec_masks && uni && (u0 & 3) == 0) {
          // Eight threads share four consecutive pixels (16-byte loads), eight
          // channels each; the partial masks are OR-ed with shuffles.
          const int nq = p.W >> 2;
          const int mtotal = p.th_in * nq * 8;
          for (int base = 0; base < mtotal; base += kThreads) {
            const int it = base + tid;  // every lane iterates: full-warp shuffles
            const int part = it & 7, qd = it >> 3;
            const int hl = qd / nq;
            const int qx = qd - hl * nq;
            const int ih = ihs + hl;
            unsigned long long m0 = 0, m1 = 0, m2 = 0, m3 = 0;
            // Part j takes channels j, j+8, j+16, ...: the eight lanes of a
            // quarter-warp then read eight different shared-memory banks.
            if (it < mtotal && ih >= ih_lo && ih < ih_hi && part < cc) {
              const float* src = reinterpret_cast<const float*>(st) + u0 + hl * p.W + qx * 4;
#pragma unroll 4
              for (int ci = part; ci < cc; ci += 8) {
                const float4 f = *reinterpret_cast<const float4*>(src + ci * p.slot_elems);
                const unsigned long long bit = 1ull << ci;
                if (f.x != 0.f) { m0 |= bit; binary &= (f.x == 1.f); }
                if (f.y != 0.f) { m1 |= bit; binary &= (f.y == 1.f); }
                if (f.z != 0.f) { m2 |= bit; binary &= (f.z == 1.f); }
                if (f.w != 0.f) { m3 |= bit; binary &= (f.w == 1.f); }
              }
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
              m0 |= __shfl_xor_sync(0xffffffffu, m0, o);
              m1 |= __shfl_xor_sync(0xffffffffu, m1, o);
              m2 |= __shfl_xor_sync(0xffffffffu, m2, o);
              m3 |= __shfl_xor_sync(0xffffffffu, m3, o);
            }
            if (part == 0 && it < mtotal) {
              unsigned long long* mr = masks + hl * Wp + 1 + qx * 4;
              mr[0] = m0;
              mr[1] = m1;
              mr[2] = m2;
              mr[3] = m3;
            }
          }
        } else {
          // Four threads per pixel, sixteen channels each.
          const int mtotal = p.th_in * p.W * 4;
          for (int base = 0; base < mtotal; base += kThreads) {
            const int it = base + tid;  // every lane iterates: full-warp shuffles
            const int q = it >> 2, part = it & 3;
            const int hl = q / p.W;
            const int iw = q - hl * p.W;
            const int ih = ihs + hl;
            unsigned long long m = 0ull;
            const int cfirst = part * 16;
            if (it < mtotal && ih >= ih_lo && ih < ih_hi && cfirst < cc) {
              const int off = hl * p.W + iw;
              const int cend = min(cc, cfirst + 16);
#pragma unroll 4
              for (int ci = cfirst; ci < cend; ++ci) {
                const XT v = st[(uni ? ci * p.slot_elems + u0 : cb[ci]) + off];
                if (DT<XT>::nonzero(v)) {
                  m |= 1ull << ci;
                  binary &= is_zero_or_one(v);
                }
              }
            }
            m |= __shfl_xor_sync(0xffffffffu, m, 1);
            m |= __shfl_xor_sync(0xffffffffu, m, 2);
            if (part == 0 && it < mtotal) masks[hl * Wp + 1 + iw] = m;
          }
        }
        binary = __syncthreads_and(binary);
        SF_PHASE(1);

        // Gather over this warp's row segment.
        if (active) {
          const WT* wchunk = wp + (size_t)c0 * KK * p.Co_pad + co_base + lane * CPL;
          auto gather = [&](auto binary_tag) {
            constexpr bool BIN = decltype(binary_tag)::value;
#pragma unroll
            for (int kh = 0; kh < K; ++kh) {
#pragma unroll
              for (int qq = 0; qq < QN; ++qq) {
                unsigned long long m = masks[mbase + kh * Wp + qq];
                while (m) {
                  const int ci = __ffsll((long long)m) - 1;
                  m &= m - 1ull;
                  const WT* wc = wchunk + ((size_t)ci * KK + kh * K) * p.Co_pad;
                  float xv = 1.f;
                  if constexpr (!BIN) {
                    const int bse = uni ? ci * p.slot_elems + u0 : cb[ci];
                    xv = DT<XT>::to_f(st[bse + xbase + kh * p.W + qq]);
                  }
#pragma unroll
                  for (int kw = 0; kw < K; ++kw) {
                    const int d = qq - kw;
                    if (d >= 0 && d % S == 0 && d / S < R) {
                      float w[CPL];
                      WVec<WT, CPL>::ld(wc + kw * p.Co_pad, w);
#pragma unroll
                      for (int j = 0; j < CPL; ++j) {
                        if constexpr (BIN)
                          acc[d / S][j] += w[j];
                        else
                          acc[d / S][j] = fmaf(xv, w[j], acc[d / S][j]);
                      }
                    }
                  }
                }
              }
            }
          };
          if (binary)
            gather(std::true_type{});
          else
            gather(std::false_type{});
        }
        __syncthreads();
        SF_PHASE(2);
        if (warp == 0) {
          fence_proxy_async_smem();
          issue(g + p.nstage);
        }
        SF_PHASE(3);
      }

      // Epilogue for (unit, t): straight from registers to NCHW rows.
      if (active) {
        XT* y = static_cast<XT*>(p.y);
        const size_t img = (size_t)(LIF ? t * p.N + n : n);
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int co = co_base + lane * CPL + j;
          if (co < p.Co) {
            const float b = (p.bias != nullptr) ? __ldg(p.bias + co) : 0.f;
            float out[R];
#pragma unroll
            for (int i = 0; i < R; ++i) {
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
              out[i] = val;
            }
            store_run<XT, R>(y + (img * p.Co + co) * hw_out + (size_t)orow * p.Wo + seg0, out, nvalid);
          }
        }
      }
    }

    if (LIF && active) {
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int co = co_base + lane * CPL + j;
        if (co < p.Co) {
          float tmp[R];
#pragma unroll
          for (int i = 0; i < R; ++i) tmp[i] = vreg[i][j];
          store_run<float, R>(p.v + ((size_t)n * p.Co + co) * hw_out + (size_t)orow * p.Wo + seg0, tmp, nvalid);
        }
      }
    }
  }
}

template <int K, int S, int CPL, int R, typename XT, typename WT, bool LIF>
sf_status launch_conv(const ConvParams& p, const CUtensorMap& tmap, int smem, cudaStream_t st) {
  auto kern = sparse_conv_kernel<K, S, CPL, R, XT, WT, LIF>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return SF_ERR_CUDA;
  const int grid = std::max(1, std::min(p.n_units, kCtasPerSm * num_sms_current_device()));
  kern<<<grid, kThreads, smem, st>>>(p, tmap);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <int K, int S, typename XT, typename WT, bool LIF>
sf_status dispatch_cpl(const ConvParams& p, const CUtensorMap& tm, const Plan& pl, cudaStream_t st) {
  if (pl.CPL == 1) return launch_conv<K, S, 1, 8, XT, WT, LIF>(p, tm, pl.smem, st);
  if (pl.CPL == 2) return launch_conv<K, S, 2, 8, XT, WT, LIF>(p, tm, pl.smem, st);
  return launch_conv<K, S, 4, 4, XT, WT, LIF>(p, tm, pl.smem, st);
}

template <typename XT, typename WT, bool LIF>
sf_status dispatch_geom(int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl, cudaStream_t st) {
  if (K == 3 && S == 1) return dispatch_cpl<3, 1, XT, WT, LIF>(p, tm, pl, st);
  if constexpr (!LIF) {
    if (K == 3 && S == 2) return dispatch_cpl<3, 2, XT, WT, LIF>(p, tm, pl, st);
  }
  if (K == 1 && S == 1) return dispatch_cpl<1, 1, XT, WT, LIF>(p, tm, pl, st);
  return SF_ERR_UNSUPPORTED;
}

// Per input dtype: launches the kernel instantiation matching (LIF, weight
// dtype, kernel/stride, channels per lane). Defined in conv_<dtype>.cu.
sf_status dispatch_f32(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                       cudaStream_t st);
sf_status dispatch_f16(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                       cudaStream_t st);
sf_status dispatch_bf16(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                        cudaStream_t st);

template <typename XT>
sf_status dispatch_x(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                     cudaStream_t st) {
  if (lif) {
    if (wdt == SF_DTYPE_F32) return dispatch_geom<XT, float, true>(K, S, p, tm, pl, st);
    if (wdt == SF_DTYPE_BF16) return dispatch_geom<XT, __nv_bfloat16, true>(K, S, p, tm, pl, st);
  } else {
    if (wdt == SF_DTYPE_F32) return dispatch_geom<XT, float, false>(K, S, p, tm, pl, st);
    if (wdt == SF_DTYPE_BF16) return dispatch_geom<XT, __nv_bfloat16, false>(K, S, p, tm, pl, st);
  }
  return SF_ERR_UNSUPPORTED;
}

}  // namespace conv
}  // namespace sf
