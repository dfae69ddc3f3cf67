// Stage 2: gather-style sparse convolution, and the same kernel with a fused
// (BN-folded) bias + LIF epilogue run over all T steps.
//
// Reference semantics: Kernels/conv2d.py:563-886 (3x3 s1/s2) and :236-460
// (1x1) compute y = conv2d(x, w) + bias over active (tile, channel-group)
// blocks; Ops/sparse_conv2d.py:819-834 (F.conv2d) is the exact result they
// approximate. Ops/sparse_fused_conv_lif.py:271-293 defines the LIF update.
//
// B200 design: one persistent CTA per SM, warp-specialised.
//   * Warp 31 is the producer. A work unit is (image, band of TH output rows,
//     block of up to 128 output channels); a chunk is cc <= 64 input channels
//     of the band's input rows (band + halo). The producer fills a ring of
//     shared-memory stages with ONE 4-D tensor TMA copy per chunk (box
//     W x rows x channels; halo rows outside the image arrive as zeros), or
//     with one bulk copy per channel when the row pitch is not 16-byte
//     aligned. Stages hand over through full/empty mbarriers, so loads run
//     ahead of compute and no CTA-wide barrier is needed.
//   * Warps 0..30 compute, each owning a segment of R output pixels of one
//     row; lanes own CPL consecutive output channels. Per chunk a warp builds,
//     in registers, the 64-bit nonzero-channel masks of the K x ((R-1)S+K)
//     input pixels it reads (element-level sparsity: exact zeros are skipped,
//     so results are exact), and learns whether every nonzero is 1.0 (binary
//     spikes: then x is never read again). Each set bit (ascending channel) is
//     an input event that feeds up to K taps of the segment, with one vector
//     weight load per tap into register accumulators; tap/pixel pairing is
//     resolved at compile time. No atomics, fixed order: bit-identical runs.
//   * Weights sit in shared memory for the whole kernel when they fit (one
//     bulk copy per CTA); otherwise they are read through L1/L2.
//   * Epilogue: bias (or the LIF update with v held in registers across all T
//     steps); lane pairs exchange halves by shuffle so every 16-byte store of
//     the warp completes a 32-byte sector of an NCHW row.
#pragma once
#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include "common.cuh"

namespace sf {
namespace conv {

constexpr int kNWarps = 32;
constexpr int kThreads = kNWarps * 32;
constexpr int kComputeWarps = kNWarps - 1;
constexpr int kProducerWarp = kNWarps - 1;
constexpr int kCC = 64;  // max channels per chunk (one mask bit each); p.cc <= kCC is used
constexpr int kMaxStages = 4;
constexpr int kSmemLimit = 227 * 1024;

// Output-channel block of one unit (32 lanes x CPL) and the padded C_out of
// the packed weights.
inline int co_block(int co) { return co <= 32 ? 32 : (co <= 64 ? 64 : 128); }
inline int co_padded(int co) {
  const int b = co_block(co);
  return ((co + b - 1) / b) * b;
}

// Optional phase timing (builds with -DSF_CONV_PHASE_PROFILE only): thread 0
// accumulates cycles per phase in registers and adds them to g_conv_phase.
#ifdef SF_CONV_PHASE_PROFILE
__device__ unsigned long long g_conv_phase[8];
#define SF_PHASE(i)                  \
  do {                               \
    const long long t1_ = clock64(); \
    ph_acc[i] += t1_ - ph_t0;        \
    ph_t0 = t1_;                     \
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
  int TH, nbands, ncob, n_units, tpr;  // tpr: row segments per output row (whole image)
  int tpu, ncolb;                     // row segments per unit, column blocks per band
  int th_in;
  int slot_elems;
  int cc;  // channels per chunk
  int nchunks;
  int nstage;
  int use_tmap;        // 1: one 4-D tensor copy per chunk; 0: one bulk copy per channel
  uint32_t box_bytes;  // bytes of one tensor copy
  uint32_t w_bytes;    // packed weight bytes staged in shared memory (WSMEM kernels)
  int w_off, cb_off, bar_off;  // byte offsets in dynamic smem
};

struct Plan {
  int CPL, R, TH, th_in, nstage, slot_elems, cc, use_tmap, wsmem;
  int w_off, cb_off, bar_off, smem;
};

// Per-stage table in shared memory: kCC channel base offsets, then a uniform
// flag and the uniform base (element index of channel 0, halo row 0).
constexpr int kCbStride = kCC + 2;

template <typename WT, int CPL, bool SMEM>
struct WVec;
template <bool SMEM>
struct WVec<float, 1, SMEM> {
  static __device__ __forceinline__ void ld(const float* p, float (&w)[1]) { w[0] = SMEM ? *p : __ldg(p); }
};
template <bool SMEM>
struct WVec<float, 2, SMEM> {
  static __device__ __forceinline__ void ld(const float* p, float (&w)[2]) {
    const float2 v = SMEM ? *reinterpret_cast<const float2*>(p) : __ldg(reinterpret_cast<const float2*>(p));
    w[0] = v.x;
    w[1] = v.y;
  }
};
template <bool SMEM>
struct WVec<float, 4, SMEM> {
  static __device__ __forceinline__ void ld(const float* p, float (&w)[4]) {
    const float4 v = SMEM ? *reinterpret_cast<const float4*>(p) : __ldg(reinterpret_cast<const float4*>(p));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
};
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
template <bool SMEM>
struct WVec<__nv_bfloat16, 1, SMEM> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&w)[1]) {
    const unsigned short* q = reinterpret_cast<const unsigned short*>(p);
    w[0] = __uint_as_float((uint32_t)(SMEM ? *q : __ldg(q)) << 16);
  }
};
template <bool SMEM>
struct WVec<__nv_bfloat16, 2, SMEM> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&w)[2]) {
    const unsigned int* q = reinterpret_cast<const unsigned int*>(p);
    const uint32_t u = SMEM ? *q : __ldg(q);
    w[0] = bf16_lo(u);
    w[1] = bf16_hi(u);
  }
};
template <bool SMEM>
struct WVec<__nv_bfloat16, 4, SMEM> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&w)[4]) {
    const uint2* q = reinterpret_cast<const uint2*>(p);
    const uint2 u = SMEM ? *q : __ldg(q);
    w[0] = bf16_lo(u.x);
    w[1] = bf16_hi(u.x);
    w[2] = bf16_lo(u.y);
    w[3] = bf16_hi(u.y);
  }
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ unsigned long long shfl64(unsigned long long v, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src);
  const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
  return ((unsigned long long)hi << 32) | lo;
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

// Writes a warp's tile (lane owns channels lane*CPL + j, R pixels each) to
// rows base + co * co_stride. For fp32 with R = 8 and CPL <= 2, aligned full
// segments go out as lane-pair sector stores: lanes 2m and 2m+1 exchange half
// rows so that each 16-byte store instruction completes 16 32-byte sectors.
template <typename T, int CPL, int R>
__device__ __forceinline__ void store_tile(T* base, size_t co_stride, int co_lim, int lane, int nvalid,
                                           const float (&v)[CPL][R]) {
  if constexpr (sizeof(T) == 4 && R == 8 && CPL <= 2) {
    const bool pairable = nvalid == R && (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && (co_stride & 3u) == 0;
    if (pairable) {
      const int h = lane & 1;
      // Send the half the partner stores: the even lane sends pixels 4..7,
      // the odd lane pixels 0..3.
      float recv[CPL][4];
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) recv[j][i] = __shfl_xor_sync(0xffffffffu, h ? v[j][i] : v[j][4 + i], 1);
      // Pair m owns channels 2*CPL*m .. 2*CPL*m + 2*CPL - 1 (even lane's CPL
      // first); store q writes channel 2*CPL*m + q, even lane pixels 0..3,
      // odd lane pixels 4..7.
#pragma unroll
      for (int q = 0; q < 2 * CPL; ++q) {
        const int co = (lane >> 1) * 2 * CPL + q;
        const bool own = (q < CPL) ? (h == 0) : (h == 1);
        const int j = q % CPL;
        float4 out;
        if (own)
          out = h ? make_float4(v[j][4], v[j][5], v[j][6], v[j][7]) : make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
        else
          out = make_float4(recv[j][0], recv[j][1], recv[j][2], recv[j][3]);
        if (co < co_lim) *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + co * co_stride + h * 4) = out;
      }
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int co = lane * CPL + j;
    if (co < co_lim) store_run<T, R>(base + co * co_stride, v[j], nvalid);
  }
}

template <int K, int S, int CPL, int R, typename XT, typename WT, bool LIF, bool WSMEM>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_conv_kernel(const ConvParams p, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int KK = K * K;
  constexpr int COB = 32 * CPL;
  constexpr int ESZ = (int)sizeof(XT);
  constexpr int QN = (R - 1) * S + K;  // input columns a row segment reads
  constexpr int NPOS = K * QN;         // input pixels a row segment reads
  constexpr int ROUNDS = (NPOS + 31) / 32;

  XT* stages = reinterpret_cast<XT*>(smem);
  const WT* wsm = reinterpret_cast<const WT*>(smem + p.w_off);
  int* cbtab = reinterpret_cast<int*>(smem + p.cb_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* wbar = empty + kMaxStages;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const XT* __restrict__ x = static_cast<const XT*>(p.x);
  const int T = LIF ? p.T : 1;
  const int chunks_per_unit = T * p.nchunks;
  const int stage_elems = p.cc * p.slot_elems;

  if (tid == 0) {
    for (int s = 0; s < p.nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kComputeWarps);
    }
    mbar_init(wbar, 1);
    fence_mbar_init();
  }
  __syncthreads();  // the only CTA-wide barrier

  if (warp == kProducerWarp) {
    if (WSMEM && lane == 0) {
      mbar_arrive_expect_tx(wbar, p.w_bytes);
      bulk_g2s(smem + p.w_off, p.wp, p.w_bytes, wbar);
    }
    for (int g = 0;; ++g) {
      const int ul = g / chunks_per_unit;
      const int u = blockIdx.x + ul * gridDim.x;
      if (u >= p.n_units) break;
      const int s = g % p.nstage;
      if (g >= p.nstage) {
        if (!mbar_wait_bounded(&empty[s], (uint32_t)(((g / p.nstage) - 1) & 1))) {
          if (lane == 0) atomicExch(p.err, 1u);
          return;
        }
      }
      const int rem = g - ul * chunks_per_unit;
      const int t = rem / p.nchunks;
      const int k = rem - t * p.nchunks;
      const int nb = u / p.ncob / p.ncolb;
      const int band = nb % p.nbands;
      const int n = nb / p.nbands;
      const int ihs = band * p.TH * S - p.P;
      const int ih_lo = max(0, ihs);
      const int ih_hi = min(p.H, ihs + p.th_in);
      const int c0 = k * p.cc;
      const int cc = min(p.cc, p.C - c0);
      const int img = LIF ? t * p.N + n : n;
      int* cbs = cbtab + s * kCbStride;
      if (p.use_tmap) {
        // Box (W, th_in rows from ihs, cc channels, 1 image); rows outside the
        // image and channels past C arrive as zeros.
        if (lane == 0) {
          cbs[kCC] = 1;
          cbs[kCC + 1] = 0;
          mbar_arrive_expect_tx(&full[s], p.box_bytes);
          tma_load_4d(stages + (size_t)s * stage_elems, &tmap, 0, ihs, c0, img, &full[s]);
        }
        continue;
      }
      size_t a0[2] = {0, 0};
      uint32_t bytes[2] = {0, 0};
      int e0[2] = {-1, -1};
      const int row_shift = (ih_lo - ihs) * p.W;  // halo row 0 sits row_shift elements before the copied rows
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ci = lane + 32 * hh;
        if (ci < cc) {
          const size_t start = (((size_t)img * p.C + c0 + ci) * p.H + ih_lo) * (size_t)p.W * ESZ;
          const size_t end = start + (size_t)(ih_hi - ih_lo) * p.W * ESZ;
          a0[hh] = start & ~(size_t)15;
          bytes[hh] = (uint32_t)(((end + 15) & ~(size_t)15) - a0[hh]);
          e0[hh] = (int)((start - a0[hh]) / ESZ);
          cbs[ci] = ci * p.slot_elems + e0[hh] - row_shift;
        }
      }
      const uint32_t total = __reduce_add_sync(0xffffffffu, bytes[0] + bytes[1]);
      const int e0_first = __shfl_sync(0xffffffffu, e0[0], 0);
      const bool uniform =
          __all_sync(0xffffffffu, (e0[0] < 0 || e0[0] == e0_first) && (e0[1] < 0 || e0[1] == e0_first));
      if (lane == 0) {
        cbs[kCC] = uniform ? 1 : 0;
        cbs[kCC + 1] = e0_first - row_shift;
        mbar_arrive_expect_tx(&full[s], total);
      }
      __syncwarp();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ci = lane + 32 * hh;
        if (ci < cc)
          bulk_g2s(stages + (size_t)s * stage_elems + (size_t)ci * p.slot_elems,
                   reinterpret_cast<const char*>(x) + a0[hh], bytes[hh], &full[s]);
      }
    }
    return;
  }

  // ---------------------------------------------------------------- compute
#ifdef SF_CONV_PHASE_PROFILE
  long long ph_t0 = clock64();
  long long ph_acc[5] = {0, 0, 0, 0, 0};
#endif
  if (WSMEM) {
    if (!mbar_wait_bounded(wbar, 0)) {
      if (lane == 0) atomicExch(p.err, 1u);
      return;
    }
  }
  const WT* __restrict__ wglob = static_cast<const WT*>(p.wp);

  float acc[R][CPL];
  float vreg[LIF ? CPL : 1][LIF ? R : 1];
  int g = 0;

  for (int ul = 0;; ++ul) {
    const int u = blockIdx.x + ul * gridDim.x;
    if (u >= p.n_units) break;
    const int cob = u % p.ncob;
    const int colb = (u / p.ncob) % p.ncolb;
    const int nb = u / p.ncob / p.ncolb;
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
    const int tr = warp / p.tpu;
    const int segi = colb * p.tpu + (warp - tr * p.tpu);
    const int seg0 = segi * R;
    const bool active = tr < rows_out && segi < p.tpr;
    const int nvalid = min(R, p.Wo - seg0);
    const int orow = r0 + tr;
    const int hl0 = tr * S;
    const int col0 = seg0 * S - p.P;  // input column of position qq = 0

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
        for (int i = 0; i < R; ++i) vreg[j][i] = tmp[i];
      }
    }

    for (int t = 0; t < T; ++t) {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[i][j] = 0.f;

      for (int k = 0; k < p.nchunks; ++k, ++g) {
        const int s = g % p.nstage;
        SF_PHASE(4);
        if (!mbar_wait_bounded(&full[s], (uint32_t)((g / p.nstage) & 1))) {
          if (lane == 0) atomicExch(p.err, 1u);
          return;
        }
        SF_PHASE(0);
        const XT* st = stages + (size_t)s * stage_elems;
        const int* cb = cbtab + s * kCbStride;
        const bool uni = cb[kCC] != 0;
        const int u0 = cb[kCC + 1];
        const int c0 = k * p.cc;
        const int cc = min(p.cc, p.C - c0);

        // Nonzero-channel masks of this segment's input pixels (lane = pixel),
        // built 32 channels at a time with constant shifts; `bad` records a
        // nonzero that is not exactly 1.
        unsigned long long mk[ROUNDS];
        uint32_t bad = 0u;
#pragma unroll
        for (int rd = 0; rd < ROUNDS; ++rd) {
          const int pos = rd * 32 + lane;
          const int kh = pos / QN;
          const int qq = pos - kh * QN;
          const int ih = ihs + hl0 + kh;
          const int iw = col0 + qq;
          uint32_t half_m[2] = {0u, 0u};
          if (active && pos < NPOS && iw >= 0 && iw < p.W && ih >= ih_lo && ih < ih_hi) {
            const int off = (hl0 + kh) * p.W + iw;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              if (hh * 32 < cc) {
                uint32_t mm = 0u;
                if (uni) {
                  const XT* src = st + u0 + off + hh * 32 * p.slot_elems;
#pragma unroll
                  for (int q = 0; q < 32; ++q) {
                    if (hh * 32 + q < cc) {
                      const XT v = src[q * p.slot_elems];
                      const uint32_t nzb = DT<XT>::nz_bit(v);
                      mm |= nzb << q;
                      bad |= nzb & DT<XT>::not_one(v);
                    }
                  }
                } else {
#pragma unroll 8
                  for (int q = 0; q < 32; ++q) {
                    if (hh * 32 + q < cc) {
                      const XT v = st[cb[hh * 32 + q] + off];
                      const uint32_t nzb = DT<XT>::nz_bit(v);
                      mm |= nzb << q;
                      bad |= nzb & DT<XT>::not_one(v);
                    }
                  }
                }
                half_m[hh] = mm;
              }
            }
          }
          mk[rd] = ((unsigned long long)half_m[1] << 32) | half_m[0];
        }
        const bool binary = !__any_sync(0xffffffffu, bad != 0u);
        uint32_t nzpos[ROUNDS];
#pragma unroll
        for (int rd = 0; rd < ROUNDS; ++rd) nzpos[rd] = __ballot_sync(0xffffffffu, mk[rd] != 0ull);
        SF_PHASE(1);

        // Gather over the segment's input events.
        if (active) {
          const WT* wchunk = (WSMEM ? wsm : wglob) + (size_t)c0 * KK * p.Co_pad + co_base + lane * CPL;
          const int xrow0 = u0 + hl0 * p.W + col0;
          auto gather = [&](auto binary_tag) {
            constexpr bool BIN = decltype(binary_tag)::value;
#pragma unroll
            for (int pos = 0; pos < NPOS; ++pos) {
              const int kh = pos / QN;
              const int qq = pos - kh * QN;
              if (((nzpos[pos / 32] >> (pos % 32)) & 1u) == 0u) continue;
              unsigned long long m = shfl64(mk[pos / 32], pos % 32);
              while (m) {
                const int ci = __ffsll((long long)m) - 1;
                m &= m - 1ull;
                const WT* wc = wchunk + ((size_t)ci * KK + kh * K) * p.Co_pad;
                float xv = 1.f;
                if constexpr (!BIN) {
                  const int bse = uni ? ci * p.slot_elems + xrow0 : cb[ci] + hl0 * p.W + col0;
                  xv = DT<XT>::to_f(st[bse + kh * p.W + qq]);
                }
#pragma unroll
                for (int kw = 0; kw < K; ++kw) {
                  const int d = qq - kw;
                  if (d >= 0 && d % S == 0 && d / S < R) {
                    float w[CPL];
                    WVec<WT, CPL, WSMEM>::ld(wc + kw * p.Co_pad, w);
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
          };
          if (binary)
            gather(std::true_type{});
          else
            gather(std::false_type{});
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        SF_PHASE(2);
      }

      // Epilogue for (unit, t).
      if (active) {
        const size_t img = (size_t)(LIF ? t * p.N + n : n);
        float out[CPL][R];
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int co = co_base + lane * CPL + j;
          const float b = (p.bias != nullptr && co < p.Co) ? __ldg(p.bias + co) : 0.f;
#pragma unroll
          for (int i = 0; i < R; ++i) {
            float val = acc[i][j] + b;
            if (LIF) {
              const float vp = vreg[j][i];
              const float vr = p.hard_reset ? p.vreset : 0.f;
              float vt;
              if (p.decay_input)
                vt = vp + (val - (vp - vr)) / p.tau;
              else
                vt = vp - (vp - vr) / p.tau + val;
              const bool spk = vt >= p.vth;
              vreg[j][i] = p.hard_reset ? (spk ? p.vreset : vt) : (vt - (spk ? p.vth : 0.f));
              val = spk ? 1.f : 0.f;
            }
            out[j][i] = val;
          }
        }
        XT* ybase = static_cast<XT*>(p.y) + (img * p.Co + co_base) * hw_out + (size_t)orow * p.Wo + seg0;
        store_tile<XT, CPL, R>(ybase, hw_out, p.Co - co_base, lane, nvalid, out);
      }
      SF_PHASE(3);
    }

    if constexpr (LIF) {
      if (active) {
        float* vbase = p.v + ((size_t)n * p.Co + co_base) * hw_out + (size_t)orow * p.Wo + seg0;
        store_tile<float, CPL, R>(vbase, hw_out, p.Co - co_base, lane, nvalid, vreg);
      }
    }
  }
#ifdef SF_CONV_PHASE_PROFILE
  if (tid == 0)
    for (int i = 0; i < 5; ++i) atomicAdd(&g_conv_phase[i], (unsigned long long)ph_acc[i]);
#endif
}

template <int K, int S, int CPL, int R, typename XT, typename WT, bool LIF, bool WSMEM>
sf_status launch_conv(const ConvParams& p, const CUtensorMap& tmap, int smem, cudaStream_t st) {
  auto kern = sparse_conv_kernel<K, S, CPL, R, XT, WT, LIF, WSMEM>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return SF_ERR_CUDA;
  const int grid = std::max(1, std::min(p.n_units, num_sms_current_device()));
  kern<<<grid, kThreads, smem, st>>>(p, tmap);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <int K, int S, typename XT, typename WT, bool LIF, bool WSMEM>
sf_status dispatch_cpl(const ConvParams& p, const CUtensorMap& tm, const Plan& pl, cudaStream_t st) {
  if (pl.CPL == 1) return launch_conv<K, S, 1, 8, XT, WT, LIF, WSMEM>(p, tm, pl.smem, st);
  if (pl.CPL == 2) return launch_conv<K, S, 2, 8, XT, WT, LIF, WSMEM>(p, tm, pl.smem, st);
  return launch_conv<K, S, 4, 4, XT, WT, LIF, WSMEM>(p, tm, pl.smem, st);
}

template <typename XT, typename WT, bool LIF, bool WSMEM>
sf_status dispatch_geom(int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl, cudaStream_t st) {
  if (K == 3 && S == 1) return dispatch_cpl<3, 1, XT, WT, LIF, WSMEM>(p, tm, pl, st);
  if constexpr (!LIF) {
    if (K == 3 && S == 2) return dispatch_cpl<3, 2, XT, WT, LIF, WSMEM>(p, tm, pl, st);
  }
  if (K == 1 && S == 1) return dispatch_cpl<1, 1, XT, WT, LIF, WSMEM>(p, tm, pl, st);
  return SF_ERR_UNSUPPORTED;
}

// Per input dtype: launches the kernel instantiation matching (LIF, weight
// dtype, weights in shared memory, kernel/stride, channels per lane). Defined
// in conv_<dtype>.cu.
sf_status dispatch_f32(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                       cudaStream_t st);
sf_status dispatch_f16(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                       cudaStream_t st);
sf_status dispatch_bf16(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                        cudaStream_t st);

template <typename XT, typename WT, bool LIF>
sf_status dispatch_ws(int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl, cudaStream_t st) {
  if (pl.wsmem) return dispatch_geom<XT, WT, LIF, true>(K, S, p, tm, pl, st);
  return dispatch_geom<XT, WT, LIF, false>(K, S, p, tm, pl, st);
}

template <typename XT>
sf_status dispatch_x(bool lif, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm, const Plan& pl,
                     cudaStream_t st) {
  if (lif) {
    if (wdt == SF_DTYPE_F32) return dispatch_ws<XT, float, true>(K, S, p, tm, pl, st);
    if (wdt == SF_DTYPE_BF16) return dispatch_ws<XT, __nv_bfloat16, true>(K, S, p, tm, pl, st);
  } else {
    if (wdt == SF_DTYPE_F32) return dispatch_ws<XT, float, false>(K, S, p, tm, pl, st);
    if (wdt == SF_DTYPE_BF16) return dispatch_ws<XT, __nv_bfloat16, false>(K, S, p, tm, pl, st);
  }
  return SF_ERR_UNSUPPORTED;
}

}  // namespace conv
}  // namespace sf
