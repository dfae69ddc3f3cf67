// Stage 2: gather-style sparse convolution from spike-event masks, and the
// same kernel with a fused (BN-folded) bias + LIF epilogue over all T steps.
//
// Reference semantics: Kernels/conv2d.py:563-886 (3x3 s1/s2) and :236-460
// (1x1) compute y = conv2d(x, w) + bias over active (tile, channel-group)
// blocks; Ops/sparse_conv2d.py:819-834 (F.conv2d) is the exact result they
// approximate. Ops/sparse_fused_conv_lif.py:271-293 defines the LIF update.
//
// Input: the per-pixel nonzero-channel masks written by events.cu (64-bit
// words, [image][h][w][nw]) and, only for images flagged as holding values
// other than 0/1, x itself.
//
// B200 design: one persistent CTA per SM, warp-specialised, no CTA-wide
// barrier after set-up.
//   * Warp 31 is the producer. A work unit is (image, band of TH output rows,
//     column block, block of 32*CPL output channels). For each unit (and time
//     step) it copies the band's mask rows (band + halo; a few KB, contiguous
//     in memory) into a ring of shared-memory stages with one bulk copy (TMA
//     engine), handing stages over through full/empty mbarriers. When the
//     output-channel block changes it also bulk-copies that block's packed
//     weights into shared memory, after the consumers have drained the ring.
//   * Warps 0..30 compute, each owning a segment of R output pixels of one
//     row; lane l owns output channels (slice j) * 32 + l, j < CPL. A warp
//     reads the K x ((R-1)S+K) masks its segment needs (lane = pixel),
//     ballots which are nonzero, and walks their set bits (ascending channel):
//     each is an input event feeding up to K taps of the segment, one vector
//     weight load (the lane's CPL channels) per tap into register accumulators
//     (tap/pixel pairing is resolved at compile time). Binary spikes add weights; other values are
//     read from x and multiplied. No atomics, fixed order: bit-identical runs.
//   * Epilogue: bias (or the LIF update with v held in registers across all T
//     steps); the warp's [channels x R pixels] tile goes to a shared-memory
//     slot and leaves with one asynchronous TMA tensor store, so output
//     traffic overlaps the next unit. Where the row pitch rules TMA out, lane
//     pairs exchange half rows by shuffle so every 16-byte store completes
//     32-byte sectors of NCHW rows.
#pragma once
#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include "common.cuh"

namespace sf {
namespace conv {

#ifndef SF_CONV_NWARPS
#define SF_CONV_NWARPS 32
#endif
// Warps per CTA (one CTA per SM): the last is the producer, the rest compute.
// 24 and 16 warps (more registers per thread) measured slower.
constexpr int kNWarps = SF_CONV_NWARPS;
constexpr int kThreads = kNWarps * 32;
constexpr int kComputeWarps = kNWarps - 1;
#ifndef SF_CONV_ROWS_PER_WARP
#define SF_CONV_ROWS_PER_WARP 1
#endif
// Output rows each compute warp accumulates (non-LIF kernels). Two rows read
// each input event for more outputs per visit (2.5 instead of 3.75 visits per
// event for 3x3 s1), but the doubled accumulator file spills at the 64
// registers a 1024-thread CTA allows and measured 30% slower; one row is the
// default.
constexpr int kRowsPerWarp = SF_CONV_ROWS_PER_WARP;
#ifndef SF_CONV_GATHER_ROW_LOOP
#define SF_CONV_GATHER_ROW_LOOP 1
#endif
constexpr bool kGatherRowLoop = SF_CONV_GATHER_ROW_LOOP != 0;
constexpr int kProducerWarp = kNWarps - 1;
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 227 * 1024;

// Weights live in shared memory when one output-channel block fits this.
constexpr size_t kWsmemMax = 160 * 1024;

// 32-channel slices per lane (CPL) of the packed weight blocks: the widest
// block (<= the layer) whose weights fit shared memory, else the widest block.
inline int weight_block_cpl(int C, int K, int Co, int wsz) {
  const int slices = (Co + 31) / 32;
  for (int cpl = 4; cpl >= 1; cpl /= 2) {
    if (cpl > 1 && cpl > slices) continue;
    if ((size_t)C * K * K * 32 * cpl * wsz <= kWsmemMax) return cpl;
  }
  // No block fits shared memory: weights are read from L2. Four slices per
  // lane walk each event for 128 output channels at once (4-pixel segments).
#ifdef SF_DEV_KNOBS
  // Development builds: SF_CONV_L2_CPL=2 keeps 8-pixel segments.
  const char* e = getenv("SF_CONV_L2_CPL");
  if (e && atoi(e) == 2) return slices >= 2 ? 2 : 1;
#endif
  return slices >= 4 ? 4 : (slices >= 2 ? 2 : 1);
}

// Packed weights: [block][C_in][k*k][32 lanes][CPL], block b holding output
// channels b*32*CPL + j*32 + lane; zero padded past C_out. A lane reads its
// CPL channels of one (channel, tap) with one vector load.
inline int weight_blocks(int Co, int cpl) { return ((Co + 31) / 32 + cpl - 1) / cpl; }


struct ConvParams {
  const void* x;
  const void* wp;
  const float* bias;
  void* y;   // conv output or spikes
  float* v;  // LIF membrane state [N, Co, Ho, Wo]
  uint32_t* err;
  const unsigned long long* masks;  // [T*N][H][W][nw]
  const uint32_t* flags;            // [T*N]: bit 0 set when values other than 0/1 occur
  uint32_t* mask_out;               // LIF: spike masks [T*N][Ho][Wo][2*nw_out] 32-bit halves, or null
  int nw_out;                       // ceil(Co / 64)
  int nw;
  float tau, vth, vreset;
  float inv_tau;  // 1 / tau when tau is a power of two (MODE 3/4)
  int hard_reset, decay_input;
  int T, N, C, H, W, Co, Ho, Wo, P;
  int TH, nbands, ncolb, ncob, n_units, tpr, tpu;  // tpr: row segments per output row; tpu: per unit
  int units_per_cta;
  int th_in;
  int slot_words;  // 64-bit words per mask stage
  int nstage;
  uint32_t w_cob_bytes;  // bytes of one output-channel block of packed weights (WSMEM kernels)
  int tma_store;         // 1: epilogue tiles leave through TMA tensor stores (y map)
  int w_off, stg_off, bar_off;  // byte offsets in dynamic smem
  Gate gate;                    // runs only when the gate selects this path
};

struct Plan {
  int CPL, R, TH, th_in, nstage, slot_words, wsmem, tma_store;
  int w_off, stg_off, bar_off, smem;
};

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

// Packed fp32 pair arithmetic (sm_100 add/fma .f32x2): each half is rounded
// exactly like a scalar add.rn.f32 / fma.rn.f32, one instruction for two.
__device__ __forceinline__ void add_f32x2(float& a0, float& a1, float b0, float b1) {
#ifdef SF_CONV_NO_F32X2
  a0 += b0;
  a1 += b1;
#else
  asm("{\n\t.reg .b64 ra, rb;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 ra, ra, rb;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
#endif
}
__device__ __forceinline__ void fma_f32x2(float& a0, float& a1, float x, float b0, float b1) {
#ifdef SF_CONV_NO_F32X2
  a0 = fmaf(x, b0, a0);
  a1 = fmaf(x, b1, a1);
#else
  asm("{\n\t.reg .b64 ra, rb, rx;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "mov.b64 rx, {%4, %4};\n\tfma.rn.f32x2 ra, rx, rb, ra;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1), "f"(x));
#endif
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
  if constexpr (sizeof(T) == 4 && R % 2 == 0) {
    // Rows whose length breaks 16-byte alignment (W = 14, 7, ...) or ragged
    // last segments: 8-byte stores where two pixels are valid.
    if ((reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
#pragma unroll
      for (int j = 0; j < R; j += 2) {
        if (j + 1 < nvalid)
          *reinterpret_cast<float2*>(dst + j) = make_float2(v[j], v[j + 1]);
        else if (j < nvalid)
          dst[j] = DT<T>::from_f(v[j]);
      }
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

// Writes one slice of a warp's tile: lane l holds R pixels of channel
// co0 + l at base + l * co_stride. For fp32 with R = 8, aligned full rows go
// out as lane-pair stores: lanes 2m and 2m+1 swap half rows so each 16-byte
// store instruction completes sixteen 32-byte sectors.
template <typename T, int R>
__device__ __forceinline__ void store_slice(T* base, size_t co_stride, int co_lim, int lane, int nvalid,
                                            const float (&v)[R]) {
  if constexpr (sizeof(T) == 4 && R == 8) {
#ifdef SF_CONV_V8_STORE
    // sm_100 256-bit stores: each lane writes its channel's 8 pixels, one
    // whole 32-byte sector, with no lane exchange. Off by default: on the C5
    // cell 1.8 % faster at 1 % density but 8.6 % slower at 0 % (each store
    // instruction touches 32 lines instead of 16).
    if (nvalid == R && (reinterpret_cast<uintptr_t>(base) & 31u) == 0 && (co_stride & 7u) == 0) {
      if (lane < co_lim) {
        T* dst = base + (size_t)lane * co_stride;
        asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "f"(v[0]), "f"(v[1]),
                     "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                     : "memory");
      }
      return;
    }
#endif
    if (nvalid == R && (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && (co_stride & 3u) == 0) {
      const int h = lane & 1;
      float recv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) recv[i] = __shfl_xor_sync(0xffffffffu, h ? v[i] : v[4 + i], 1);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int co = (lane & ~1) + q;  // store q writes channel 2m + q: even lane pixels 0..3, odd 4..7
        float4 out;
        if (q == h)
          out = h ? make_float4(v[4], v[5], v[6], v[7]) : make_float4(v[0], v[1], v[2], v[3]);
        else
          out = make_float4(recv[0], recv[1], recv[2], recv[3]);
        if (co < co_lim) *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + co * co_stride + h * 4) = out;
      }
      return;
    }
  }
  if (lane < co_lim) store_run<T, R>(base + lane * co_stride, v, nvalid);
}

// MODE 0: convolution; 1: fused conv + LIF; 2: fused conv + LIF that also
// writes the spikes' event masks (a separate instantiation, so the plain LIF
// kernel carries none of that code); 3 / 4: as 1 / 2 for a power-of-two tau.
template <int K, int S, int CPL, int R, int B, typename XT, typename WT, int MODE, bool WSMEM>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_conv_kernel(const ConvParams p, const __grid_constant__ CUtensorMap ymap) {
  constexpr bool LIF = MODE >= 1;
  constexpr bool EMIT = MODE == 2 || MODE == 4;
  // MODE 3/4: tau a power of two, so x / tau == x * (1 / tau) exactly (both
  // the correctly rounded value of one real number) and the LIF epilogue
  // carries no division code.
  constexpr bool TAU_POW2 = MODE >= 3;
  if (!gate_open(p.gate)) return;  // uniform across the grid: before any barrier
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int KK = K * K;
  constexpr int QN = (R - 1) * S + K;  // input columns a row segment reads
  constexpr int HH = (B - 1) * S + K;  // input rows a warp tile (B output rows) reads
  constexpr int NPOS = HH * QN;        // input pixels a warp tile reads
  static_assert(!LIF || B == 1, "LIF keeps one output row per warp (register budget)");
  constexpr int ROUNDS = (NPOS + 31) / 32;

  unsigned long long* stages = reinterpret_cast<unsigned long long*>(smem);
  const WT* wsm = reinterpret_cast<const WT*>(smem + p.w_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* wbar = empty + kMaxStages;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = LIF ? p.T : 1;
  const int u_begin = blockIdx.x * p.units_per_cta;
  const int u_end = min(p.n_units, u_begin + p.units_per_cta);
  const int upc = p.n_units / p.ncob;  // units per output-channel block
  const size_t wblock = (size_t)p.C * KK * 32 * CPL;  // elements of one packed weight block

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
    if (lane == 0) {
      int g = 0, cur_cob = -1;
      for (int u = u_begin; u < u_end; ++u) {
        const int cob = u / upc;
        const int rest = u - cob * upc;
        const int n = rest / (p.nbands * p.ncolb);
        const int band = (rest - n * p.nbands * p.ncolb) / p.ncolb;
        if (WSMEM && cob != cur_cob) {
          // Drain: every stage handed out so far must be released before the
          // weights in shared memory change.
          for (int q = max(0, g - p.nstage); q < g; ++q) {
            if (!mbar_wait_bounded(&empty[q % p.nstage], (uint32_t)((q / p.nstage) & 1))) {
              atomicExch(p.err, 1u);
              return;
            }
          }
          mbar_arrive_expect_tx(wbar, p.w_cob_bytes);
          bulk_g2s(smem + p.w_off, static_cast<const WT*>(p.wp) + (size_t)cob * wblock, p.w_cob_bytes, wbar);
          cur_cob = cob;
        }
        const int ihs = band * p.TH * S - p.P;
        const int ih_lo = max(0, ihs);
        const int ih_hi = min(p.H, ihs + p.th_in);
        for (int t = 0; t < T; ++t, ++g) {
          const int s = g % p.nstage;
          if (g >= p.nstage) {
            if (!mbar_wait_bounded(&empty[s], (uint32_t)(((g / p.nstage) - 1) & 1))) {
              atomicExch(p.err, 1u);
              return;
            }
          }
          const size_t img = (size_t)(LIF ? t * p.N + n : n);
          const size_t w0 = ((img * p.H + ih_lo) * p.W) * p.nw;
          const size_t w1 = w0 + (size_t)(ih_hi - ih_lo) * p.W * p.nw;
          const size_t a0 = (w0 * 8) & ~(size_t)15, a1 = (w1 * 8 + 15) & ~(size_t)15;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(a1 - a0));
          bulk_g2s(stages + (size_t)s * p.slot_words, reinterpret_cast<const char*>(p.masks) + a0, (uint32_t)(a1 - a0),
                   &full[s]);
        }
      }
    }
    return;
  }

  // ---------------------------------------------------------------- compute
  const XT* __restrict__ x = static_cast<const XT*>(p.x);
  const WT* __restrict__ wglob = static_cast<const WT*>(p.wp);
  float acc[B * R][CPL];
  float vreg[LIF ? CPL : 1][LIF ? R : 1];
  int g = 0, cur_cob = -1, wloads = 0;

  // This warp's place in every unit: row tile tr (output rows tr*B .. +B-1)
  // of the band, segment si of the column block.
  const int tr = warp / p.tpu;
  const int si = warp - tr * p.tpu;
  // Unit coordinates of u_begin; advanced with carries below.
  int cob = u_begin / upc;
  int rest0 = u_begin - cob * upc;
  int n = rest0 / (p.nbands * p.ncolb);
  rest0 -= n * p.nbands * p.ncolb;
  int band = rest0 / p.ncolb;
  int colb = rest0 - band * p.ncolb;
  const size_t hw_out = (size_t)p.Ho * p.Wo;

  for (int u = u_begin; u < u_end; ++u) {
    if (u > u_begin) {
      if (++colb == p.ncolb) {
        colb = 0;
        if (++band == p.nbands) {
          band = 0;
          if (++n == p.N) {
            n = 0;
            ++cob;
          }
        }
      }
    }
    if (WSMEM && cob != cur_cob) {
      if (!mbar_wait_bounded(wbar, (uint32_t)(wloads & 1))) {
        if (lane == 0) atomicExch(p.err, 1u);
        return;
      }
      ++wloads;
      cur_cob = cob;
    }
    const int r0 = band * p.TH;
    const int rows_out = min(p.TH, p.Ho - r0);
    const int ihs = r0 * S - p.P;
    const int ih_lo = max(0, ihs);
    const int ih_hi = min(p.H, ihs + p.th_in);

    // This warp's row segment.
    const int segi = colb * p.tpu + si;
    const int seg0 = segi * R;
    const bool active = tr * B < rows_out && segi < p.tpr;
    const int nrows = min(B, rows_out - tr * B);
    const int nvalid = min(R, p.Wo - seg0);
    const int orow = r0 + tr * B;
    const int ih0 = ihs + tr * B * S;  // input row of the tile's first input row
    const int col0 = seg0 * S - p.P;  // input column of position 0
    const WT* wbase = (WSMEM ? wsm : wglob + (size_t)cob * wblock) + lane * CPL;

    if constexpr (LIF) {
      if (active) {
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int co = (cob * CPL + j) * 32 + lane;
          if (co < p.Co) {
            load_run<R>(p.v + ((size_t)n * p.Co + co) * hw_out + (size_t)orow * p.Wo + seg0, vreg[j], nvalid);
          } else {
#pragma unroll
            for (int i = 0; i < R; ++i) vreg[j][i] = 0.f;
          }
        }
      }
    }

    for (int t = 0; t < T; ++t, ++g) {
      const int s = g % p.nstage;
      const size_t img = (size_t)(LIF ? t * p.N + n : n);
      if (!mbar_wait_bounded(&full[s], (uint32_t)((g / p.nstage) & 1))) {
        if (lane == 0) atomicExch(p.err, 1u);
        return;
      }
      const unsigned long long* st = stages + (size_t)s * p.slot_words;
      const int e0 = (int)((((img * p.H + ih_lo) * p.W) * p.nw) & 1);  // word offset of the aligned copy
      const bool binary = (__ldg(p.flags + img) & 1u) == 0u;

#pragma unroll
      for (int i = 0; i < B * R; ++i)
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[i][j] = 0.f;

      for (int wd = 0; wd < p.nw; ++wd) {
        // Masks of this segment's input pixels (lane = pixel) and which are nonzero.
        unsigned long long mk[ROUNDS];
        uint32_t nzpos[ROUNDS];
#pragma unroll
        for (int rd = 0; rd < ROUNDS; ++rd) {
          const int pos = rd * 32 + lane;
          const int hh = pos / QN;
          const int qq = pos - hh * QN;
          const int ih = ih0 + hh;
          const int iw = col0 + qq;
          unsigned long long m = 0ull;
          if (active && pos < NPOS && iw >= 0 && iw < p.W && ih >= ih_lo && ih < ih_hi)
            m = st[e0 + ((ih - ih_lo) * p.W + iw) * p.nw + wd];
          mk[rd] = m;
          nzpos[rd] = __ballot_sync(0xffffffffu, m != 0ull);
        }
        // Events: each set bit of a nonzero position feeds up to K taps.
        // One output row per warp (B == 1): input row hh feeds only kernel
        // row hh, so the rows run as a loop and only the columns (which fix
        // the accumulator) are unrolled: a third of the code of the fully
        // unrolled form below, which the instruction cache holds better.
        auto gather_rows = [&](auto binary_tag) {
          constexpr bool BIN = decltype(binary_tag)::value;
          const WT* wrow = wbase + (size_t)wd * 64 * KK * 32 * CPL;
#pragma unroll 1
          for (int hh = 0; hh < K; ++hh) {
            const WT* wkh = wrow + hh * K * 32 * CPL;
            const XT* xrow = x + ((img * p.C + wd * 64) * p.H + (ih0 + hh)) * p.W + col0;
#pragma unroll
            for (int qq = 0; qq < QN; ++qq) {
              const int pos = hh * QN + qq;
              uint32_t nzw = nzpos[0];
              unsigned long long mw = mk[0];
#pragma unroll
              for (int rd = 1; rd < ROUNDS; ++rd)
                if ((pos >> 5) == rd) {
                  nzw = nzpos[rd];
                  mw = mk[rd];
                }
              if (((nzw >> (pos & 31)) & 1u) == 0u) continue;
              const unsigned long long m64 = shfl64(mw, pos & 31);
#pragma unroll
              for (int hw = 0; hw < 2; ++hw) {
                uint32_t m = hw ? (uint32_t)(m64 >> 32) : (uint32_t)m64;
                while (m) {
                  const int ci = __ffs(m) - 1 + 32 * hw;
                  m &= m - 1u;
                  const WT* wc = wkh + (size_t)ci * (KK * 32 * CPL);
                  float xv = 1.f;
                  if constexpr (!BIN) xv = DT<XT>::to_f(__ldg(xrow + (size_t)ci * p.H * p.W + qq));
                  float w[K][CPL];
#pragma unroll
                  for (int kw = 0; kw < K; ++kw) {
                    const int d = qq - kw;
                    if (d >= 0 && d % S == 0 && d / S < R) WVec<WT, CPL, WSMEM>::ld(wc + kw * 32 * CPL, w[kw]);
                  }
#pragma unroll
                  for (int kw = 0; kw < K; ++kw) {
                    const int d = qq - kw;
                    if (d >= 0 && d % S == 0 && d / S < R) {
                      float(&a)[CPL] = acc[d / S];
                      if constexpr (CPL % 2 == 0 && std::is_same<WT, float>::value) {
#pragma unroll
                        for (int j = 0; j < CPL; j += 2) {
                          if constexpr (BIN)
                            add_f32x2(a[j], a[j + 1], w[kw][j], w[kw][j + 1]);
                          else
                            fma_f32x2(a[j], a[j + 1], xv, w[kw][j], w[kw][j + 1]);
                        }
                      } else {
#pragma unroll
                        for (int j = 0; j < CPL; ++j) {
                          if constexpr (BIN)
                            a[j] += w[kw][j];
                          else
                            a[j] = fmaf(xv, w[kw][j], a[j]);
                        }
                      }
                    }
                  }
                }
              }
            }
          }
        };
        auto gather = [&](auto binary_tag) {
          constexpr bool BIN = decltype(binary_tag)::value;
#pragma unroll
          for (int pos = 0; pos < NPOS; ++pos) {
            const int hh = pos / QN;
            const int qq = pos - hh * QN;
            if (((nzpos[pos / 32] >> (pos % 32)) & 1u) == 0u) continue;
            const unsigned long long m64 = shfl64(mk[pos / 32], pos % 32);
            const WT* wrow = wbase + (size_t)wd * 64 * KK * 32 * CPL;
#pragma unroll
            for (int hw = 0; hw < 2; ++hw) {
              uint32_t m = hw ? (uint32_t)(m64 >> 32) : (uint32_t)m64;
              while (m) {
                const int ci = __ffs(m) - 1 + 32 * hw;
                m &= m - 1u;
                const WT* wc = wrow + (size_t)ci * (KK * 32 * CPL);
                float xv = 1.f;
                if constexpr (!BIN)
                  xv = DT<XT>::to_f(
                      __ldg(x + ((img * p.C + wd * 64 + ci) * p.H + (ih0 + hh)) * p.W + (col0 + qq)));
#pragma unroll
                for (int kh = 0; kh < K; ++kh) {
                  const int rb = hh - kh;  // S * (output row within the tile)
                  if (rb >= 0 && rb % S == 0 && rb / S < B) {
                    // All taps' weight vectors first, then the adds: with weights
                    // in L2 (no shared-memory copy) the loads overlap.
                    float w[K][CPL];
#pragma unroll
                    for (int kw = 0; kw < K; ++kw) {
                      const int d = qq - kw;
                      if (d >= 0 && d % S == 0 && d / S < R)
                        WVec<WT, CPL, WSMEM>::ld(wc + (kh * K + kw) * 32 * CPL, w[kw]);
                    }
#pragma unroll
                    for (int kw = 0; kw < K; ++kw) {
                      const int d = qq - kw;
                      if (d >= 0 && d % S == 0 && d / S < R) {
                        float(&a)[CPL] = acc[(rb / S) * R + d / S];
                        // Pairs for fp32 weights (a float2 load feeds add.f32x2 directly);
                        // bf16 weights measured faster with scalar adds.
                        if constexpr (CPL % 2 == 0 && std::is_same<WT, float>::value) {
#pragma unroll
                          for (int j = 0; j < CPL; j += 2) {
                            if constexpr (BIN)
                              add_f32x2(a[j], a[j + 1], w[kw][j], w[kw][j + 1]);
                            else
                              fma_f32x2(a[j], a[j + 1], xv, w[kw][j], w[kw][j + 1]);
                          }
                        } else {
#pragma unroll
                          for (int j = 0; j < CPL; ++j) {
                            if constexpr (BIN)
                              a[j] += w[kw][j];
                            else
                              a[j] = fmaf(xv, w[kw][j], a[j]);
                          }
                        }
                      }
                    }
                  }
                }
              }
            }
          }
        };
        // Warp-uniform skip of the unrolled position tests when no input
        // pixel of this tile has an event in this channel word.
        uint32_t nz_any = 0u;
#pragma unroll
        for (int rd = 0; rd < ROUNDS; ++rd) nz_any |= nzpos[rd];
        if (active && nz_any != 0u) {
          if constexpr (B == 1 && kGatherRowLoop) {
            if (binary)
              gather_rows(std::true_type{});
            else
              gather_rows(std::false_type{});
          } else {
            if (binary)
              gather(std::true_type{});
            else
              gather(std::false_type{});
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);

      // Epilogue for (unit, t).
      if (active) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
          if (b >= nrows) break;
          float out[CPL][R];
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const int co = (cob * CPL + j) * 32 + lane;
            const float bias_v = (p.bias != nullptr && co < p.Co) ? __ldg(p.bias + co) : 0.f;
#pragma unroll
            for (int i = 0; i < R; ++i) {
              float val = acc[b * R + i][j] + bias_v;
              if constexpr (LIF) {
                const float vp = vreg[j][i];
                const float vr = p.hard_reset ? p.vreset : 0.f;
                float vt;
                if (p.decay_input)
                  vt = vp + (TAU_POW2 ? __fmul_rn(val - (vp - vr), p.inv_tau) : (val - (vp - vr)) / p.tau);
                else
                  vt = vp - (TAU_POW2 ? __fmul_rn(vp - vr, p.inv_tau) : (vp - vr) / p.tau) + val;
                const bool spk = vt >= p.vth;
                vreg[j][i] = p.hard_reset ? (spk ? p.vreset : vt) : (vt - (spk ? p.vth : 0.f));
                val = spk ? 1.f : 0.f;
              }
              out[j][i] = val;
            }
          }
          if constexpr (EMIT) {
            // Next layer's events: bit (co % 32) of half co / 32 of the 64-bit
            // mask word of each output pixel, the same layout the mask pass
            // writes, so a following convolution can skip that pass.
            {
#pragma unroll
              for (int j = 0; j < CPL; ++j) {
                const int co0 = (cob * CPL + j) * 32;
                if (co0 >= p.Co) break;
                uint32_t mine = 0u;
#pragma unroll
                for (int i = 0; i < R; ++i) {
                  const uint32_t bits = __ballot_sync(0xffffffffu, out[j][i] != 0.f && co0 + lane < p.Co);
                  if (lane == i) mine = bits;
                }
                if (lane < nvalid)
                  p.mask_out[((img * p.Ho + orow + b) * p.Wo + seg0 + lane) * (size_t)(2 * p.nw_out) + co0 / 32] = mine;
              }
            }
          }
          if (p.tma_store) {
            // Tile [32*CPL channels][R pixels] through this warp's staging
            // slot; one TMA tensor store writes it (clipped at the edges).
            XT* stg = reinterpret_cast<XT*>(smem + p.stg_off) + (size_t)warp * (32 * CPL * R);
            if (lane == 0) bulk_wait_group_read0();  // previous tile has left the slot
            __syncwarp();
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
              XT* row = stg + (size_t)(j * 32 + lane) * R;
#pragma unroll
              for (int i = 0; i < R; ++i) row[i] = DT<XT>::from_f(out[j][i]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_4d(&ymap, stg, seg0, orow + b, cob * CPL * 32, (int)img);
              bulk_commit_group();
            }
          } else {
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
              const int co0 = (cob * CPL + j) * 32;
              XT* ybase = static_cast<XT*>(p.y) + (img * p.Co + co0) * hw_out + (size_t)(orow + b) * p.Wo + seg0;
              store_slice<XT, R>(ybase, hw_out, p.Co - co0, lane, nvalid, out[j]);
            }
          }
        }
      }
    }

    if constexpr (LIF) {
      if (active) {
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int co0 = (cob * CPL + j) * 32;
          float* vb = p.v + ((size_t)n * p.Co + co0) * hw_out + (size_t)orow * p.Wo + seg0;
          store_slice<float, R>(vb, hw_out, p.Co - co0, lane, nvalid, vreg[j]);
        }
      }
    }
  }
  if (p.tma_store && lane == 0) bulk_wait_group0();  // stores complete before the CTA leaves
}

template <int K, int S, int CPL, int R, int B, typename XT, typename WT, int MODE, bool WSMEM>
sf_status launch_conv(const ConvParams& p, const CUtensorMap& ymap, int grid, int smem, cudaStream_t st) {
  auto kern = sparse_conv_kernel<K, S, CPL, R, B, XT, WT, MODE, WSMEM>;
  if (!allow_max_smem(reinterpret_cast<const void*>(kern))) return SF_ERR_CUDA;
  kern<<<grid, kThreads, smem, st>>>(p, ymap);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <int K, int S, typename XT, typename WT, int MODE, bool WSMEM>
sf_status dispatch_cpl(const ConvParams& p, const CUtensorMap& ym, int grid, const Plan& pl, cudaStream_t st) {
  constexpr int B = MODE >= 1 ? 1 : kRowsPerWarp;  // output rows per warp
  if (pl.CPL == 1) return launch_conv<K, S, 1, 8, B, XT, WT, MODE, WSMEM>(p, ym, grid, pl.smem, st);
  if (pl.CPL == 2) return launch_conv<K, S, 2, 8, B, XT, WT, MODE, WSMEM>(p, ym, grid, pl.smem, st);
  return launch_conv<K, S, 4, 4, B, XT, WT, MODE, WSMEM>(p, ym, grid, pl.smem, st);
}

template <typename XT, typename WT, int MODE, bool WSMEM>
sf_status dispatch_geom(int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid, const Plan& pl,
                        cudaStream_t st) {
  if (K == 3 && S == 1) return dispatch_cpl<3, 1, XT, WT, MODE, WSMEM>(p, ym, grid, pl, st);
  if constexpr (MODE == 0) {
    if (K == 3 && S == 2) return dispatch_cpl<3, 2, XT, WT, MODE, WSMEM>(p, ym, grid, pl, st);
  }
  if (K == 1 && S == 1) return dispatch_cpl<1, 1, XT, WT, MODE, WSMEM>(p, ym, grid, pl, st);
  return SF_ERR_UNSUPPORTED;
}

// Per input dtype: launches the kernel instantiation matching (mode, weight
// dtype, weights in shared memory, kernel/stride, slices per lane). Defined
// in conv_<dtype>.cu.
sf_status dispatch_f32(int mode, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                       const Plan& pl, cudaStream_t st);
sf_status dispatch_f16(int mode, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                       const Plan& pl, cudaStream_t st);
sf_status dispatch_bf16(int mode, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                        const Plan& pl, cudaStream_t st);

template <typename XT, typename WT, int MODE>
sf_status dispatch_ws(int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid, const Plan& pl,
                      cudaStream_t st) {
  if (pl.wsmem) return dispatch_geom<XT, WT, MODE, true>(K, S, p, ym, grid, pl, st);
  return dispatch_geom<XT, WT, MODE, false>(K, S, p, ym, grid, pl, st);
}

template <typename XT>
sf_status dispatch_x(int mode, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                     const Plan& pl, cudaStream_t st) {
  if (wdt != SF_DTYPE_F32 && wdt != SF_DTYPE_BF16) return SF_ERR_UNSUPPORTED;
  const bool f32 = wdt == SF_DTYPE_F32;
  switch (mode) {
    case 0: return f32 ? dispatch_ws<XT, float, 0>(K, S, p, ym, grid, pl, st)
                       : dispatch_ws<XT, __nv_bfloat16, 0>(K, S, p, ym, grid, pl, st);
    case 1: return f32 ? dispatch_ws<XT, float, 1>(K, S, p, ym, grid, pl, st)
                       : dispatch_ws<XT, __nv_bfloat16, 1>(K, S, p, ym, grid, pl, st);
    case 2: return f32 ? dispatch_ws<XT, float, 2>(K, S, p, ym, grid, pl, st)
                       : dispatch_ws<XT, __nv_bfloat16, 2>(K, S, p, ym, grid, pl, st);
    case 3: return f32 ? dispatch_ws<XT, float, 3>(K, S, p, ym, grid, pl, st)
                       : dispatch_ws<XT, __nv_bfloat16, 3>(K, S, p, ym, grid, pl, st);
    case 4: return f32 ? dispatch_ws<XT, float, 4>(K, S, p, ym, grid, pl, st)
                       : dispatch_ws<XT, __nv_bfloat16, 4>(K, S, p, ym, grid, pl, st);
  }
  return SF_ERR_INVALID_ARG;
}

}  // namespace conv
}  // namespace sf
