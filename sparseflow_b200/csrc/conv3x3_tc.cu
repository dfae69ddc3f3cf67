// 3x3 / stride 1 / pad 1 convolution of spike inputs on the tcgen05 tensor
// cores (implicit GEMM, integer MMA).
//
// Reference semantics: Kernels/conv2d.py:563-886 computes y = conv2d(x, w) +
// bias over the active (tile, channel-group) blocks, routing dense groups
// through tensor-core dots (:607-638); Ops/sparse_conv2d.py:819-834
// (F.conv2d) is the exact result it approximates.
//
// Exactness. Spikes are 0 or 1, so x is exact as a signed 8-bit integer. The
// weights of output channel co are written in 23-bit fixed point relative to
// s = max |w[co]|: q = rint(w / s * 2^22), split into three signed 8-bit
// digits q = d0 * 2^16 + d1 * 2^8 + d2 (balanced digits, |d0| <= 64). Each
// digit plane is a block of output columns of the same GEMM (N = 3 * 64), so
// one kind::i8 MMA accumulates all three planes as exact int32 sums, and the
// epilogue forms y = s*2^-6 * D0 + s*2^-14 * D1 + s*2^-22 * D2 + bias in
// fp32. The weight error is at most 0.75 * s * 2^-22 per weight: fp32-level
// precision at 1.5x the MMA cost of one bf16 plane. A unit whose input holds
// any value other than 0 or 1 is recomputed in the epilogue with fp32 FMAs
// from x and the fp32 / bf16 weights, and its MMA result is discarded.
//
// Geometry. The N images are stacked vertically into one zero-padded plane
// of pitch Wp = W + 2: padded row R holds image (R-1) / (H+1), row
// (R-1) % (H+1), where row H of each image (the separator) and row 0 are
// zero, as are padded columns 0 and W + 1. Output position o = Ro * Wp + c
// (c < W, Ro % (H+1) < H) reads input position o + kh * Wp + kw for tap
// (kh, kw), so every tap is the A matrix shifted by kh * Wp + kw rows. A is
// kept K-major without swizzle: for each 16-channel slice, one contiguous run
// of 16-byte rows (one per input position), and a shift is a change of the
// descriptor's start address. Tiles are 128 consecutive output positions; a
// unit is U consecutive tiles of one 64-channel output block.
//
// Per CTA (persistent, one per SM, a contiguous range of units):
//   warps 0-14  convert: read x (NCHW, lane = input position: coalesced rows
//               of 32 values per channel), write the int8 A rows of a unit
//               into one of two A buffers, flag non-binary units;
//   warps 15-30 epilogue: per tile, tcgen05.ld the three planes (lane =
//               position), combine, add bias, store y (lane = position: rows
//               of NCHW written as 128-byte runs);
//   warp 31     allocates TMEM (two accumulators of 3 * 64 columns), copies
//               the weight digits of the current output block into shared
//               memory, and issues 9 taps x C/32 MMAs per tile.
// Every mbarrier wait gives up after one second (error word set, CTA
// drains); TMEM is freed before the CTA exits. No TMA multicast.
#include <algorithm>
#include <cmath>
#include <cstring>
#include "conv_kernel.cuh"
#include "tc_common.cuh"
#include "conv3x3_tc.cuh"

namespace sf {
namespace c3tc {
namespace {

using conv::mbar_arrive;

// Warp roles (1024 threads): converters 0..14 (0..13 when the weights are
// streamed, warp 14 then copies weight stages), epilogue 15..30, MMA 31.
// With the LIF epilogue (LM > 0) the CTA has 24 warps: converters 0..6
// (0..5 and the weight-stage copier 6 when streamed), epilogue 7..22, MMA
// 23. The converters have slack at one step's plane, and 768 threads leave
// the epilogue 80 registers for the membranes of two tiles in flight.
constexpr int kEpiWarps = 16;
constexpr int kLifU = 3;  // most tiles per unit with the LIF epilogue
template <int LM>
constexpr int epi0() { return LM ? 7 : 15; }
template <int LM>
constexpr int mma_warp() { return epi0<LM>() + kEpiWarps; }
template <int LM>
constexpr int cta_threads() { return (mma_warp<LM>() + 1) * 32; }
constexpr int kMaxBStages = 8;
constexpr int kMaxKch = 16;  // 16-channel slices per weight stage
constexpr int kM = 128;
constexpr int kTags = 4;

// Division of n < 2^31 by a fixed divisor d >= 1 with a multiply-high
// (round-up reciprocal m = floor(2^32 (2^s - d) / d) + 1, s = ceil(log2 d)):
// q = (umulhi(m, n) + n) >> s.
struct FastDiv {
  uint32_t d, m, s;
};
inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  const uint64_t m = ((1ull << 32) * ((1ull << s) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, s};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (__umulhi(f.m, n) + n) >> f.s;
}

struct Params {
  const void* x;
  const unsigned char* bimg;  // [ncob][9][kcores][N3][16] int8 digits
  const float* scales;        // [3][ncob * CB]
  const float* bias;
  const void* wg;             // gather-packed weights (fallback path)
  int cpl;
  void* y;
  uint32_t* err;
  int N, C, H, W, Co, Wp, Hs;
  FastDiv fd_wp, fd_hs, fd_upcob;  // by Wp, by H + 1, by units per output block
  int kcores, CB, N3, ncob;
  long long ntiles, upcob, nunits, units_per_cta;
  int U;
  uint32_t rows_a, a_plane, a_bytes, b_bytes, a_off, bar_off, tmem_cols;
  // Streamed weights (C_in > 64): nA A buffers, nbs weight stages of kch
  // 16-channel slices of one tap of one 32-channel output block.
  int nA, nbs, kch;
  int ngb;  // TMEM group buffers (2: the epilogue of a group overlaps the next one's MMAs)
  uint32_t b_off, bstage_bytes;
  Gate gate;  // runs only when the gate selects this path
  // Multi-step LIF epilogue (LM > 0): the plane holds the N images of one
  // step, every unit runs t = 0..T-1 in turn (x, y of image t * N + n), and
  // the epilogue turns the preactivation into a spike with membrane v
  // [N, Co, H, W] (fp32, read and written by the same thread at every step).
  int T;
  float* v;
  uint32_t vs_off;  // shared-memory staging of the membranes (streamed weights), or 0
  float tau, vth, vr, inv_tau;
  int hard, decay_input;
};

struct Bars {
  uint64_t a_full[2], a_empty[2], d_full[2], d_empty[2], b_full, b_free;
  uint64_t s_full[kMaxBStages], s_empty[kMaxBStages];
  uint32_t tmem_base;
  uint32_t tag[kTags];  // = u + 1 when unit u holds a value other than 0 / 1
  alignas(16) float2 tab[kEpiWarps][16];
};

template <typename XT>
__device__ __forceinline__ uint32_t raw_bits(XT v) {
  if constexpr (sizeof(XT) == 4)
    return __float_as_uint(v);
  else
    return (uint32_t)(*reinterpret_cast<const unsigned short*>(&v));
}
template <typename XT>
__device__ __forceinline__ constexpr uint32_t one_bits() {
  if constexpr (std::is_same<XT, float>::value) return 0x3f800000u;
  if constexpr (std::is_same<XT, __half>::value) return 0x3c00u;
  return 0x3f80u;
}

__device__ __forceinline__ void st_cs(float* p, float v) { __stcs(p, v); }
__device__ __forceinline__ void st_cs(__half* p, __half v) { __stcs(reinterpret_cast<unsigned short*>(p), __half_as_ushort(v)); }
__device__ __forceinline__ void st_cs(__nv_bfloat16* p, __nv_bfloat16 v) {
  __stcs(reinterpret_cast<unsigned short*>(p), __bfloat16_as_ushort(v));
}

// Writes one output element: the preactivation a itself (LM = 0), or the
// multi-step LIF update of membrane *vm with input a and its spike (LM = 1:
// IEEE division by tau; LM = 2: multiplication by the exact reciprocal of a
// power-of-two tau). Operation order as sf_lif_multistep's, so spikes equal
// those of the convolution followed by that kernel bit for bit.
template <int LM, typename XT>
__device__ __forceinline__ void emit(XT* y, float* vm, float vold, float a, const Params& p) {
  if constexpr (LM == 0) {
    st_cs(y, DT<XT>::from_f(a));
  } else {
    float h;
    if (p.decay_input)
      h = LM == 2 ? vold + __fmul_rn(a - (vold - p.vr), p.inv_tau) : vold + __fdiv_rn(a - (vold - p.vr), p.tau);
    else
      h = LM == 2 ? __fadd_rn(vold - __fmul_rn(vold - p.vr, p.inv_tau), a)
                  : __fadd_rn(vold - __fdiv_rn(vold - p.vr, p.tau), a);
    const bool s = h >= p.vth;
    *vm = p.hard ? (s ? p.vr : h) : (h - (s ? p.vth : 0.f));
    st_cs(y, DT<XT>::from_f(s ? 1.f : 0.f));
  }
}

// Two channels' outputs from their digit sums, with packed fp32 pairs
// (sm_100 add/fma .f32x2, each half rounded exactly like the scalar form):
// x2 = (D2 + 1.5 * 2^23 as float) - 1.5 * 2^23, t = x01 * 256 + x2,
// y = s * t + bias.
__device__ __forceinline__ void combine2(float x01a, float x01b, uint32_t d2a, uint32_t d2b, float4 sb, float& ya,
                                         float& yb) {
  asm("{\n\t.reg .b64 rx, rt, rk, rc, rs, rb;\n\t"
      "mov.b64 rt, {%4, %5};\n\tmov.b64 rc, {%10, %10};\n\tadd.rn.f32x2 rt, rt, rc;\n\t"
      "mov.b64 rx, {%2, %3};\n\tmov.b64 rk, {%11, %11};\n\tfma.rn.f32x2 rt, rx, rk, rt;\n\t"
      "mov.b64 rs, {%6, %7};\n\tmov.b64 rb, {%8, %9};\n\tfma.rn.f32x2 rt, rs, rt, rb;\n\t"
      "mov.b64 {%0, %1}, rt;\n\t}"
      : "=f"(ya), "=f"(yb)
      : "f"(x01a), "f"(x01b), "f"(__int_as_float((int)d2a + 0x4B400000)), "f"(__int_as_float((int)d2b + 0x4B400000)),
        "f"(sb.x), "f"(sb.z), "f"(sb.y), "f"(sb.w), "f"(-12582912.f), "f"(256.f));
}

template <typename WT>
__device__ __forceinline__ float gather_w(const Params& p, int co, int ci, int tap) {
  const int blk = co / (32 * p.cpl), rem = co - blk * 32 * p.cpl;
  const int j = rem >> 5, l = rem & 31;
  const WT* w = static_cast<const WT*>(p.wg) + ((((size_t)blk * p.C + ci) * 9 + tap) * 32 + l) * p.cpl + j;
  return DT<WT>::to_f(*w);
}

// Converter work for one unit, scalar form (any W, any dtype): item =
// (group of 32 A rows, 16-channel slice), lane = A row.
template <typename XT>
__device__ __forceinline__ void convert_unit_scalar(const Params& p, const XT* __restrict__ x, unsigned char* ab,
                                                    long long q0, int warp, int lane, int nconv, uint32_t& nb) {
  const size_t HW = (size_t)p.H * p.W;
  const int kc_n = p.kcores;
  const int items = (int)(p.rows_a / 32) * kc_n;
  for (int it = warp; it < items; it += nconv) {
    const int grp = it / kc_n, kc = it - grp * kc_n;
    const uint32_t q = (uint32_t)q0 + grp * 32 + lane;
    const uint32_t R = fdiv(q, p.fd_wp);
    const int iw = (int)(q - R * p.Wp) - 1;
    const uint32_t R1 = R - 1;  // wraps for the top padding row; R >= 1 is tested below
    const uint32_t img = fdiv(R1 & 0x7fffffffu, p.fd_hs);
    const int h = (int)(R1 - img * p.Hs);
    const bool valid = R >= 1 && iw >= 0 && iw < p.W && h < p.H && img < (uint32_t)p.N;
    const int c0 = kc * 16;
    const XT* src = x + ((size_t)img * p.C + c0) * HW + (size_t)h * p.W + iw;
    const int ne = valid ? min(16, p.C - c0) : 0;
    uint32_t ub[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) ub[e] = e < ne ? raw_bits<XT>(src[(uint32_t)e * (uint32_t)HW]) : 0u;
    uint32_t wv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t w = 0u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t uu = ub[4 * k + b];
        nb |= min(uu, uu ^ one_bits<XT>());  // 0 exactly when uu is 0 or 1
        w |= (uint32_t)(uu != 0u) << (8 * b);
      }
      wv[k] = w;
    }
    *reinterpret_cast<uint4*>(ab + (size_t)kc * p.a_plane + (size_t)(grp * 32 + lane) * 16) =
        make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// Converter work for one unit, fp32 rows of a multiple of 4 values (16-byte
// aligned): lane task = (padded row, quad of 4 columns), item = 32 tasks x
// 8 channels (half of a 16-channel slice); each lane loads 8 float4 (4
// positions x 8 channels), tests x*x == x (true exactly for 0 and 1; -0
// counts as 0, NaN fails) and writes the 8-byte halves of four A rows. The
// two padding columns of each row are written as zeros by a separate loop.
// 16-byte load that does not allocate in L1 (NA) or the default __ldg.
template <bool NA>
__device__ __forceinline__ float4 ld_x4(const float4* p) {
  if constexpr (NA) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
  } else {
    return __ldg(p);
  }
}

template <bool NA>
__device__ __forceinline__ void convert_unit_vec4(const Params& p, const float* __restrict__ x, unsigned char* ab,
                                                  long long q0, int warp, int lane, int nconv, uint32_t& nb) {
  const uint32_t HW = (uint32_t)(p.H * p.W);
  const int kh_n = p.kcores * 2;  // 8-channel halves
  const uint32_t R0 = fdiv((uint32_t)q0, p.fd_wp);
  const uint32_t Rl = fdiv((uint32_t)q0 + p.rows_a - 1, p.fd_wp);
  const int nrows = (int)(Rl - R0) + 1;
  const int qw = p.W >> 2;
  const int ntask = nrows * qw;
  const int ngrp = (ntask + 31) >> 5;
  const int items = ngrp * kh_n;
  const int rows_a = (int)p.rows_a;
  for (int it = warp; it < items; it += nconv) {
    const int grp = it / kh_n, kh = it - grp * kh_n;
    const int t = grp * 32 + lane;
    const int rr = t / qw, k4 = t - rr * qw;
    const uint32_t R = R0 + rr;
    const int r = (int)(R * p.Wp + 1 + 4 * k4 - (uint32_t)q0);  // A row of column 4 * k4
    const uint32_t R1 = R - 1;
    const uint32_t img = fdiv(R1 & 0x7fffffffu, p.fd_hs);
    const int h = (int)(R1 - img * p.Hs);
    const bool inside = t < ntask && r + 3 >= 0 && r < rows_a;
    const bool valid = inside && R >= 1 && h < p.H && img < (uint32_t)p.N;
    const int c0 = kh * 8;
    float4 v[8];
    if (valid) {
      const float4* src =
          reinterpret_cast<const float4*>(x + ((size_t)img * p.C + c0) * HW + (size_t)h * p.W) + k4;
      const uint32_t step = HW >> 2;
      const int ne = min(8, p.C - c0);
      if (ne == 8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = ld_x4<NA>(src + e * step);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = e < ne ? ld_x4<NA>(src + e * step) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint32_t chk = 0u;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      chk |= __float_as_uint(fmaf(v[e].x, v[e].x, -v[e].x)) | __float_as_uint(fmaf(v[e].y, v[e].y, -v[e].y)) |
             __float_as_uint(fmaf(v[e].z, v[e].z, -v[e].z)) | __float_as_uint(fmaf(v[e].w, v[e].w, -v[e].w));
    }
    nb |= chk;
    if (inside) {
      unsigned char* dst = ab + (size_t)(kh >> 1) * p.a_plane + (size_t)(kh & 1) * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t wv[2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const float* a0 = reinterpret_cast<const float*>(&v[4 * kk]);
          const float* a1 = reinterpret_cast<const float*>(&v[4 * kk + 1]);
          const float* a2 = reinterpret_cast<const float*>(&v[4 * kk + 2]);
          const float* a3 = reinterpret_cast<const float*>(&v[4 * kk + 3]);
          // The high byte of 1.0f (0x3f) has bit 0 set; of 0.0f, clear.
          const uint32_t lo = __byte_perm(__float_as_uint(a0[j]), __float_as_uint(a1[j]), 0x0073u);
          const uint32_t hi = __byte_perm(__float_as_uint(a2[j]), __float_as_uint(a3[j]), 0x0073u);
          wv[kk] = __byte_perm(lo, hi, 0x5410u) & 0x01010101u;
        }
        if (r + j >= 0 && r + j < rows_a)
          *reinterpret_cast<uint2*>(dst + (size_t)(r + j) * 16) = make_uint2(wv[0], wv[1]);
      }
    }
  }
  // Padding columns 0 and W + 1 of every padded row the unit touches.
  const int kc_n = p.kcores;
  const int npad = nrows * 2 * kc_n;
  for (int t = warp * 32 + lane; t < npad; t += nconv * 32) {
    const int rr = t / (2 * kc_n), rem = t - rr * 2 * kc_n;
    const int side = rem / kc_n, kc = rem - side * kc_n;
    const int r = (int)((R0 + rr) * p.Wp + (side ? p.W + 1 : 0) - (uint32_t)q0);
    if (r >= 0 && r < rows_a)
      *reinterpret_cast<uint4*>(ab + (size_t)kc * p.a_plane + (size_t)r * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// One tile's epilogue for the warp's channels [cbeg, cbeg + cwq) of output
// block cob: D (three digit planes at TMEM column dcol) -> y, or, for a unit
// holding values other than 0 / 1, fp32 FMAs from x and the weights. x and
// ybase are those of the unit's step; vbase is the LIF membrane (LM > 0).
template <typename XT, typename WT, int LM>
__device__ __forceinline__ void epilogue_tile(const Params& p, const XT* __restrict__ x, XT* ybase, float* vbase,
                                              uint32_t tmem, uint32_t dcol, long long tile, int cob, int qd,
                                              int lane, int cbeg, int cwq, int nco, const float2* tab, bool odd) {
  const size_t HW = (size_t)p.H * p.W;
  const uint32_t o = (uint32_t)(tile * kM) + qd * 32 + lane;
  const uint32_t Ro = fdiv(o, p.fd_wp);
  const int c = (int)(o - Ro * p.Wp);
  const uint32_t img = fdiv(Ro, p.fd_hs);
  const int h = (int)(Ro - img * p.Hs);
  const bool valid = c < p.W && h < p.H && img < (uint32_t)p.N;
  const int cbase = cob * p.CB + cbeg;
  const size_t off = ((size_t)img * p.Co + cbase) * HW + (size_t)h * p.W + c;
  XT* yp = ybase + off;
  float* vp = LM ? vbase + off : nullptr;
  if (!odd && nco == cwq) {
    // Every channel of the warp's quarter exists (cwq is 8 or 16): no
    // per-element bounds checks. The arithmetic is the one below.
    const float4* tb = reinterpret_cast<const float4*>(tab);
    for (int c8 = 0; c8 < cwq; c8 += 8) {
      uint32_t r0[8], r1[8], r2[8];
      const uint32_t ta = tmem + ((uint32_t)(qd * 32) << 16) + dcol + (uint32_t)(cbeg + c8);
      tc::tmem_ld8(ta, r0);
      tc::tmem_ld8(ta + (uint32_t)p.CB, r1);
      tc::tmem_ld8(ta + (uint32_t)(2 * p.CB), r2);
      tc::tmem_wait_ld();
      if (LM == 0 && valid) {
        XT* yc = yp + (size_t)c8 * HW;
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float ya, yb;
          combine2(__int2float_rn((int)r0[e] * 256 + (int)r1[e]), __int2float_rn((int)r0[e + 1] * 256 + (int)r1[e + 1]),
                   r2[e], r2[e + 1], tb[(c8 + e) >> 1], ya, yb);
          st_cs(yc, DT<XT>::from_f(ya));
          st_cs(yc + HW, DT<XT>::from_f(yb));
          yc += 2 * HW;
        }
      } else if (valid) {
        XT* yc = yp + (size_t)c8 * HW;
        float* vc = LM ? vp + (size_t)c8 * HW : nullptr;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float4 sb = tb[(c8 + e) >> 1];
          const float x01 = __int2float_rn((int)r0[e] * 256 + (int)r1[e]);
          const float x2 = __int_as_float((int)r2[e] + 0x4B400000) - 12582912.f;
          const float v = fmaf((e & 1) ? sb.z : sb.x, fmaf(x01, 256.f, x2), (e & 1) ? sb.w : sb.y);
          emit<LM>(yc, vc, LM ? *vc : 0.f, v, p);
          yc += HW;
          if (LM) vc += HW;
        }
      }
    }
  } else if (!odd) {
    const float4* tb = reinterpret_cast<const float4*>(tab);
    for (int c8 = 0; c8 < cwq; c8 += 8) {
      uint32_t r0[8], r1[8], r2[8];
      const uint32_t ta = tmem + ((uint32_t)(qd * 32) << 16) + dcol + (uint32_t)(cbeg + c8);
      tc::tmem_ld8(ta, r0);
      tc::tmem_ld8(ta + (uint32_t)p.CB, r1);
      tc::tmem_ld8(ta + (uint32_t)(2 * p.CB), r2);
      tc::tmem_wait_ld();
      if (valid) {
        // D0 * 256 + D1 is exact in int32 (|D0| <= 64 * 9 * C_in, |D1| <=
        // 128 * 9 * C_in) and converts with one rounding (none below 2^24,
        // e.g. always for C_in <= 64); |D2| < 2^22, so adding 1.5 * 2^23 to
        // its bits gives the float 1.5 * 2^23 + D2 exactly. Then the sum and
        // the scaling round.
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          if (c8 + e >= nco) break;
          const float4 sb = tb[(c8 + e) >> 1];
#pragma unroll
          for (int f = 0; f < 2; ++f) {
            const float x01 = __int2float_rn((int)r0[e + f] * 256 + (int)r1[e + f]);
            const float x2 = __int_as_float((int)r2[e + f] + 0x4B400000) - 12582912.f;
            const float v = fmaf(f ? sb.z : sb.x, fmaf(x01, 256.f, x2), f ? sb.w : sb.y);
            // Evict-first stores: y is not read again here (1.7 % faster on the C5 cell).
            if (c8 + e + f < nco) {
              const uint32_t o2 = (uint32_t)(c8 + e + f) * (uint32_t)HW;
              emit<LM>(yp + o2, LM ? vp + o2 : nullptr, LM ? vp[o2] : 0.f, v, p);
            }
          }
        }
      }
    }
  } else if (valid) {
    const XT* ximg = x + (size_t)img * p.C * HW;
    for (int cc = 0; cc < nco; ++cc) {
      const int co = cbase + cc;
      float acc = 0.f;
      for (int ci = 0; ci < p.C; ++ci) {
        for (int tap = 0; tap < 9; ++tap) {
          const int ih = h + tap / 3 - 1, iw = c + tap % 3 - 1;
          if (ih < 0 || ih >= p.H || iw < 0 || iw >= p.W) continue;
          const float xv = DT<XT>::to_f(ximg[(size_t)ci * HW + (size_t)ih * p.W + iw]);
          if (xv != 0.f) acc = fmaf(xv, gather_w<WT>(p, co, ci, tap), acc);
        }
      }
      const float a = acc + (p.bias ? __ldg(p.bias + co) : 0.f);
      if constexpr (LM == 0)
        yp[(size_t)cc * HW] = DT<XT>::from_f(a);
      else
        emit<LM>(yp + (size_t)cc * HW, vp + (size_t)cc * HW, vp[(size_t)cc * HW], a, p);
    }
  }
}

// LIF epilogue over 8 full channels (streamed weights: cwq = 8), in two
// halves so the membrane loads of the next tile overlap this one: lif_v_load
// fetches a tile's 8 membranes of this thread; lif_tile8 combines the digit
// planes and updates them (the arithmetic of epilogue_tile).
struct TilePos {
  uint32_t off;  // within one step (N * Co * H * W < 2^32, checked on the host)
  bool valid;
};
__device__ __forceinline__ TilePos tile_pos(const Params& p, long long tile, int cob, int qd, int lane, int cbeg) {
  const size_t HW = (size_t)p.H * p.W;
  const uint32_t o = (uint32_t)(tile * kM) + qd * 32 + lane;
  const uint32_t Ro = fdiv(o, p.fd_wp);
  const int c = (int)(o - Ro * p.Wp);
  const uint32_t img = fdiv(Ro, p.fd_hs);
  const int h = (int)(Ro - img * p.Hs);
  TilePos t;
  t.valid = c < p.W && h < p.H && img < (uint32_t)p.N;
  t.off = ((uint32_t)img * (uint32_t)p.Co + (uint32_t)(cob * p.CB + cbeg)) * (uint32_t)HW + (uint32_t)(h * p.W + c);
  return t;
}
// Copies a tile's 8 membranes of this thread into its shared-memory slab
// (8 floats 32 apart) with asynchronous 4-byte copies: no registers wait on
// them. Each thread reads back only what it copied itself.
__device__ __forceinline__ void lif_v_stage(const Params& p, const TilePos& tp, float* slab) {
  if (!tp.valid) return;
  const uint32_t HW = (uint32_t)(p.H * p.W);
  const float* vp = p.v + tp.off;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(slab + e * 32)), "l"(vp + e * HW)
                 : "memory");
}
template <typename XT, int LM>
__device__ __forceinline__ void lif_tile8(const Params& p, XT* ybase, const TilePos& tp, uint32_t ta,
                                          const float* vo, const float2* tab) {
  const size_t HW = (size_t)p.H * p.W;
  // The membranes wait in shared memory, so all three digit planes load
  // with one TMEM round trip.
  uint32_t r0[8], r1[8], r2[8];
  tc::tmem_ld8(ta, r0);
  tc::tmem_ld8(ta + (uint32_t)p.CB, r1);
  tc::tmem_ld8(ta + (uint32_t)(2 * p.CB), r2);
  tc::tmem_wait_ld();
  if (!tp.valid) return;
  const float4* tb = reinterpret_cast<const float4*>(tab);
  XT* yc = ybase + tp.off;
  float* vc = p.v + tp.off;
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    float a0, a1;
    combine2(__int2float_rn((int)r0[e] * 256 + (int)r1[e]), __int2float_rn((int)r0[e + 1] * 256 + (int)r1[e + 1]),
             r2[e], r2[e + 1], tb[e >> 1], a0, a1);
    emit<LM>(yc, vc, vo[e * 32], a0, p);
    emit<LM>(yc + HW, vc + HW, vo[(e + 1) * 32], a1, p);
    yc += 2 * HW;
    vc += 2 * HW;
  }
}

#ifdef SF_C3TC_PROF
__device__ unsigned long long g_c3tc_prof[8];
#define PROF_T0() const long long pt0_ = clock64()
#define PROF_ADD(slot) atomicAdd(&g_c3tc_prof[slot], (unsigned long long)(clock64() - pt0_))
#else
#define PROF_T0()
#define PROF_ADD(slot)
#endif

// STREAM = false: the weight digits of one output block stay in shared
// memory (C_in <= 64); D per tile, double buffered. STREAM = true: weight
// stages stream past the resident A of a unit once per output block; D per
// (unit, block) group of U tiles, double buffered.
// MMAs of one weight stage (PK slice pairs) for the nt tiles of a unit; tile j
// accumulates at TMEM column dt0 + j*n3 and reads A 128 rows further on.
// Unrolled per PK: the MMA warp's issue loop bounds the streamed layers.
template <int PK>
__device__ __forceinline__ void issue_stage(uint32_t dt0, uint32_t n3, int nt, uint64_t a0, uint64_t bstage,
                                            uint64_t astep, uint64_t bstep, uint32_t idesc, uint32_t first) {
  for (int j = 0; j < nt; ++j) {
    const uint32_t dt = dt0 + (uint32_t)j * n3;
    const uint64_t ad = a0 + (uint64_t)(j * kM);  // 128 rows of 16 bytes
    tc::mma_s8(dt, ad, bstage, idesc, first);
#pragma unroll
    for (int kp = 1; kp < PK; ++kp) tc::mma_s8(dt, ad + kp * astep, bstage + kp * bstep, idesc, 1u);
  }
}

// Any other pair count (C_in of 96, 160, 192, ...): a plain loop.
__device__ __forceinline__ void issue_stage_n(int pk, uint32_t dt0, uint32_t n3, int nt, uint64_t a0,
                                              uint64_t bstage, uint64_t astep, uint64_t bstep, uint32_t idesc,
                                              uint32_t first) {
  for (int j = 0; j < nt; ++j) {
    const uint32_t dt = dt0 + (uint32_t)j * n3;
    const uint64_t ad = a0 + (uint64_t)(j * kM);
    tc::mma_s8(dt, ad, bstage, idesc, first);
#pragma unroll 1
    for (int kp = 1; kp < pk; ++kp) tc::mma_s8(dt, ad + kp * astep, bstage + kp * bstep, idesc, 1u);
  }
}

template <typename XT, typename WT, bool VEC, bool STREAM, int LM>
__global__ void __launch_bounds__(cta_threads<LM>(), 1) conv3x3_tc_kernel(const Params p) {
  constexpr int kEpi0 = epi0<LM>();
  constexpr int kMmaWarp = mma_warp<LM>();
  constexpr int kConv = STREAM ? kEpi0 - 1 : kEpi0;  // converter warps
  constexpr int kProducer = kEpi0 - 1;              // weight-stage copier (STREAM)
  if (!gate_open(p.gate)) return;  // uniform across the grid: before any barrier or TMEM allocation
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* bsm = smem + p.b_off;
  unsigned char* abuf = smem + p.a_off;
  Bars* bars = reinterpret_cast<Bars*>(smem + p.bar_off);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long u0 = (long long)blockIdx.x * p.units_per_cta;
  const long long u1 = min(p.nunits, u0 + p.units_per_cta);
  // Every role walks the CTA's units in order, each T times (t = 0..T-1)
  // with the LIF epilogue, once otherwise: nu steps, step i = unit
  // u0 + i / TT at t = i % TT.
  const int TT = LM ? p.T : 1;
  const int nu = (int)max(0ll, u1 - u0) * TT;
  const XT* __restrict__ x = static_cast<const XT*>(p.x);
  const size_t step_elems = (size_t)p.N * p.H * p.W;  // per channel, one step
  // Unit u: tiles [t0, t0 + nt) of output block cob (resident weights), or of
  // every block in turn (streamed weights: then cob of the unit is 0).
  auto unit_of = [&](long long u, int& cob, long long& t0, int& nt) {
    cob = STREAM ? 0 : (int)fdiv((uint32_t)u, p.fd_upcob);
    t0 = (u - (long long)cob * p.upcob) * p.U;
    nt = (int)min((long long)p.U, p.ntiles - t0);
  };
  // Step i: its unit, its t, and the tag key (unique per step of the grid).
  auto step_of = [&](int i, long long& u, int& t) {
    const int iu = LM ? i / TT : i;
    t = i - iu * TT;
    u = u0 + iu;
  };

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->a_full[i], kConv);
      mbar_init(&bars->a_empty[i], 1);
      mbar_init(&bars->d_full[i], 1);
      mbar_init(&bars->d_empty[i], kEpiWarps);
    }
    for (int i = 0; i < kMaxBStages; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], 1);
    }
    mbar_init(&bars->b_full, 1);
    mbar_init(&bars->b_free, 1);
    for (int i = 0; i < kTags; ++i) bars->tag[i] = 0u;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars->tmem_base)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool failed = false;

  if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_s8(kM, p.N3);
      const uint32_t bsa = smem_u32(bsm);
      const uint32_t lbo_b = (uint32_t)p.N3 * 16u;
      // Descriptors advance by adding to their address fields (16-byte
      // units; no offset here carries out of the 14-bit field).
      const uint64_t astep = (uint64_t)(2u * p.a_plane) >> 4, bstep = (uint64_t)(2u * lbo_b) >> 4;
      if constexpr (!STREAM) {
        // The MMAs of one tile walk tap (kh, kw) x pair of 16-channel slices;
        // B advances by one slice pair per MMA, A by the tap's row shift plus
        // one slice pair.
        const int pk = p.kcores / 2;
        const uint64_t bbase = tc::desc_interleave(bsa, lbo_b, 128u);
        int cur_cob = -1, bloads = 0;
        long long g = 0;  // tiles issued by this CTA
        for (int i = 0; i < nu && !failed; ++i) {
          int cob, nt, ts;
          long long t0, uu;
          step_of(i, uu, ts);
          unit_of(uu, cob, t0, nt);
          if (cob != cur_cob) {
            if (cur_cob >= 0) {
              // Every MMA reading the old weights must finish before they are replaced.
              tc::mma_commit(&bars->b_free);
              if (!tc::mbar_wait_sleep(&bars->b_free, (uint32_t)((bloads - 1) & 1))) {
                failed = true;
                break;
              }
            }
            mbar_arrive_expect_tx(&bars->b_full, p.b_bytes);
            const unsigned char* src = p.bimg + (size_t)cob * p.b_bytes;
            for (uint32_t off = 0; off < p.b_bytes; off += 32768u)
              bulk_g2s(bsm + off, src + off, min(32768u, p.b_bytes - off), &bars->b_full);
            if (!tc::mbar_wait_sleep(&bars->b_full, (uint32_t)(bloads & 1))) {
              failed = true;
              break;
            }
            ++bloads;
            cur_cob = cob;
          }
          const int a = i & 1;
          if (!tc::mbar_wait_sleep(&bars->a_full[a], (uint32_t)((i >> 1) & 1))) {
            failed = true;
            break;
          }
          tc::fence_after();
          const uint32_t asa = smem_u32(abuf + (size_t)a * p.a_bytes);
          for (int j = 0; j < nt; ++j, ++g) {
            const int d = (int)(g & 1);
            if (g >= 2 && !tc::mbar_wait_sleep(&bars->d_empty[d], (uint32_t)(((g >> 1) - 1) & 1))) {
              failed = true;
              break;
            }
            tc::fence_after();
            const uint32_t dt = tmem + (uint32_t)(d * p.N3);
            const uint64_t abase = tc::desc_interleave(asa + (uint32_t)(j * kM) * 16u, p.a_plane, 128u);
            // Nine taps of one or two slice pairs, fully unrolled per case.
            if (pk == 2) {
#pragma unroll
              for (int t = 0; t < 9; ++t) {
                const uint64_t ad = abase + (uint64_t)((t / 3) * p.Wp + t % 3);
                tc::mma_s8(dt, ad, bbase + (uint64_t)(2 * t) * bstep, idesc, t == 0 ? 0u : 1u);
                tc::mma_s8(dt, ad + astep, bbase + (uint64_t)(2 * t + 1) * bstep, idesc, 1u);
              }
            } else {
#pragma unroll
              for (int t = 0; t < 9; ++t) {
                const uint64_t ad = abase + (uint64_t)((t / 3) * p.Wp + t % 3);
                tc::mma_s8(dt, ad, bbase + (uint64_t)t * bstep, idesc, t == 0 ? 0u : 1u);
              }
            }
            tc::mma_commit(&bars->d_full[d]);
          }
          if (failed) break;
          tc::mma_commit(&bars->a_empty[a]);
        }
      } else {
        const int nkc = p.kcores / p.kch;  // weight stages per tap
        const int pkc = p.kch / 2;          // MMAs per tile per stage
        long long g = 0;                    // (unit, block) groups issued
        int s = 0;                          // weight stage slot
        uint32_t sphase = 0;                // its mbarrier phase (flips at each ring wrap)
        for (int i = 0; i < nu && !failed; ++i) {
          int cob0, nt, ts;
          long long t0, uu;
          step_of(i, uu, ts);
          unit_of(uu, cob0, t0, nt);
          const int a = i % p.nA;
          {
            PROF_T0();
            if (!tc::mbar_wait_sleep(&bars->a_full[a], (uint32_t)((i / p.nA) & 1))) {
              failed = true;
              break;
            }
            PROF_ADD(0);
          }
          tc::fence_after();
          const uint32_t asa = smem_u32(abuf + (size_t)a * p.a_bytes);
          for (int cob = 0; cob < p.ncob && !failed; ++cob, ++g) {
            const int gb = p.ngb == 2 ? (int)(g & 1) : 0;
            const long long gr = p.ngb == 2 ? (g >> 1) : g;  // uses of this buffer so far
            {
              PROF_T0();
              if (g >= p.ngb && !tc::mbar_wait_sleep(&bars->d_empty[gb], (uint32_t)((gr - 1) & 1))) {
                failed = true;
                break;
              }
              PROF_ADD(1);
            }
            tc::fence_after();
            for (int tap = 0; tap < 9 && !failed; ++tap) {
              const int kh = tap / 3, kw = tap - kh * 3;
              for (int kc = 0; kc < nkc; ++kc) {
                {
                  PROF_T0();
                  if (!tc::mbar_wait_sleep(&bars->s_full[s], sphase)) {
                    failed = true;
                    break;
                  }
                  PROF_ADD(2);
                }
                PROF_T0();
                tc::fence_after();
                const uint64_t bstage = tc::desc_interleave(bsa + (uint32_t)s * p.bstage_bytes, lbo_b, 128u);
                const uint64_t a0 = tc::desc_interleave(asa + (uint32_t)(kh * p.Wp + kw) * 16u +
                                                            (uint32_t)(kc * p.kch) * p.a_plane,
                                                        p.a_plane, 128u);
                const uint32_t first = (tap | kc) == 0 ? 0u : 1u;
                // One stage: kch/2 slice pairs for each tile of the unit.
                const uint32_t dt0 = tmem + (uint32_t)(gb * p.U * p.N3);
                if (pkc == 8)
                  issue_stage<8>(dt0, p.N3, nt, a0, bstage, astep, bstep, idesc, first);
                else if (pkc == 4)
                  issue_stage<4>(dt0, p.N3, nt, a0, bstage, astep, bstep, idesc, first);
                else
                  issue_stage_n(pkc, dt0, p.N3, nt, a0, bstage, astep, bstep, idesc, first);
                tc::mma_commit(&bars->s_empty[s]);
                PROF_ADD(3);
                if (++s == p.nbs) {
                  s = 0;
                  sphase ^= 1u;
                }
              }
            }
            if (failed) break;
            tc::mma_commit(&bars->d_full[gb]);
          }
          if (failed) break;
          tc::mma_commit(&bars->a_empty[a]);
        }
      }
      if (failed) atomicExch(p.err, 1u);
    }
    __syncwarp();
  } else if (warp >= kEpi0) {
    // Epilogue: warp w reads TMEM lane quarter w % 4 (32 positions of the
    // tile) and a quarter of the block's output channels (16, or 8 when the
    // block is 32 wide).
    const int ew = warp - kEpi0;
    const int qd = warp & 3;
    const int cwq = p.CB / 4;
    const int cbeg = (ew >> 2) * cwq;
    float2* tab = bars->tab[ew];  // (scale of digit 2, bias) of this warp's channels
    int tab_cob = -1;
    long long g = 0;
    auto load_tab = [&](int cob) {
      if (cob == tab_cob) return;
      if (lane < 16) {
        const int co = cob * p.CB + cbeg + lane;
        tab[lane] = (lane < cwq && co < p.Co)
                        ? make_float2(__ldg(p.scales + 2 * p.ncob * p.CB + co), p.bias ? __ldg(p.bias + co) : 0.f)
                        : make_float2(0.f, 0.f);
      }
      __syncwarp();
      tab_cob = cob;
    };
    for (int i = 0; i < nu && !failed; ++i) {
      long long u;
      int ts;
      step_of(i, u, ts);
      const long long key = u * TT + ts;
      int cob0, nt;
      long long t0;
      unit_of(u, cob0, t0, nt);
      const XT* xs = x + (size_t)ts * p.C * step_elems;
      XT* ys = static_cast<XT*>(p.y) + (size_t)ts * p.Co * step_elems;
      if constexpr (!STREAM) {
        load_tab(cob0);
        const int nco = min(cwq, p.Co - (cob0 * p.CB + cbeg));  // valid channels of this warp (may be <= 0)
        for (int j = 0; j < nt; ++j, ++g) {
          const int d = (int)(g & 1);
          if (!tc::mbar_wait_sleep(&bars->d_full[d], (uint32_t)((g >> 1) & 1))) {
            failed = true;
            break;
          }
          tc::fence_after();
          const bool odd = *reinterpret_cast<volatile uint32_t*>(&bars->tag[key % kTags]) == (uint32_t)(key + 1);
          epilogue_tile<XT, WT, LM>(p, xs, ys, p.v, tmem, (uint32_t)(d * p.N3), t0 + j, cob0, qd, lane, cbeg, cwq,
                                    nco, tab, odd);
          tc::fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->d_empty[d]);
        }
      } else {
        for (int cob = 0; cob < p.ncob && !failed; ++cob, ++g) {
          load_tab(cob);
          const int nco = min(cwq, p.Co - (cob * p.CB + cbeg));
          const int gb = p.ngb == 2 ? (int)(g & 1) : 0;
          const long long gr = p.ngb == 2 ? (g >> 1) : g;
          auto dcol = [&](int j) { return (uint32_t)((gb * p.U + j) * p.N3); };  // TMEM column of tile j
          // LIF over full 8-channel groups: the membranes of all the group's
          // tiles (at most kLifU) load before the wait for D, so their L2
          // latency hides behind the MMAs.
          const bool lif8 = LM != 0 && p.vs_off != 0 && cwq == 8 && nco == 8 && nt <= kLifU;
          float* slab = reinterpret_cast<float*>(smem + p.vs_off) + ew * (kLifU * 8 * 32) + lane;
          TilePos tp[kLifU];
          if (lif8) {
#pragma unroll
            for (int j = 0; j < kLifU; ++j) {
              if (j < nt) {
                tp[j] = tile_pos(p, t0 + j, cob, qd, lane, cbeg);
                lif_v_stage(p, tp[j], slab + j * 256);
              }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
          }
#ifdef SF_C3TC_PROF
          const long long pw0 = clock64();
#endif
          if (!tc::mbar_wait_sleep(&bars->d_full[gb], (uint32_t)(gr & 1))) {
            failed = true;
            break;
          }
#ifdef SF_C3TC_PROF
          const long long pw1 = clock64();
          if (lane == 0) atomicAdd(&g_c3tc_prof[5], (unsigned long long)(pw1 - pw0));
#endif
          tc::fence_after();
          const bool odd = *reinterpret_cast<volatile uint32_t*>(&bars->tag[key % kTags]) == (uint32_t)(key + 1);
          if (lif8) asm volatile("cp.async.wait_group 0;" ::: "memory");
          if (lif8 && !odd) {
#pragma unroll
            for (int j = 0; j < kLifU; ++j) {
              if (j < nt) {
                lif_tile8<XT, LM>(p, ys, tp[j], tmem + ((uint32_t)(qd * 32) << 16) + dcol(j) + cbeg, slab + j * 256,
                                  tab);
              }
            }
          } else {
            for (int j = 0; j < nt; ++j) {
              epilogue_tile<XT, WT, LM>(p, xs, ys, p.v, tmem, dcol(j), t0 + j, cob, qd, lane, cbeg, cwq, nco, tab,
                                        odd);
            }
          }
#ifdef SF_C3TC_PROF
          if (lane == 0) atomicAdd(&g_c3tc_prof[4], (unsigned long long)(clock64() - pw1));
#endif
          tc::fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->d_empty[gb]);
        }
      }
    }
    if (failed && lane == 0) atomicExch(p.err, 1u);
  } else if (STREAM && warp == kProducer) {
    if (lane == 0) {
      const int nkc = p.kcores / p.kch;
      int s = 0;
      uint32_t round = 0;  // passes over the ring
      for (int i = 0; i < nu && !failed; ++i) {
        for (int cob = 0; cob < p.ncob && !failed; ++cob) {
          for (int tap = 0; tap < 9 && !failed; ++tap) {
            for (int kc = 0; kc < nkc; ++kc) {
              if (round > 0 && !tc::mbar_wait_sleep(&bars->s_empty[s], (round - 1) & 1u)) {
                failed = true;
                break;
              }
              mbar_arrive_expect_tx(&bars->s_full[s], p.bstage_bytes);
              const unsigned char* src =
                  p.bimg + (((size_t)cob * 9 + tap) * p.kcores + (size_t)kc * p.kch) * p.N3 * 16;
              bulk_g2s(bsm + (size_t)s * p.bstage_bytes, src, p.bstage_bytes, &bars->s_full[s]);
              if (++s == p.nbs) {
                s = 0;
                ++round;
              }
            }
          }
        }
      }
      if (failed) atomicExch(p.err, 1u);
    }
    __syncwarp();
  } else {
    for (int i = 0; i < nu && !failed; ++i) {
      long long u;
      int ts;
      step_of(i, u, ts);
      const long long key = u * TT + ts;
      int cob, nt;
      long long t0;
      unit_of(u, cob, t0, nt);
      const XT* xs = x + (size_t)ts * p.C * step_elems;
      const int na = STREAM ? p.nA : 2;
      const int a = i % na;
      if (i >= na && !tc::mbar_wait_sleep(&bars->a_empty[a], (uint32_t)(((i / na) - 1) & 1))) {
        failed = true;
        break;
      }
      unsigned char* ab = abuf + (size_t)a * p.a_bytes;
      uint32_t nb = 0u;
      if constexpr (VEC)
        // Streamed weights keep x out of L1 (C128 28x28 0.5 % faster): their
        // units span many channels, so a unit's halo rows are gone from L1
        // before the next unit reads them. With resident weights the next
        // unit's halo rows still hit in L1: not allocating there cost the
        // C64 56x56 cell 6 %.
        convert_unit_vec4<STREAM>(p, reinterpret_cast<const float*>(xs), ab, t0 * kM, warp, lane, kConv, nb);
      else
        convert_unit_scalar<XT>(p, xs, ab, t0 * kM, warp, lane, kConv, nb);
      if (__any_sync(0xffffffffu, nb != 0u) && lane == 0)
        *reinterpret_cast<volatile uint32_t*>(&bars->tag[key % kTags]) = (uint32_t)(key + 1);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->a_full[a]);
    }
    if (failed && lane == 0) atomicExch(p.err, 1u);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after();
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}

// Per output channel: s = max |w[co]|, stored as the three digit scales.
__global__ void tc_scales_kernel(const void* w, int src_dtype, int Co, int C, int ncob, int CB, float* scales) {
  const int co = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (co >= ncob * CB) return;
  float m = 0.f;
  if (co < Co) {
    for (int i = lane; i < C * 9; i += 32) {
      const size_t idx = (size_t)co * C * 9 + i;
      float v;
      if (src_dtype == SF_DTYPE_F32)
        v = static_cast<const float*>(w)[idx];
      else if (src_dtype == SF_DTYPE_F16)
        v = __half2float(static_cast<const __half*>(w)[idx]);
      else
        v = __bfloat162float(static_cast<const __nv_bfloat16*>(w)[idx]);
      m = fmaxf(m, fabsf(v));
    }
  }
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) {
    const int tot = ncob * CB;
    scales[co] = m * 0x1p-6f;
    scales[tot + co] = m * 0x1p-14f;
    scales[2 * tot + co] = m * 0x1p-22f;
  }
}

// Digit bytes of the B image [cob][tap][kcore][N3][16].
__global__ void tc_digits_kernel(const void* w, int src_dtype, int Co, int C, int ncob, int CB, int kcores,
                                 const float* scales, signed char* bimg) {
  const int N3 = 3 * CB;
  const size_t total = (size_t)ncob * 9 * kcores * N3 * 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(i & 15);
    size_t r = i >> 4;
    const int n = (int)(r % N3);
    r /= N3;
    const int kc = (int)(r % kcores);
    r /= kcores;
    const int tap = (int)(r % 9);
    const int cob = (int)(r / 9);
    const int plane = n / CB;
    const int co = cob * CB + (n - plane * CB);
    const int ci = kc * 16 + b;
    int digit = 0;
    if (co < Co && ci < C) {
      const size_t idx = ((size_t)co * C + ci) * 9 + tap;
      float v;
      if (src_dtype == SF_DTYPE_F32)
        v = static_cast<const float*>(w)[idx];
      else if (src_dtype == SF_DTYPE_F16)
        v = __half2float(static_cast<const __half*>(w)[idx]);
      else
        v = __bfloat162float(static_cast<const __nv_bfloat16*>(w)[idx]);
      const float s = scales[co] * 64.f;  // max |w[co]|, exactly
      if (s > 0.f) {
        const int q = __float2int_rn(__fdiv_rn(v, s) * 4194304.f);  // |q| <= 2^22
        const int d2 = ((q + 128) & 255) - 128;
        const int q1 = (q - d2) >> 8;
        const int d1 = ((q1 + 128) & 255) - 128;
        const int d0 = (q1 - d1) >> 8;
        digit = plane == 0 ? d0 : (plane == 1 ? d1 : d2);
      }
    }
    bimg[i] = (signed char)digit;
  }
}

inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

struct Geo {
  int CB, ncob, N3, kcores;
  size_t scale_bytes, b_bytes;
};
Geo geometry(int Co, int C) {
  Geo g;
  // 64-channel output blocks (N = 192) when the weights stay resident; 32
  // (N = 96) when they stream (C_in > 64), so two tiles' D of two blocks
  // fit TMEM.
  g.CB = (Co <= 32 || C > kTcResidentMaxC) ? 32 : 64;
  g.ncob = (Co + g.CB - 1) / g.CB;
  g.N3 = 3 * g.CB;
  g.kcores = (C + 31) / 32 * 2;
  g.scale_bytes = align256((size_t)3 * g.ncob * g.CB * 4);
  g.b_bytes = (size_t)9 * g.kcores * g.N3 * 16;
  return g;
}

template <typename XT, typename WT, int LM>
sf_status launch_lm(const Params& p, size_t smem, cudaStream_t st) {
  // 16-byte row loads: fp32 rows of a multiple of 4 values, 16-byte aligned x.
  const bool vec = std::is_same<XT, float>::value && p.W % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0;
  const bool stream = p.nbs > 0;
  auto kern = stream ? (vec ? conv3x3_tc_kernel<XT, WT, true, true, LM> : conv3x3_tc_kernel<XT, WT, false, true, LM>)
                     : (vec ? conv3x3_tc_kernel<XT, WT, true, false, LM> : conv3x3_tc_kernel<XT, WT, false, false, LM>);
  if (!allow_max_smem(reinterpret_cast<const void*>(kern))) return SF_ERR_CUDA;
  const long long grid = (p.nunits + p.units_per_cta - 1) / p.units_per_cta;
  kern<<<(unsigned)grid, cta_threads<LM>(), smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

// LM from the parameters: 0 without a membrane, 2 for a power-of-two tau
// (p.inv_tau set), 1 otherwise.
template <typename XT, typename WT>
sf_status launch(const Params& p, size_t smem, cudaStream_t st) {
  if (p.v == nullptr) return launch_lm<XT, WT, 0>(p, smem, st);
  if constexpr (std::is_same<XT, float>::value) {  // fp32 spike buffers only
    if (p.inv_tau != 0.f) return launch_lm<XT, WT, 2>(p, smem, st);
    return launch_lm<XT, WT, 1>(p, smem, st);
  }
  return SF_ERR_UNSUPPORTED;
}

template <typename XT>
sf_status dispatch_w(int wdt, const Params& p, size_t smem, cudaStream_t st) {
  if (wdt == SF_DTYPE_F32) return launch<XT, float>(p, smem, st);
  if (wdt == SF_DTYPE_BF16) return launch<XT, __nv_bfloat16>(p, smem, st);
  return SF_ERR_UNSUPPORTED;
}

}  // namespace

#ifdef SF_C3TC_PROF
extern "C" int sf_dev_c3tc_prof(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, g_c3tc_prof, 8 * sizeof(unsigned long long));
  unsigned long long z[8] = {0};
  return (int)cudaMemcpyToSymbol(g_c3tc_prof, z, sizeof(z));
}
#endif

bool tc3_packs(int Co, int C, int K) { return K == 3 && C >= 1 && C <= kTcMaxC && Co >= 1 && Co <= 4096; }

size_t tc3_section_bytes(int Co, int C) {
  const Geo g = geometry(Co, C);
  return g.scale_bytes + (size_t)g.ncob * g.b_bytes;
}

sf_status tc3_pack(const void* w, int src_dtype, int Co, int C, void* section, cudaStream_t st) {
  const Geo g = geometry(Co, C);
  float* scales = static_cast<float*>(section);
  signed char* bimg = static_cast<signed char*>(section) + g.scale_bytes;
  const int warps = g.ncob * g.CB;
  tc_scales_kernel<<<(warps + 7) / 8, 256, 0, st>>>(w, src_dtype, Co, C, g.ncob, g.CB, scales);
  if (cudaGetLastError() != cudaSuccess) return SF_ERR_CUDA;
  const size_t total = (size_t)g.ncob * g.b_bytes;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
  tc_digits_kernel<<<blocks, 256, 0, st>>>(w, src_dtype, Co, C, g.ncob, g.CB, g.kcores, scales, bimg);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

namespace {
// Launch plan (geometry, unit size, shared-memory layout, TMEM columns);
// false for shapes the kernel does not take.
bool plan_tc(Params& p, size_t& smem_out, int N, int C, int H, int W, int Co, bool lif = false) {
  if (!tc3_packs(Co, C, 3)) return false;
  const Geo g = geometry(Co, C);
  p.N = N; p.C = C; p.H = H; p.W = W; p.Co = Co;
  p.Wp = W + 2;
  p.Hs = H + 1;
  p.fd_wp = make_fastdiv((uint32_t)p.Wp);
  p.fd_hs = make_fastdiv((uint32_t)p.Hs);
  p.kcores = g.kcores;
  p.CB = g.CB;
  p.N3 = g.N3;
  p.ncob = g.ncob;
  const long long positions = (long long)N * p.Hs * p.Wp;
  p.ntiles = (positions + kM - 1) / kM;
  // Positions (and the A rows past the last tile) are decoded in 32 bits.
  if (p.ntiles * kM + 4ll * kM + 2ll * p.Wp >= (1ll << 31)) return false;
  p.b_bytes = (uint32_t)g.b_bytes;
  const size_t limit = 227 * 1024;
  size_t smem = 0;
  int U = 0;
  auto rows_for = [&](int u) { return (uint32_t)((u * kM + 2 * p.Wp + 2 + 31) / 32 * 32); };
  if (C <= kTcResidentMaxC) {
    // Resident weights: [B digits][2 A buffers][barriers]. Units of up to 6
    // tiles (the halo rows a unit converts twice shrink with U) within 200 KB
    // of shared memory: past that the L1 left beside it is too small and the
    // x stream slows (U = 6 at 226 KB measured 24 % slower on the C64 56x56
    // cell than U = 4 at 191 KB). The full 227 KB only when nothing smaller
    // fits.
    for (size_t budget : {(size_t)200 * 1024, limit}) {
      for (int u = 6; u >= 1 && U == 0; --u) {
        const uint32_t rows = rows_for(u);
        const size_t a_bytes = (size_t)rows * 16 * g.kcores;
        const size_t a_off = (g.b_bytes + 127) / 128 * 128;
        const size_t bar_off = a_off + 2 * a_bytes;
        const size_t total = bar_off + sizeof(Bars);
        if (total <= budget) {
          U = u;
          p.rows_a = rows;
          p.a_plane = rows * 16;
          p.a_bytes = (uint32_t)a_bytes;
          p.b_off = 0;
          p.a_off = (uint32_t)a_off;
          p.bar_off = (uint32_t)bar_off;
          p.nA = 2;
          p.nbs = 0;
          smem = total;
        }
      }
      if (U) break;
    }
  } else {
    // Streamed weights: [nA A buffers][nbs weight stages][barriers]. A stage
    // holds kch 16-channel slices of one tap of one 32-channel block. Prefer
    // two tiles per unit (each weight stage feeds both), then double-buffered
    // A, then more stages.
    // Stages of up to 16 slices (24 KB): each stage costs the MMA warp a
    // wait, fences and a commit, which bound these layers at 8 slices
    // (C256 14x14: 0.61 ms with 8-slice stages, 0.45 ms with 16).
    p.kch = std::min(g.kcores, kMaxKch);
    while (g.kcores % p.kch) p.kch -= 2;
    p.bstage_bytes = (uint32_t)(p.kch * g.N3 * 16);
    const int cand[6][2] = {{4, 2}, {4, 1}, {2, 2}, {2, 1}, {1, 2}, {1, 1}};
    // More tiles per unit cut the weight bytes and the per-stage overhead per
    // MMA, which bound these layers, so they win even at the full 227 KB
    // (C512 14x14: 2.9 ms with one tile per unit at 180 KB, 2.2 ms with two).
    // Four tiles of 96 columns leave TMEM room for one group only; that pays
    // on maps of width >= 28 (C128 28x28: 0.547 against 0.588 ms) but not on
    // 14x14 (C256: 0.67 against 0.58 ms).
    for (int ci = (W >= 28 ? 0 : 2); ci < 6 && U == 0; ++ci) {
      for (size_t budget : {(size_t)200 * 1024, limit}) {
        for (int nbs = kMaxBStages; nbs >= 2 && U == 0; --nbs) {
          const int u = cand[ci][0], na = cand[ci][1];
          const uint32_t rows = rows_for(u);
          const size_t a_bytes = (size_t)rows * 16 * g.kcores;
          const size_t b_off = (size_t)na * a_bytes;
          const size_t bar_off = (b_off + (size_t)nbs * p.bstage_bytes + 127) / 128 * 128;
          const size_t total = bar_off + sizeof(Bars);
          if (total <= budget && (nbs >= 4 || budget == limit)) {
            U = u;
            p.rows_a = rows;
            p.a_plane = rows * 16;
            p.a_bytes = (uint32_t)a_bytes;
            p.a_off = 0;
            p.b_off = (uint32_t)b_off;
            p.bar_off = (uint32_t)bar_off;
            p.nA = na;
            p.nbs = nbs;
            smem = total;
          }
        }
        if (U) break;
      }
    }
  }
  if (U == 0) return false;
  // Small problems: fewer tiles per unit until every SM has a unit (C1, 32
  // images of 32x32: 281 tiles, 71 four-tile units for 148 SMs).
  const int sms = num_sms_current_device();
  const int u_max = lif ? std::min(U, kLifU) : U;
  while (U > 1 && (p.ntiles + U - 1) / U * (p.nbs > 0 ? 1 : p.ncob) < sms) {
    --U;
    p.rows_a = rows_for(U);
    p.a_plane = p.rows_a * 16;
  }
  if (lif) {
    // With the LIF epilogue each CTA runs its units T times over one step's
    // plane, which is small (C3: 435 tiles for 148 SMs): fewer tiles per unit
    // where that lowers the most tiles any CTA gets (C3: 3-tile units, 3 per
    // CTA, against 2 x 2 with 2-tile units).
    auto most = [&](int u) {
      const long long units = (p.ntiles + u - 1) / u * (p.nbs > 0 ? 1 : p.ncob);
      const long long ctas = std::min<long long>(units, sms);
      return (units + ctas - 1) / ctas * u;
    };
    int best = u_max;
    for (int u = u_max - 1; u >= 1; --u)
      if (most(u) < most(best)) best = u;
    U = best;
#ifdef SF_DEV_KNOBS
    if (const char* e = getenv("SF_C3TC_LIF_U")) U = std::max(1, std::min(u_max, atoi(e)));
#endif
    p.rows_a = rows_for(U);
    p.a_plane = p.rows_a * 16;
    if (p.nbs > 0) {
      // Streamed weights: [A buffers][membrane slabs][weight stages][barriers],
      // the most weight stages (2..8) that fit, two A buffers if possible.
      const size_t a_bytes = (size_t)p.rows_a * 16 * g.kcores;
      const size_t vs_bytes = (size_t)kEpiWarps * kLifU * 8 * 32 * 4;
      bool ok = false;
      for (int na = 2; na >= 1 && !ok; --na) {
        for (int nbs = kMaxBStages; nbs >= 2 && !ok; --nbs) {
          const size_t vs_off = (size_t)na * a_bytes;
          const size_t b_off = vs_off + vs_bytes;
          const size_t bar_off = (b_off + (size_t)nbs * p.bstage_bytes + 127) / 128 * 128;
          const size_t total = bar_off + sizeof(Bars);
          if (total <= limit) {
            ok = true;
            p.a_bytes = (uint32_t)a_bytes;
            p.nA = na;
            p.nbs = nbs;
            p.vs_off = (uint32_t)vs_off;
            p.b_off = (uint32_t)b_off;
            p.bar_off = (uint32_t)bar_off;
            smem = total;
          }
        }
      }
      if (!ok) p.vs_off = 0;  // direct membrane loads (the general epilogue)
    }
  }
  smem = std::max<size_t>(smem, 120 * 1024);  // one CTA (and one TMEM allocation) per SM
  p.U = U;
  if (p.nbs > 0) {
    p.upcob = (p.ntiles + U - 1) / U;  // units cover every block in turn
    p.nunits = p.upcob;
  } else {
    p.upcob = (p.ntiles + U - 1) / U;
    p.nunits = p.upcob * p.ncob;
  }
  p.fd_upcob = make_fastdiv((uint32_t)p.upcob);
  p.ngb = (p.nbs > 0 && 2 * U * p.N3 > 512) ? 1 : 2;
  uint32_t cols = 32;
  while (cols < (uint32_t)(p.ngb * U * p.N3) && p.nbs > 0) cols <<= 1;
  while (cols < (uint32_t)(2 * p.N3)) cols <<= 1;
  p.tmem_cols = cols;
  if (cols > 512) return false;
  const long long ctas = std::min<long long>(p.nunits, (long long)num_sms_current_device());
  p.units_per_cta = (p.nunits + ctas - 1) / ctas;
  smem_out = smem;
  return true;
}
}  // namespace

bool tc3_supported(int N, int C, int H, int W, int Co) {
  Params p;
  memset(&p, 0, sizeof(p));
  size_t smem = 0;
  return plan_tc(p, smem, N, C, H, W, Co);
}

namespace {
// 1 / tau when tau is a power of two with a normal reciprocal, else 0.
float pow2_reciprocal(float tau) {
  int e = 0;
  const float m = std::frexp(std::fabs(tau), &e);
  if (m != 0.5f || e < -124 || e > 126) return 0.f;
  return 1.f / tau;
}
}  // namespace

sf_status run_conv3x3_tc(const void* x, const void* w_gather, int cpl, const void* section, const float* bias,
                         void* y, uint32_t* err, int N, int C, int H, int W, int Co, int xdt, int wdt,
                         cudaStream_t st, const Gate& gate, const TcLif* lif) {
  if (wdt != SF_DTYPE_F32 && wdt != SF_DTYPE_BF16) return SF_ERR_UNSUPPORTED;
  Params p;
  memset(&p, 0, sizeof(p));
  size_t smem = 0;
  if (lif) {
    if (lif->T < 1 || !lif->v || N % lif->T != 0 || !(lif->tau != 0.f)) return SF_ERR_INVALID_ARG;
    // The plane holds one step's images; units repeat over the T steps.
    if (!plan_tc(p, smem, N / lif->T, C, H, W, Co, true)) return SF_ERR_UNSUPPORTED;
    p.T = lif->T;
    p.v = lif->v;
    p.tau = lif->tau;
    p.inv_tau = pow2_reciprocal(lif->tau);
    p.vth = lif->v_threshold;
    p.hard = lif->hard_reset;
    p.vr = lif->hard_reset ? lif->v_reset : 0.f;
    p.decay_input = lif->decay_input;
    // Streamed weights with staged membranes only. With resident weights
    // (C_in <= 64) the epilogue's membrane traffic outweighs the MMAs of a
    // tile: C64 56x56 took 1.37 ms with direct membrane loads and 0.79 ms
    // with staged ones, against 0.68 ms for the two launches. And one step's
    // plane must give every SM a few tiles: C256 14x14 (120 tiles) took
    // 0.74 ms against 0.55.
    if (p.vs_off == 0) return SF_ERR_UNSUPPORTED;
    if (!lif->always && p.ntiles < 2ll * num_sms_current_device()) return SF_ERR_UNSUPPORTED;
  } else if (!plan_tc(p, smem, N, C, H, W, Co)) {
    return SF_ERR_UNSUPPORTED;
  }
  const Geo g = geometry(Co, C);
  p.x = x;
  p.scales = static_cast<const float*>(section);
  p.bimg = static_cast<const unsigned char*>(section) + g.scale_bytes;
  p.bias = bias;
  p.wg = w_gather;
  p.cpl = cpl;
  p.y = y;
  p.err = err;
  p.gate = gate;
  switch (xdt) {
    case SF_DTYPE_F32: return dispatch_w<float>(wdt, p, smem, st);
    case SF_DTYPE_F16: return dispatch_w<__half>(wdt, p, smem, st);
    case SF_DTYPE_BF16: return dispatch_w<__nv_bfloat16>(wdt, p, smem, st);
  }
  return SF_ERR_INVALID_ARG;
}

}  // namespace c3tc
}  // namespace sf
