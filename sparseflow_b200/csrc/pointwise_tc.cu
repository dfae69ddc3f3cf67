// Sparse 1x1 convolution (stride 1) on the tcgen05 tensor cores.
//
// The reference's default 1x1 path (Kernels/conv2d.py:364-560) dots the
// active channel groups of each tile. With block-clustered spikes (the C2
// config: dense inside active 16x16 blocks) a tile's active channels form a
// real dense contraction, and the cost that matters is streaming x once at
// HBM speed; per-event gathers on CUDA cores spend more instructions per
// output than that allows. Here a 1x1 convolution is a GEMM per image,
//   D[px][co] = sum_ci X[ci][px] * W[co][ci],
// with M = 128 pixels per tile, N = C_out (padded to 32), K = C_in (padded
// to 64), run on tcgen05 with fp32 accumulators in TMEM. Per CTA
// (persistent, a contiguous range of tiles):
//
//   warp 24    TMA producer: 3-D tensor loads of x chunks [64 channels][128
//              pixels] (zero-filled past C and H*W) into a ring of up to 6
//              staging buffers (as many as shared memory holds), on
//              full/empty mbarriers;
//   warps 0-15 convert each staged chunk to bf16 (exact for 0/1 spikes) as
//              the A operand, K-major with the 128-byte swizzle, into a ring
//              of 2 A slots, noting whether the chunk has a nonzero and
//              whether any value is neither 0 nor 1;
//   warps 16-23 read each tile's D from TMEM (tcgen05.ld, lane = pixel), add
//              the bias and store y in coalesced rows;
//   warp 25    allocates TMEM (two accumulators: the epilogue of tile t
//              overlaps the MMAs of tile t+1); one thread issues
//              tcgen05.mma kind::f16 for each nonzero chunk and commits to
//              the mbarriers that free the A slot and hand D over.
//
// Exactness: the B operand is the weights split into bf16 planes
// w = hi + mid + lo (one plane for bf16 weights), and A holds x in bf16; when
// every x of a tile is exactly a bf16 (spikes 0/1 are; so are small integers
// and powers of two) every product is exact and the fp32 accumulation
// matches the fp32 reference to a few ulp. A tile holding any other value is
// computed on the CUDA cores instead (fp32 FMAs in ascending channel order)
// and its D is discarded.
//
// Every mbarrier wait gives up after one second of wall time (the error word
// is set and the CTA drains); TMA loads without multicast; TMEM is released
// before the CTA exits.
#include <cudaTypedefs.h>
#include <cstdlib>
#include <cstring>
#include "conv_kernel.cuh"
#include "policy.cuh"

namespace sf {
namespace pwtc {
namespace {

using conv::mbar_arrive;

constexpr int kConvWarps = 16;                   // warps 0-15: convert x chunks
constexpr int kEpiWarps = 8;                     // warps 16-23: TMEM -> y
constexpr int kProducerWarp = kConvWarps + kEpiWarps;
constexpr int kMmaWarp = kProducerWarp + 1;
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr int kM = 128;       // pixels per tile = MMA M = TMEM lanes
constexpr int kKC = 64;       // channels per chunk (one 128-byte swizzle row of bf16)
constexpr int kMaxStages = 6; // staging ring (as many as shared memory allows)
constexpr int kASlots = 4;    // bf16 A ring (16 KB chunks) when x is streamed
constexpr int kASlotsMasks = 8;  // ... and when A comes from masks (cheap to build: the ring depth
                                 // then decides how many chunk round trips overlap)
constexpr int kMaxD = 4;      // TMEM accumulators (as many as 512 columns hold)

struct TcParams {
  const void* x;
  const void* wp;  // sf_pack_weights layout [block][C][1][32][cpl]
  const float* bias;
  void* y;
  uint32_t* err;
  int N, C, HW, Co;
  int Kpad, Npad, nplanes, nchunks, nstages, nd;
  int cpl;
  int tiles_per_img;
  long long ntiles, tiles_per_cta;
  uint32_t stage_bytes, a_bytes, b_plane_bytes;
  uint32_t tmem_cols;
  // Mask-fed mode: the spikes' nonzero-channel masks ([image][pixel][nw]
  // 64-bit words, as a spike producer writes them) instead of x.
  const unsigned long long* masks;
  int nw;
  int aslots;  // 16 KB A chunks in the ring: kASlots, or up to kASlotsMasks in mask-fed mode
};

__device__ __forceinline__ void tma_load_3d(void* dst_smem, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst_smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of element (row, k) in a K-major, 128-byte-swizzled bf16 tile
// of `rows` rows: K blocks of 64 elements, each [rows][128 B]; within an
// 8-row (1024 B) atom the 16-byte chunk c of row r sits at chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t sw128(int row, int k, int rows) {
  return (uint32_t)((k >> 6) * rows * 128 + row * 128 + ((((k & 63) >> 3) ^ (row & 7)) << 4) + (k & 7) * 2);
}

__device__ __forceinline__ void st_cs(float* p, float v) { __stcs(p, v); }
__device__ __forceinline__ void st_cs(__half* p, __half v) { __stcs(reinterpret_cast<unsigned short*>(p), __half_as_ushort(v)); }
__device__ __forceinline__ void st_cs(__nv_bfloat16* p, __nv_bfloat16 v) {
  __stcs(reinterpret_cast<unsigned short*>(p), __bfloat16_as_ushort(v));
}

// tcgen05 shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 B apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)1u << 16;             // LBO (unused by swizzled K-major): 16 B
  d |= (uint64_t)(1024u >> 4) << 32;   // SBO
  d |= (uint64_t)1u << 46;             // version
  d |= (uint64_t)2u << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D f32, A and B bf16, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Weight (co, ci) from the sf_pack_weights layout.
template <typename WT>
__device__ __forceinline__ float packed_w(const TcParams& p, int co, int ci) {
  const int blk = co / (32 * p.cpl), rem = co - blk * 32 * p.cpl;
  const int j = rem / 32, lane = rem - j * 32;
  const WT* w = static_cast<const WT*>(p.wp) + (((size_t)blk * p.C + ci) * 32 + lane) * p.cpl + j;
  return DT<WT>::to_f(*w);
}

struct Bars {
  uint64_t s_full[kMaxStages], s_empty[kMaxStages];
  uint64_t a_full[kASlotsMasks], a_empty[kASlotsMasks];
  uint64_t d_full[kMaxD], d_empty[kMaxD];
  uint32_t tmem_base;
  uint32_t a_nz[kASlotsMasks][kConvWarps];  // per converter warp: its part of the chunk has a nonzero
  uint32_t odd[kMaxD];                  // = i + 1 when tile i (in D[b]) holds a value that is not exactly a bf16
  float bias_s[256];                    // bias (0 without one), read by the epilogue as a broadcast
};

// SUB: MMA sub-tiles of 128 pixels per tile. Two make each TMA row 1 KB
// (256 pixels) instead of 512 B.
// MASKS: A comes from the masks (bit c of a pixel's word = channel c is a
// spike, i.e. exactly 1.0): a stage holds one tile's words for all channels
// (kTile pixels x nw x 8 bytes, one bulk copy) and serves every chunk.
template <typename XT, typename WT, int SUB, bool MASKS>
__global__ void __launch_bounds__(kThreads, 1)
    pointwise_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap xmap) {
  constexpr int kTile = kM * SUB;          // pixels per tile
  const int kSlots = p.aslots / SUB;  // A ring (each slot SUB x 16 KB); a power of two
  const int kSlotShift = __ffs(kSlots) - 1;
  constexpr uint32_t kSubA = kM * kKC * 2; // bytes of one sub-tile's A chunk
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* stage = smem;                                   // nstages x [64][128] of XT
  unsigned char* abuf = stage + p.nstages * p.stage_bytes;       // kASlots x A chunk (16 KB)
  unsigned char* bbuf = abuf + kSlots * p.a_bytes;               // nplanes x [Npad][Kpad] bf16
  Bars* bars = reinterpret_cast<Bars*>(bbuf + (size_t)p.nplanes * p.b_plane_bytes);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long t0 = (long long)blockIdx.x * p.tiles_per_cta;
  const long long t1 = min(p.ntiles, t0 + p.tiles_per_cta);
  const int nt = (int)max(0ll, t1 - t0);
  const int KC = p.nchunks;
  const XT* __restrict__ x = static_cast<const XT*>(p.x);

  if (tid == 0) {
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_empty[s], kConvWarps);
    }
    for (int a = 0; a < kSlots; ++a) {
      mbar_init(&bars->a_full[a], kConvWarps);
      mbar_init(&bars->a_empty[a], 1);
    }
    for (int b = 0; b < p.nd; ++b) {
      mbar_init(&bars->d_full[b], 1);
      mbar_init(&bars->d_empty[b], kEpiWarps);
      bars->odd[b] = 0u;
    }
    fence_mbar_init();
  }
  for (int co = tid; co < 256; co += kThreads) bars->bias_s[co] = (p.bias != nullptr && co < p.Co) ? p.bias[co] : 0.f;
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars->tmem_base)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // B operand: weight planes, [Npad rows = co][Kpad = ci], swizzled K-major.
  for (int i = tid; i < p.Npad * (p.Kpad / 8); i += kThreads) {
    const int co = i / (p.Kpad / 8);
    const int k0 = (i - co * (p.Kpad / 8)) * 8;
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = (co < p.Co && k0 + e < p.C) ? packed_w<WT>(p, co, k0 + e) : 0.f;
    for (int pl = 0; pl < p.nplanes; ++pl) {
      float h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        h[e] = __bfloat162float(__float2bfloat16_rn(r[e]));
        r[e] -= h[e];  // exact: the next plane holds what bf16 dropped
      }
      uint4 q;
      q.x = pack_bf16x2(h[0], h[1]);
      q.y = pack_bf16x2(h[2], h[3]);
      q.z = pack_bf16x2(h[4], h[5]);
      q.w = pack_bf16x2(h[6], h[7]);
      *reinterpret_cast<uint4*>(bbuf + (size_t)pl * p.b_plane_bytes + sw128(co, k0, p.Npad)) = q;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool failed = false;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      int s = 0;
      uint32_t round = 0;  // passes over the ring (ring position advanced incrementally: no division)
      for (int i = 0; i < nt && !failed; ++i) {
        const long long tile = t0 + i;
        const int img = (int)(tile / p.tiles_per_img);
        const int px0 = (int)(tile - (long long)img * p.tiles_per_img) * kTile;
        if constexpr (MASKS) {
          // One stage per tile: its pixels' words for all channels (a
          // multiple of 16 bytes: H*W even, checked on the host).
          if (round > 0 && !mbar_wait_ns(&bars->s_empty[s], (round - 1) & 1u)) {
            failed = true;
            break;
          }
          const int npx = min(kTile, p.HW - px0);
          const uint32_t bytes = (uint32_t)npx * p.nw * 8u;
          mbar_arrive_expect_tx(&bars->s_full[s], bytes);
          bulk_g2s(stage + (size_t)s * p.stage_bytes, p.masks + ((size_t)img * p.HW + px0) * p.nw, bytes,
                   &bars->s_full[s]);
          if (++s == p.nstages) {
            s = 0;
            ++round;
          }
        } else {
          for (int kc = 0; kc < KC; ++kc) {
            if (round > 0 && !mbar_wait_ns(&bars->s_empty[s], (round - 1) & 1u)) {
              failed = true;
              break;
            }
            mbar_arrive_expect_tx(&bars->s_full[s], p.stage_bytes);
            tma_load_3d(stage + (size_t)s * p.stage_bytes, &xmap, px0, kc * kKC, img, &bars->s_full[s]);
            if (++s == p.nstages) {
              s = 0;
              ++round;
            }
          }
        }
      }
      if (failed) atomicExch(p.err, 1u);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kM, p.Npad);
      const uint32_t bsa = smem_u32(bbuf);
      for (int i = 0; i < nt && !failed; ++i) {
        const int b = i % p.nd;
        if (i >= p.nd && !mbar_wait_ns(&bars->d_empty[b], (uint32_t)(((i / p.nd) - 1) & 1))) {
          failed = true;
          break;
        }
        const uint32_t d = tmem + (uint32_t)(b * SUB * p.Npad);
        uint32_t acc = 0u;
        for (int kc = 0; kc < KC; ++kc) {
          const int g = i * KC + kc, a = g & (kSlots - 1);
          if (!mbar_wait_ns(&bars->a_full[a], (uint32_t)((g >> kSlotShift) & 1))) {
            failed = true;
            break;
          }
          tc_fence_after();
          uint32_t nz = 0u;
#pragma unroll
          for (int w = 0; w < kConvWarps; ++w) nz |= bars->a_nz[a][w];
          // Skip all-zero chunks; the last chunk always runs if nothing ran, to clear D.
          if (nz != 0u || (kc == KC - 1 && acc == 0u)) {
            const uint32_t asa = smem_u32(abuf + (size_t)a * p.a_bytes);
#pragma unroll
            for (int k16 = 0; k16 < kKC / 16; ++k16) {
              for (int pl = 0; pl < p.nplanes; ++pl) {
                const uint64_t bd = sdesc(bsa + (uint32_t)(pl * p.b_plane_bytes + kc * p.Npad * 128 + k16 * 32));
#pragma unroll
                for (int sb = 0; sb < SUB; ++sb)
                  mma_bf16(d + (uint32_t)(sb * p.Npad), sdesc(asa + sb * kSubA + (uint32_t)(k16 * 32)), bd, idesc,
                           acc);
                acc = 1u;
              }
            }
          }
          mma_commit(&bars->a_empty[a]);  // A slot a has been read
        }
        if (failed) break;
        mma_commit(&bars->d_full[b]);  // D[b] holds the tile
      }
      if (failed) atomicExch(p.err, 1u);
    }
    __syncwarp();
  } else if (warp >= kConvWarps) {
    // Epilogue warps 16-23: warp w reads TMEM lane quarter w % 4 (its pixels)
    // and one half of the columns (output channels).
    auto epilogue = [&](int i) {
      const int b = i % p.nd;
      const long long tile = t0 + i;
      const int img = (int)(tile / p.tiles_per_img);
      const int px0 = (int)(tile - (long long)img * p.tiles_per_img) * kTile;
      if (!mbar_wait_ns(&bars->d_full[b], (uint32_t)((i / p.nd) & 1))) {
        failed = true;
        return;
      }
      tc_fence_after();
      const bool odd = bars->odd[b] == (uint32_t)(i + 1);
      const int ew = warp - kConvWarps;
      const int quarter = warp & 3;  // TMEM lane quarter this warp may read
      const int half = ew >> 2;      // column half
      const int ncol = p.Npad / 2;
      XT* yimg = static_cast<XT*>(p.y) + (size_t)img * p.Co * p.HW;
#pragma unroll
      for (int sb = 0; sb < SUB; ++sb) {
      const int px = px0 + sb * kM + quarter * 32 + lane;
      if (!odd) {
        for (int c0 = half * ncol; c0 < (half + 1) * ncol; c0 += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((b * SUB + sb) * p.Npad + c0), v);
          if (px < p.HW) {
            // Row pointer advanced by adds; evict-first stores (y is not read again here).
            XT* yq = yimg + (size_t)c0 * p.HW + px;
            if (c0 + 16 <= p.Co) {
#pragma unroll
              for (int e = 0; e < 16; ++e, yq += p.HW) st_cs(yq, DT<XT>::from_f(v[e] + bars->bias_s[c0 + e]));
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e, yq += p.HW)
                if (c0 + e < p.Co) st_cs(yq, DT<XT>::from_f(v[e] + bars->bias_s[c0 + e]));
            }
          }
        }
      } else if (px < p.HW) {
        // Exact CUDA-core path: ascending-channel fp32 FMAs, as the gather kernels do.
        const XT* ximg = x + (size_t)img * p.C * p.HW + px;
        for (int co = half * ncol; co < min(p.Co, (half + 1) * ncol); ++co) {
          float acc = 0.f;
          for (int ci = 0; ci < p.C; ++ci) {
            const float xv = DT<XT>::to_f(ximg[(size_t)ci * p.HW]);
            if (xv != 0.f) acc = fmaf(xv, packed_w<WT>(p, co, ci), acc);
          }
          yimg[(size_t)co * p.HW + px] = DT<XT>::from_f(acc + (p.bias ? __ldg(p.bias + co) : 0.f));
        }
      }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->d_empty[b]);
    };
    for (int i = 0; i < nt && !failed; ++i) epilogue(i);
    if (failed && lane == 0) atomicExch(p.err, 1u);
  } else {
    // Converter warps 0-15: warp w converts channel octet w % 8 for pixel
    // half w / 8.
    const int o = warp & 7, phalf = warp >> 3;
    int s = 0;
    uint32_t sround = 0;  // staging ring position, advanced incrementally
    for (int i = 0; i < nt; ++i) {
      const int b = i % p.nd;
      const long long tile = t0 + i;
      const int tile_px0 = (int)(tile - (tile / p.tiles_per_img) * p.tiles_per_img) * kTile;
      for (int kc = 0; kc < KC && !failed; ++kc) {
        const int g = i * KC + kc, a = g & (kSlots - 1);
        if (!mbar_wait_ns(&bars->s_full[s], sround & 1u)) {
          failed = true;
          break;
        }
        if (g >= kSlots && !mbar_wait_ns(&bars->a_empty[a], (uint32_t)(((g >> kSlotShift) - 1) & 1))) {
          failed = true;
          break;
        }
        if constexpr (MASKS) {
          // Lane l takes pixels phalf*(kTile/2) + k*32 + l; warp octet o
          // expands channels kc*64 + o*8 .. +7 of each: bit set -> bf16 1.0.
          const unsigned long long* st = reinterpret_cast<const unsigned long long*>(stage + (size_t)s * p.stage_bytes);
          unsigned char* ab = abuf + (size_t)a * p.a_bytes;
          uint32_t orall = 0u;
          constexpr int kPP = kTile / 64;
#pragma unroll
          for (int k = 0; k < kPP; ++k) {
            const int px = phalf * (kTile / 2) + k * 32 + lane;
            const bool in = tile_px0 + px < p.HW;
            const uint32_t byte = in ? (uint32_t)(st[(size_t)px * p.nw + kc] >> (o * 8)) & 0xffu : 0u;
            orall |= byte;
            uint4 qv;
            uint32_t* qq = &qv.x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t b2 = (byte >> (2 * e)) & 3u;  // channels 2e, 2e+1 -> low, high bf16
              qq[e] = (b2 & 1u) * 0x3f80u + (b2 >> 1) * 0x3f800000u;
            }
            *reinterpret_cast<uint4*>(ab + (px >> 7) * kSubA + sw128(px & (kM - 1), o * 8, kM)) = qv;
          }
          if (kc == KC - 1) {
            // The stage served every chunk of this tile.
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->s_empty[s]);
            if (++s == p.nstages) {
              s = 0;
              ++sround;
            }
          }
          const uint32_t nz = __any_sync(0xffffffffu, orall != 0u);
          if (lane == 0) bars->a_nz[a][warp] = nz;
        } else {
          const XT* st = reinterpret_cast<const XT*>(stage + (size_t)s * p.stage_bytes);  // [64][128]
          unsigned char* ab = abuf + (size_t)a * p.a_bytes;
          uint32_t nz = 0u, odd = 0u;
          // Lane l takes pixels phalf*64 + l and + 32: conflict-free 4-byte reads,
          // and each warp-wide 16-byte store covers all eight swizzle positions.
          // The stage is released as soon as its values are in registers.
          constexpr int kPP = kTile / 64;  // pixels per lane
          float v[kPP][8];
  #pragma unroll
          for (int k = 0; k < kPP; ++k)
  #pragma unroll
            for (int e = 0; e < 8; ++e)
              v[k][e] = DT<XT>::to_f(st[(o * 8 + e) * kTile + phalf * (kTile / 2) + k * 32 + lane]);
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->s_empty[s]);
          if (++s == p.nstages) {
            s = 0;
            ++sround;
          }
          // The MMA is exact whenever every x is exactly a bf16 (then each
          // product with a bf16 weight plane is exact in fp32): for the fp32
          // bits u that means u & 0xffff == 0, tested on the OR of all values,
          // which also gives "any nonzero". Such values convert by taking the
          // high halves (a byte permute).
          uint32_t orall = 0u;
  #pragma unroll
          for (int k = 0; k < kPP; ++k) {
            uint4 qv;
            uint32_t* qq = &qv.x;
  #pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const uint32_t u0 = __float_as_uint(v[k][e]), u1 = __float_as_uint(v[k][e + 1]);
              orall |= u0 | u1;
              qq[e / 2] = __byte_perm(u0, u1, 0x7632);
            }
            const int px = phalf * (kTile / 2) + k * 32 + lane;  // pixel in the tile -> sub-tile, row
            *reinterpret_cast<uint4*>(ab + (px >> 7) * kSubA + sw128(px & (kM - 1), o * 8, kM)) = qv;
          }
          nz = __any_sync(0xffffffffu, (orall & 0x7fffffffu) != 0u);
          odd = __any_sync(0xffffffffu, (orall & 0xffffu) != 0u);
          if (lane == 0) {
            bars->a_nz[a][warp] = nz;
            if (odd) bars->odd[b] = (uint32_t)(i + 1);  // tagged with the tile: no clearing needed
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->a_full[a]);
      }
    }
    if (failed && lane == 0) atomicExch(p.err, 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

template <typename XT, typename WT>
sf_status launch(TcParams p, const CUtensorMap& xmap, size_t smem, int sub, cudaStream_t st) {
  auto kern = p.masks ? (sub == 2 ? pointwise_tc_kernel<XT, WT, 2, true> : pointwise_tc_kernel<XT, WT, 1, true>)
                      : (sub == 2 ? pointwise_tc_kernel<XT, WT, 2, false> : pointwise_tc_kernel<XT, WT, 1, false>);
  if (!allow_max_smem(reinterpret_cast<const void*>(kern))) return SF_ERR_CUDA;
  const long long ctas = std::min<long long>(p.ntiles, (long long)num_sms_current_device());
  p.tiles_per_cta = (p.ntiles + ctas - 1) / ctas;
  const long long grid = (p.ntiles + p.tiles_per_cta - 1) / p.tiles_per_cta;
  kern<<<(unsigned)grid, kThreads, smem, st>>>(p, xmap);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <typename XT>
sf_status dispatch_w(int wdt, const TcParams& p, const CUtensorMap& xmap, size_t smem, int sub, cudaStream_t st) {
  if (wdt == SF_DTYPE_F32) return launch<XT, float>(p, xmap, smem, sub, st);
  if (wdt == SF_DTYPE_BF16) return launch<XT, __nv_bfloat16>(p, xmap, smem, sub, st);
  return SF_ERR_UNSUPPORTED;
}

}  // namespace

// Returns SF_ERR_UNSUPPORTED for shapes it does not take (the caller then
// runs the two-stage path): C_out > 256, C_in > 512, images smaller than one
// 128-pixel MMA tile (SF_POLICY_CONV1X1_TC_MIN_HW, default 128: on 8x8 maps half of
// every tile would be padding and the gather kernels measured faster), H*W
// rows that TMA cannot address (H*W*element size not a multiple of 16, x not
// 16-byte aligned), or operands beyond shared memory.
// masks != nullptr: A comes from the spikes' event masks (x is not read;
// H*W must be even so every tile's words are a 16-byte multiple).
sf_status run_pointwise_tc(const void* x, const void* w_packed, const float* bias, void* y, uint32_t* err, int N,
                           int C, int H, int W, int Co, int xdt, int wdt, cudaStream_t st,
                           const unsigned long long* masks) {
  if (Co > 256 || Co <= 0 || C <= 0 || C > 512) return SF_ERR_UNSUPPORTED;
  const int esz = (int)dtype_size(xdt);
  const long long HW = (long long)H * W;
  if (HW < policy(SF_POLICY_CONV1X1_TC_MIN_HW)) return SF_ERR_UNSUPPORTED;
  if (masks) {
    if (HW % 2 != 0 || (reinterpret_cast<uintptr_t>(masks) & 15u) != 0) return SF_ERR_UNSUPPORTED;
  } else if ((HW * esz) % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0) {
    return SF_ERR_UNSUPPORTED;
  }
  auto enc = encoder();
  if (!enc && !masks) return SF_ERR_UNSUPPORTED;
  TcParams p;
  memset(&p, 0, sizeof(p));
  p.masks = masks;
  p.nw = (C + 63) / 64;
  p.x = x;
  p.wp = w_packed;
  p.bias = bias;
  p.y = y;
  p.err = err;
  p.N = N;
  p.C = C;
  p.HW = (int)HW;
  p.Co = Co;
  p.Kpad = (C + kKC - 1) / kKC * kKC;
  p.nchunks = p.Kpad / kKC;
  p.Npad = std::max(32, (Co + 31) / 32 * 32);  // two epilogue column halves of multiples of 16
  p.nplanes = wdt == SF_DTYPE_F32 ? 3 : 1;
  p.cpl = conv::weight_block_cpl(C, 1, Co, (int)dtype_size(wdt));
  p.b_plane_bytes = (uint32_t)(p.Npad * p.Kpad * 2);
  // Two 128-pixel sub-tiles per tile when shared memory and TMEM allow (1 KB
  // TMA rows), else one.
  auto plan = [&](int sub, size_t* smem_out) {
    const int nd = std::min(kMaxD, 512 / (sub * p.Npad));
    if (nd < 2) return false;
    const size_t stage = masks ? (size_t)kM * sub * p.nw * 8 : (size_t)kKC * kM * sub * esz;
    size_t fixed = 0;
    for (int aslots = masks ? kASlotsMasks : kASlots; aslots >= kASlots; aslots /= 2) {
      fixed = 1024 + (size_t)aslots * kM * kKC * 2 + (size_t)p.nplanes * p.b_plane_bytes + sizeof(Bars);
      p.aslots = aslots;
      if (fixed + 2 * stage <= 232448) break;
    }
    if (fixed + 2 * stage > 232448) return false;
    p.nd = nd;
    p.nstages = (int)std::min<size_t>(kMaxStages, (232448 - fixed) / stage);
    p.stage_bytes = (uint32_t)stage;
    p.a_bytes = (uint32_t)(kM * kKC * 2 * sub);
    *smem_out = fixed + (size_t)p.nstages * stage;
    uint32_t cols = 32;
    while (cols < (uint32_t)(nd * sub * p.Npad)) cols <<= 1;
    p.tmem_cols = cols;
    p.tiles_per_img = (int)((HW + kM * sub - 1) / (kM * sub));
    p.ntiles = (long long)N * p.tiles_per_img;
    return true;
  };
  size_t smem = 0;
  int sub = HW > kM ? 2 : 1;  // an image of <= 128 pixels would leave a 256-pixel tile mostly empty
  if (sub == 1 || !plan(2, &smem)) {
    sub = 1;
    if (!plan(1, &smem)) return SF_ERR_UNSUPPORTED;
  }
  p.tiles_per_cta = 0;

  // x as a 3-D tensor (pixels, channels, images); box = one chunk.
  CUtensorMap xmap;
  memset(&xmap, 0, sizeof(xmap));
  if (masks) {
    switch (xdt) {
      case SF_DTYPE_F32: return dispatch_w<float>(wdt, p, xmap, smem, sub, st);
      case SF_DTYPE_F16: return dispatch_w<__half>(wdt, p, xmap, smem, sub, st);
      case SF_DTYPE_BF16: return dispatch_w<__nv_bfloat16>(wdt, p, xmap, smem, sub, st);
    }
    return SF_ERR_INVALID_ARG;
  }
  const CUtensorMapDataType dt = xdt == SF_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : xdt == SF_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[3] = {(cuuint64_t)HW, (cuuint64_t)C, (cuuint64_t)N};
  const cuuint64_t strides[2] = {(cuuint64_t)(HW * esz), (cuuint64_t)(HW * esz * C)};
  const cuuint32_t box[3] = {(cuuint32_t)(kM * sub), (cuuint32_t)kKC, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  if (enc(&xmap, dt, 3, const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return SF_ERR_UNSUPPORTED;
  switch (xdt) {
    case SF_DTYPE_F32: return dispatch_w<float>(wdt, p, xmap, smem, sub, st);
    case SF_DTYPE_F16: return dispatch_w<__half>(wdt, p, xmap, smem, sub, st);
    case SF_DTYPE_BF16: return dispatch_w<__nv_bfloat16>(wdt, p, xmap, smem, sub, st);
  }
  return SF_ERR_INVALID_ARG;
}

}  // namespace pwtc
}  // namespace sf
