// Stage 1: receptive-field prescan (HBM-bound).
//
// Semantics follow Kernels/_prescan_common.py:32-189 of the reference:
//   group_max[n,ih,iw,g] = amax_{c in g} |half(x)|             (:32-45)
//   rf_max   = max_pool2d(group_max, k, s, p)                   (:169-177)
//   tile_max = max_pool2d(rf_max, (BH,BW), ceil_mode=True)      (:182-187)
//   active   = tile_max > half(threshold)   (compared in half)  (:188)
//   ag_mask  = sum_g active_g << g ; class ZERO/SPARSE/DENSEISH (:48-109)
// and Kernels/conv2d.py:113-123 (ids of non-ZERO tiles, ascending).
//
// B200 design, NCHW input with the full workspace (three launches, no
// inter-CTA waits):
//   group_bits_kernel   streams x once (eight 16-byte loads in flight per
//                       thread) and writes per pixel {active groups, NaN
//                       groups}: 8 bytes per pixel, 3 % of fp32 x for C=64;
//   pool_tiles_kernel   per (image, run of tile rows): ORs every tile's
//                       receptive-field window of those words (a NaN anywhere
//                       in the window clears the group, as the reference's
//                       max-pool of a NaN compares false);
//   compact_ids_kernel  writes active ids in ascending order from per-row
//                       counts, each block summing the counts before it.
// NHWC input, or a workspace of only the look-back words (the static-workspace
// entry point), uses one kernel: a CTA per (image, tile row) folds channels
// for its receptive-field rows into shared memory, pools its tiles and
// compacts ids with a decoupled look-back over CTAs that take logical indices
// from a ticket counter.
#include <cmath>
#include <algorithm>
#include <cstring>
#include "common.cuh"

namespace sf {
namespace {

struct PrescanWs {
  uint32_t ticket;
  uint32_t done;
  uint32_t epoch;
  uint32_t error;
  // uint64_t status[nblocks] follows
};

struct PrescanParams {
  const void* x;
  int32_t* ag_mask;
  int32_t* tile_class;
  int32_t* active_ids;
  int32_t* active_count;
  PrescanWs* ws;
  uint64_t* status;
  int N, C, H, W, Ho, Wo, K, S, P, BH, BW, gs, G, GH, GW;
  uint32_t group_full;  // (1<<G)-1
  float thr;            // half(threshold) as float
  int max_rows_in;
  const uint2* bits;    // two-pass path: per-pixel {active groups, NaN groups}, else nullptr
  int32_t* row_count;   // two-pass path: non-ZERO tiles per tile row (for the compaction kernel)
};

template <typename T>
__device__ __forceinline__ void act_bits(T v, float thr, bool& act, bool& nan) {
  __half h = __float2half_rn(DT<T>::to_f(v));
  nan = __hisnan(h);
  act = !nan && (fabsf(__half2float(h)) > thr);
}
template <>
__device__ __forceinline__ void act_bits<__half>(__half v, float thr, bool& act, bool& nan) {
  nan = __hisnan(v);
  act = !nan && (fabsf(__half2float(v)) > thr);
}

template <int VEC, typename T>
struct alignas(sizeof(T) * VEC) Vec {
  T v[VEC];
};

// Phase A for NCHW input: fold channels into per-pixel group bits.
template <typename T, int VEC>
__device__ void fold_nchw(const PrescanParams& p, int n, int ih_lo, int rows_in, uint32_t* act,
                          uint32_t* nanm) {
  const T* x = static_cast<const T*>(p.x);
  const int nvec_row = p.W / VEC;
  const int per_group = rows_in * nvec_row;
  const int items = p.G * per_group;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int g = it / per_group;
    const int rv = it - g * per_group;
    const int row = rv / nvec_row;
    const int v = rv - row * nvec_row;
    const int c0 = g * p.gs;
    const int c1 = min(p.C, c0 + p.gs);
    const size_t plane = (size_t)p.H * p.W;
    const T* src = x + ((size_t)n * p.C + c0) * plane + (size_t)(ih_lo + row) * p.W + (size_t)v * VEC;
    uint32_t a_bits = 0, n_bits = 0;  // per element of the vector
    int c = c0;
#pragma unroll 1
    for (; c + 4 <= c1; c += 4) {
      Vec<VEC, T> r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) r[u] = *reinterpret_cast<const Vec<VEC, T>*>(src + (size_t)(c - c0 + u) * plane);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          bool a, nn;
          act_bits<T>(r[u].v[e], p.thr, a, nn);
          a_bits |= (uint32_t)a << e;
          n_bits |= (uint32_t)nn << e;
        }
    }
    for (; c < c1; ++c) {
      Vec<VEC, T> r = *reinterpret_cast<const Vec<VEC, T>*>(src + (size_t)(c - c0) * plane);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        bool a, nn;
        act_bits<T>(r.v[e], p.thr, a, nn);
        a_bits |= (uint32_t)a << e;
        n_bits |= (uint32_t)nn << e;
      }
    }
    if (a_bits | n_bits) {
      const int pix0 = row * p.W + v * VEC;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        if (a_bits & (1u << e)) atomicOr(&act[pix0 + e], 1u << g);
        if (n_bits & (1u << e)) atomicOr(&nanm[pix0 + e], 1u << g);
      }
    }
  }
}

// Phase A for NHWC input: each item is one vector of channels at one pixel.
template <typename T, int VEC>
__device__ void fold_nhwc(const PrescanParams& p, int n, int ih_lo, int rows_in, uint32_t* act,
                          uint32_t* nanm) {
  const T* x = static_cast<const T*>(p.x);
  const int nvec_pix = p.C / VEC;
  const int items = rows_in * p.W * nvec_pix;
  const T* base = x + (((size_t)n * p.H + ih_lo) * p.W) * p.C;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int pix = it / nvec_pix;
    const int v = it - pix * nvec_pix;
    Vec<VEC, T> r = *reinterpret_cast<const Vec<VEC, T>*>(base + (size_t)it * VEC);
    uint32_t a_m = 0, n_m = 0;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      bool a, nn;
      act_bits<T>(r.v[e], p.thr, a, nn);
      const uint32_t bit = 1u << ((v * VEC + e) / p.gs);
      a_m |= a ? bit : 0u;
      n_m |= nn ? bit : 0u;
    }
    if (a_m) atomicOr(&act[pix], a_m);
    if (n_m) atomicOr(&nanm[pix], n_m);
  }
}

// Two-pass path, pass 1 (NCHW): one streaming read of x. Each thread owns
// VEC consecutive pixels of one image and walks all channels with eight
// 16-byte loads in flight, writing per pixel {bit g: some channel of group g
// is active, bit g: some channel of group g is NaN}. `cut` is the least float
// f with |half(f)| > half(threshold), so `|v| >= cut` is the reference's
// half-precision comparison (NaN compares false) without a conversion.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) group_bits_kernel(const T* __restrict__ x, int C, int HW, int gs, float cut,
                                                         uint2* __restrict__ bits) {
  const int img = blockIdx.y;
  const int pix0 = (blockIdx.x * 256 + threadIdx.x) * VEC;
  if (pix0 >= HW) return;
  uint32_t a[VEC], nn[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) a[e] = nn[e] = 0u;
  const T* src = x + (size_t)img * C * HW + pix0;
  // Group bit of channel c, advanced with a counter (no division per channel).
  uint32_t bit = 1u;
  int in_group = 0;
  int c = 0;
#pragma unroll 1
  for (; c + 8 <= C; c += 8) {
    Vec<VEC, T> r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) r[u] = *reinterpret_cast<const Vec<VEC, T>*>(src + (size_t)(c + u) * HW);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float v = DT<T>::to_f(r[u].v[e]);
        a[e] |= fabsf(v) >= cut ? bit : 0u;
        nn[e] |= v != v ? bit : 0u;
      }
      if (++in_group == gs) {
        in_group = 0;
        bit <<= 1;
      }
    }
  }
  for (; c < C; ++c) {
    const Vec<VEC, T> r = *reinterpret_cast<const Vec<VEC, T>*>(src + (size_t)c * HW);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float v = DT<T>::to_f(r.v[e]);
      a[e] |= fabsf(v) >= cut ? bit : 0u;
      nn[e] |= v != v ? bit : 0u;
    }
    if (++in_group == gs) {
      in_group = 0;
      bit <<= 1;
    }
  }
  uint2* dst = bits + (size_t)img * HW + pix0;
#pragma unroll
  for (int e = 0; e < VEC; ++e) dst[e] = make_uint2(a[e], nn[e]);
}

template <typename T, int VEC, bool NHWC>
__global__ void __launch_bounds__(256) prescan2d_kernel(PrescanParams p) {
  extern __shared__ __align__(16) uint32_t smem[];
  __shared__ uint32_t s_block, s_epoch;
  __shared__ int32_t s_excl;
  __shared__ int32_t s_cls[256];

  const int tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&p.ws->epoch);
    s_block = atomicAdd(&p.ws->ticket, 1u);
  }
  __syncthreads();
  const int b = (int)s_block;
  const uint32_t epoch = s_epoch;
  const int n = b / p.GH;
  const int gh = b - n * p.GH;

  const int oh0 = gh * p.BH;
  const int oh1 = min(oh0 + p.BH, p.Ho);
  const int ih_lo = max(0, oh0 * p.S - p.P);
  const int ih_hi = min(p.H, (oh1 - 1) * p.S - p.P + p.K);
  const int rows_in = ih_hi - ih_lo;

  uint32_t* act = smem;
  uint32_t* nanm = smem + p.max_rows_in * p.W;
  for (int i = tid; i < rows_in * p.W; i += blockDim.x) {
    act[i] = 0u;
    nanm[i] = 0u;
  }
  __syncthreads();
  if (rows_in > 0) {
    if (NHWC)
      fold_nhwc<T, VEC>(p, n, ih_lo, rows_in, act, nanm);
    else
      fold_nchw<T, VEC>(p, n, ih_lo, rows_in, act, nanm);
  }
  __syncthreads();

  // Phase B: one warp per tile of this tile row.
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const size_t tile_base = ((size_t)n * p.GH + gh) * p.GW;
  for (int gw = warp; gw < p.GW; gw += nwarps) {
    const int ow0 = gw * p.BW;
    const int ow1 = min(ow0 + p.BW, p.Wo);
    const int iw_lo = max(0, ow0 * p.S - p.P);
    const int iw_hi = min(p.W, (ow1 - 1) * p.S - p.P + p.K);
    const int rw = iw_hi - iw_lo;
    uint32_t a = 0, nn = 0;
    for (int i = lane; i < rows_in * rw; i += 32) {
      const int r = i / rw;
      const int cidx = r * p.W + iw_lo + (i - r * rw);
      a |= act[cidx];
      nn |= nanm[cidx];
    }
    a = __reduce_or_sync(0xffffffffu, a);
    nn = __reduce_or_sync(0xffffffffu, nn);
    if (lane == 0) {
      const uint32_t m = a & ~nn & p.group_full;
      const int cls = (m == 0u) ? SF_TILE_ZERO : ((m == p.group_full) ? SF_TILE_DENSEISH : SF_TILE_SPARSE);
      p.ag_mask[tile_base + gw] = (int32_t)m;
      p.tile_class[tile_base + gw] = cls;
      if (gw < 256) s_cls[gw] = cls;
    }
  }

  if (p.active_ids != nullptr) {
    __syncthreads();
    if (warp == 0) {
      // Local count (GW <= 256 is checked on the host).
      int local = 0;
      for (int base = 0; base < p.GW; base += 32) {
        const int gw = base + lane;
        const bool f = gw < p.GW && s_cls[gw] != SF_TILE_ZERO;
        local += __popc(__ballot_sync(0xffffffffu, f));
      }
      // Decoupled look-back over logical blocks, 32 predecessors per step:
      // lane l inspects block j - l. Status words are {tag | flag << 32 |
      // count}, flag 1 = this block's own count, 2 = inclusive prefix.
      const uint64_t tag = (uint64_t)((epoch + 1u) & 0x3fffffffu) << 34;
      if (lane == 0)
        st_release_u64(&p.status[b], tag | ((b == 0 ? 2ull : 1ull) << 32) | (uint32_t)local);
      int excl = 0;
      bool failed = false;
      for (int j = b - 1; j >= 0 && !failed; j -= 32) {
        const int idx = j - lane;
        uint64_t w = 0;
        uint32_t flag = 2u;  // before block 0: an inclusive prefix of 0
        uint32_t spins = 0;
        while (true) {
          if (idx >= 0) {
            w = ld_acquire_u64(&p.status[idx]);
            flag = ((w & ~((1ull << 34) - 1)) == tag) ? (uint32_t)((w >> 32) & 3ull) : 0u;
          }
          if (__all_sync(0xffffffffu, flag != 0u)) break;
          if (++spins > kSpinLimit) {
            failed = true;
            break;
          }
        }
        if (failed) break;
        const uint32_t incl = __ballot_sync(0xffffffffu, flag == 2u);
        const int stop = incl ? __ffs(incl) - 1 : 31;  // nearest inclusive predecessor
        const uint32_t v = (lane <= stop && idx >= 0) ? (uint32_t)(w & 0xffffffffull) : 0u;
        excl += (int)__reduce_add_sync(0xffffffffu, v);
        if (incl) break;
      }
      if (lane == 0) {
        if (failed) atomicExch(&p.ws->error, 1u);
        if (b > 0) st_release_u64(&p.status[b], tag | (2ull << 32) | (uint32_t)(excl + local));
        s_excl = excl;
        if (b == p.N * p.GH - 1 && p.active_count != nullptr) *p.active_count = excl + local;
      }
      __syncwarp();
      int off = s_excl;
      for (int base = 0; base < p.GW; base += 32) {
        const int gw = base + lane;
        const bool f = gw < p.GW && s_cls[gw] != SF_TILE_ZERO;
        const uint32_t bal = __ballot_sync(0xffffffffu, f);
        if (f) p.active_ids[off + __popc(bal & ((1u << lane) - 1u))] = (int32_t)(tile_base + gw);
        off += __popc(bal);
      }
    }
  }

  // Last block resets the ticket counter and advances the epoch.
  if (tid == 0) {
    __threadfence();
    const uint32_t d = atomicAdd(&p.ws->done, 1u);
    if (d == (uint32_t)(p.N * p.GH) - 1u) {
      p.ws->ticket = 0u;
      p.ws->done = 0u;
      p.ws->epoch = epoch + 1u;
      __threadfence();
    }
  }
}

// Two-pass path, pass 2: one CTA per (image, run of tile rows). It stages
// the run's receptive-field rows of group words in shared memory once (no
// halo re-reads between tile rows), ORs each row over every tile's
// receptive-field columns (a thread per row and tile column), then each
// tile's rows (a thread per tile), and writes ag_mask, tile_class and each
// tile row's non-ZERO count.
constexpr int kPoolThreads = 256;

__global__ void __launch_bounds__(kPoolThreads) pool_tiles_kernel(PrescanParams p, int rows_per_cta) {
  extern __shared__ __align__(16) uint32_t smem[];
  __shared__ int s_cnt[64];
  const int tid = threadIdx.x;
  const int chunks = (p.GH + rows_per_cta - 1) / rows_per_cta;
  const int n = blockIdx.x / chunks;
  const int gh0 = (blockIdx.x - n * chunks) * rows_per_cta;
  const int gh1 = min(p.GH, gh0 + rows_per_cta);
  const int oh0 = gh0 * p.BH;
  const int oh1 = min(gh1 * p.BH, p.Ho);
  const int ih_lo = max(0, oh0 * p.S - p.P);
  const int ih_hi = min(p.H, (oh1 - 1) * p.S - p.P + p.K);
  const int rows_in = max(0, ih_hi - ih_lo);
  uint32_t* act = smem;
  uint32_t* nanm = smem + p.max_rows_in * p.W;
  const uint2* src = p.bits + ((size_t)n * p.H + ih_lo) * p.W;
  const int total = rows_in * p.W;
  for (int base = tid; base < total; base += 4 * kPoolThreads) {
    uint2 v[4];  // four independent loads in flight per thread
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * kPoolThreads;
      v[u] = i < total ? src[i] : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * kPoolThreads;
      if (i < total) {
        act[i] = v[u].x;
        nanm[i] = v[u].y;
      }
    }
  }
  if (tid < 64) s_cnt[tid] = 0;
  __syncthreads();
  // B1: per (staged input row, tile column) OR of the tile's receptive-field columns.
  uint32_t* racc = nanm + p.max_rows_in * p.W;  // [rows_in][GW] active groups
  uint32_t* rnan = racc + p.max_rows_in * p.GW;  // [rows_in][GW] NaN groups
  for (int idx = tid; idx < rows_in * p.GW; idx += kPoolThreads) {
    const int r = idx / p.GW;
    const int gw = idx - r * p.GW;
    const int ow0 = gw * p.BW;
    const int ow1 = min(ow0 + p.BW, p.Wo);
    const int iw_lo = max(0, ow0 * p.S - p.P);
    const int iw_hi = min(p.W, (ow1 - 1) * p.S - p.P + p.K);
    uint32_t a = 0, nn = 0;
    for (int c = iw_lo; c < iw_hi; ++c) {
      a |= act[r * p.W + c];
      nn |= nanm[r * p.W + c];
    }
    racc[idx] = a;
    rnan[idx] = nn;
  }
  __syncthreads();
  // B2: per tile, OR of its receptive-field rows.
  const int ntiles = (gh1 - gh0) * p.GW;
  for (int t = tid; t < ntiles; t += kPoolThreads) {
    const int ghl = t / p.GW;
    const int gw = t - ghl * p.GW;
    const int toh0 = (gh0 + ghl) * p.BH;
    const int toh1 = min(toh0 + p.BH, p.Ho);
    const int r_lo = max(0, toh0 * p.S - p.P) - ih_lo;
    const int r_hi = min(p.H, (toh1 - 1) * p.S - p.P + p.K) - ih_lo;
    uint32_t a = 0, nn = 0;
    for (int r = r_lo; r < r_hi; ++r) {
      a |= racc[r * p.GW + gw];
      nn |= rnan[r * p.GW + gw];
    }
    const uint32_t m = a & ~nn & p.group_full;
    const int cls = (m == 0u) ? SF_TILE_ZERO : ((m == p.group_full) ? SF_TILE_DENSEISH : SF_TILE_SPARSE);
    const size_t tile = ((size_t)n * p.GH + gh0 + ghl) * p.GW + gw;
    p.ag_mask[tile] = (int32_t)m;
    p.tile_class[tile] = cls;
    if (cls != SF_TILE_ZERO) atomicAdd(&s_cnt[ghl], 1);
  }
  __syncthreads();
  if (p.row_count != nullptr && tid < gh1 - gh0) p.row_count[(size_t)n * p.GH + gh0 + tid] = s_cnt[tid];
}

// Two-pass path, compaction: block k owns tile rows [k*R, k*R + R) (R*GW <=
// 1024 tiles). It sums the non-ZERO counts of all earlier tile rows, scans its
// own tiles' classes, and writes their ids in ascending order; no block waits
// on another.
constexpr int kCompactThreads = 256;
constexpr int kCompactTiles = 1024;

__global__ void __launch_bounds__(kCompactThreads) compact_ids_kernel(const int32_t* __restrict__ tile_class,
                                                                      const int32_t* __restrict__ row_count,
                                                                      int nrows, int GW, int rows_per_block,
                                                                      int32_t* __restrict__ active_ids,
                                                                      int32_t* __restrict__ active_count) {
  __shared__ int s_warp[kCompactThreads / 32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(nrows, row0 + rows_per_block);
  // 1) Non-ZERO tiles before this block.
  int before = 0;
  for (int r = tid; r < row0; r += 8 * kCompactThreads) {
    int v[8];  // eight independent loads in flight per thread
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = (r + u * kCompactThreads < row0) ? row_count[r + u * kCompactThreads] : 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) before += v[u];
  }
  before = __reduce_add_sync(0xffffffffu, before);
  if (lane == 0) s_warp[warp] = before;
  __syncthreads();
  if (tid == 0) {
    int t = 0;
    for (int w = 0; w < kCompactThreads / 32; ++w) t += s_warp[w];
    s_base = t;
  }
  __syncthreads();
  // 2) Scan this block's tiles: thread tid owns tiles t0 .. t0+3.
  constexpr int kPer = kCompactTiles / kCompactThreads;
  const long long first = (long long)row0 * GW;
  const long long last = (long long)row1 * GW;
  const long long t0 = first + (long long)tid * kPer;
  bool f[kPer];
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    f[i] = (t0 + i < last) && tile_class[t0 + i] != SF_TILE_ZERO;
    cnt += f[i] ? 1 : 0;
  }
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  __syncthreads();  // s_warp reuse
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int off = s_base;
  for (int w = 0; w < warp; ++w) off += s_warp[w];
  off += incl - cnt;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (f[i]) active_ids[off++] = (int32_t)(t0 + i);
  if (blockIdx.x == gridDim.x - 1 && tid == kCompactThreads - 1) *active_count = off;
}

uint16_t half_bits_rne_from_double(double v) {
  // Exact double -> IEEE binary16 rounding (round to nearest, ties to even).
  __half h = __double2half(v);
  return __half_as_ushort(h);
}

float half_bits_to_float(uint16_t b) {
  const uint32_t sign = (b >> 15) & 1u, exp = (b >> 10) & 0x1fu, man = b & 0x3ffu;
  float f;
  if (exp == 0)
    f = std::ldexp((float)man, -24);
  else if (exp == 31)
    f = man ? NAN : INFINITY;
  else
    f = std::ldexp((float)(man | 0x400u), (int)exp - 25);
  return sign ? -f : f;
}

int rows_in_max(const sf_prescan_desc* d) { return (d->block_h - 1) * d->stride + d->kernel; }

// Least non-negative float f with float(half_rn(f)) > thr (rounding to half
// is monotonic, so |v| >= f <=> |half(v)| > thr); NaN when no float qualifies.
float half_compare_cut(float thr) {
  auto above = [thr](uint32_t bits) {
    float f;
    std::memcpy(&f, &bits, 4);
    return __half2float(__float2half_rn(f)) > thr;
  };
  uint32_t lo = 0u, hi = 0x7f800000u;  // +0 .. +inf
  if (!above(hi)) return NAN;
  if (above(lo)) return 0.f;
  while (hi - lo > 1u) {  // invariant: !above(lo), above(hi)
    const uint32_t mid = lo + (hi - lo) / 2u;
    if (above(mid))
      hi = mid;
    else
      lo = mid;
  }
  float f;
  std::memcpy(&f, &hi, 4);
  return f;
}

// Offset and size of the per-pixel group words of the two-pass path.
size_t status_region_bytes(const sf_prescan_desc* d) {
  const size_t blocks = (size_t)d->n * ((d->h_out + d->block_h - 1) / d->block_h);
  return ((16 + 8 * blocks + 255) / 256) * 256;
}
size_t tile_rows(const sf_prescan_desc* d) { return (size_t)d->n * ((d->h_out + d->block_h - 1) / d->block_h); }
// Per-pixel group words, then one count per tile row.
size_t bits_region_bytes(const sf_prescan_desc* d) {
  return (((size_t)d->n * d->h * d->w * 8 + 255) / 256) * 256 + ((4 * tile_rows(d) + 255) / 256) * 256;
}
bool two_pass_ok(const sf_prescan_desc* d) {
  return d->layout == SF_LAYOUT_NCHW && d->n <= 65535;
}

template <typename T>
sf_status launch_bits(const void* x, const sf_prescan_desc* d, float cut, uint2* bits, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int HW = d->h * d->w;
  if (aligned16(x) && HW % V == 0) {
    const dim3 grid((HW + 256 * V - 1) / (256 * V), d->n);
    group_bits_kernel<T, V><<<grid, 256, 0, st>>>(static_cast<const T*>(x), d->c, HW, d->group_size, cut, bits);
  } else {
    const dim3 grid((HW + 255) / 256, d->n);
    group_bits_kernel<T, 1><<<grid, 256, 0, st>>>(static_cast<const T*>(x), d->c, HW, d->group_size, cut, bits);
  }
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <typename T>
sf_status launch_t(const PrescanParams& p, int layout, int vec, size_t smem, cudaStream_t st) {
  const int blocks = p.N * p.GH;
  if (layout == SF_LAYOUT_NHWC) {
    constexpr int V = 16 / sizeof(T);
    if (vec == V)
      prescan2d_kernel<T, V, true><<<blocks, 256, smem, st>>>(p);
    else
      prescan2d_kernel<T, 1, true><<<blocks, 256, smem, st>>>(p);
  } else {
    constexpr int V = 16 / sizeof(T);
    if (vec == V)
      prescan2d_kernel<T, V, false><<<blocks, 256, smem, st>>>(p);
    else
      prescan2d_kernel<T, 1, false><<<blocks, 256, smem, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

}  // namespace

}  // namespace sf

using namespace sf;

static sf_status validate_prescan(const sf_prescan_desc* d) {
  if (!d) return SF_ERR_INVALID_ARG;
  if (d->n <= 0 || d->c <= 0 || d->h <= 0 || d->w <= 0 || d->h_out <= 0 || d->w_out <= 0) return SF_ERR_INVALID_ARG;
  if (d->kernel <= 0 || d->stride <= 0 || d->padding < 0 || d->block_h <= 0 || d->block_w <= 0) return SF_ERR_INVALID_ARG;
  if (d->group_size <= 0) return SF_ERR_INVALID_ARG;
  const int G = (d->c + d->group_size - 1) / d->group_size;
  if (G > 32) return SF_ERR_INVALID_ARG;
  if (d->padding >= d->kernel) return SF_ERR_UNSUPPORTED;
  if (dtype_size(d->dtype) == 0) return SF_ERR_INVALID_ARG;
  if (d->layout != SF_LAYOUT_NCHW && d->layout != SF_LAYOUT_NHWC) return SF_ERR_INVALID_ARG;
  // Output size must match the conv geometry.
  if ((d->h + 2 * d->padding - d->kernel) / d->stride + 1 != d->h_out) return SF_ERR_INVALID_ARG;
  if ((d->w + 2 * d->padding - d->kernel) / d->stride + 1 != d->w_out) return SF_ERR_INVALID_ARG;
  const int GW = (d->w_out + d->block_w - 1) / d->block_w;
  if (GW > 256) return SF_ERR_UNSUPPORTED;
  const size_t smem = 2ull * rows_in_max(d) * d->w * 4ull;
  if (smem > 200u * 1024u) return SF_ERR_UNSUPPORTED;
  const long long tiles = (long long)d->n * ((d->h_out + d->block_h - 1) / d->block_h) * GW;
  if (tiles >= (1ll << 31)) return SF_ERR_UNSUPPORTED;
  return SF_OK;
}

// Look-back words only: the one-pass kernel (and sf_prescan2d_static_ws).
static size_t prescan_min_workspace(const sf_prescan_desc* d) {
  const size_t blocks = (size_t)d->n * ((d->h_out + d->block_h - 1) / d->block_h);
  return 16 + 8 * blocks;
}

extern "C" size_t sf_prescan2d_workspace_size(const sf_prescan_desc* d) {
  if (validate_prescan(d) != SF_OK) return 0;
  if (two_pass_ok(d)) return status_region_bytes(d) + bits_region_bytes(d);
  return prescan_min_workspace(d);
}

extern "C" sf_status sf_prescan2d(const void* x, const sf_prescan_desc* d, int32_t* ag_mask,
                                  int32_t* tile_class, int32_t* active_ids, int32_t* active_count,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  sf_status s = validate_prescan(d);
  if (s != SF_OK) return s;
  if (!x || !ag_mask || !tile_class) return SF_ERR_INVALID_ARG;
  if ((active_ids == nullptr) != (active_count == nullptr)) return SF_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < prescan_min_workspace(d)) return SF_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 7u) != 0) return SF_ERR_ALIGNMENT;

  PrescanParams p;
  p.x = x;
  p.ag_mask = ag_mask;
  p.tile_class = tile_class;
  p.active_ids = active_ids;
  p.active_count = active_count;
  p.ws = static_cast<PrescanWs*>(workspace);
  p.status = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + 16);
  p.N = d->n; p.C = d->c; p.H = d->h; p.W = d->w; p.Ho = d->h_out; p.Wo = d->w_out;
  p.K = d->kernel; p.S = d->stride; p.P = d->padding; p.BH = d->block_h; p.BW = d->block_w;
  p.gs = d->group_size;
  p.G = (d->c + d->group_size - 1) / d->group_size;
  p.GH = (d->h_out + d->block_h - 1) / d->block_h;
  p.GW = (d->w_out + d->block_w - 1) / d->block_w;
  p.group_full = (p.G == 32) ? 0xffffffffu : ((1u << p.G) - 1u);
  p.thr = half_bits_to_float(half_bits_rne_from_double(d->threshold));
  p.max_rows_in = rows_in_max(d);
  p.bits = nullptr;
  p.row_count = nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // With the full workspace (sf_prescan2d_workspace_size), NCHW inputs take
  // two passes: a streaming channel fold, then tile pooling from its output.
  // A workspace of only the look-back words selects the one-pass kernel.
  if (two_pass_ok(d) && workspace_bytes >= status_region_bytes(d) + bits_region_bytes(d) &&
      (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0) {
    uint2* bits = reinterpret_cast<uint2*>(static_cast<char*>(workspace) + status_region_bytes(d));
    const float cut = half_compare_cut(p.thr);
    sf_status s1 = SF_ERR_INVALID_ARG;
    switch (d->dtype) {
      case SF_DTYPE_F32: s1 = launch_bits<float>(x, d, cut, bits, st); break;
      case SF_DTYPE_F16: s1 = launch_bits<__half>(x, d, cut, bits, st); break;
      case SF_DTYPE_BF16: s1 = launch_bits<__nv_bfloat16>(x, d, cut, bits, st); break;
    }
    if (s1 != SF_OK) return s1;
    p.bits = bits;
    p.row_count = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(bits) +
                                             (((size_t)d->n * d->h * d->w * 8 + 255) / 256) * 256);
  }

  const size_t esz = dtype_size(d->dtype);
  const int V = (int)(16 / esz);
  int vec = 1;
  if (aligned16(x)) {
    if (d->layout == SF_LAYOUT_NCHW && d->w % V == 0) vec = V;
    if (d->layout == SF_LAYOUT_NHWC && d->c % V == 0) vec = V;
  }
  const size_t smem = 2ull * p.max_rows_in * p.W * 4ull;
  // Opt in to large dynamic shared memory once per instantiation.
  if (smem > 48 * 1024) {
    cudaError_t e = cudaSuccess;
#define SF_ATTR(T, V_, NH)                                                                      \
  e = cudaFuncSetAttribute(prescan2d_kernel<T, V_, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)smem);                                                          \
  if (e != cudaSuccess) return SF_ERR_CUDA;
    if (d->dtype == SF_DTYPE_F32) { SF_ATTR(float, 4, false) SF_ATTR(float, 1, false) SF_ATTR(float, 4, true) SF_ATTR(float, 1, true) }
    if (d->dtype == SF_DTYPE_F16) { SF_ATTR(__half, 8, false) SF_ATTR(__half, 1, false) SF_ATTR(__half, 8, true) SF_ATTR(__half, 1, true) }
    if (d->dtype == SF_DTYPE_BF16) { SF_ATTR(__nv_bfloat16, 8, false) SF_ATTR(__nv_bfloat16, 1, false) SF_ATTR(__nv_bfloat16, 8, true) SF_ATTR(__nv_bfloat16, 1, true) }
#undef SF_ATTR
  }
  if (p.bits != nullptr) {
    // Tile rows per pooling CTA: as many as 48 KB of staged rows allow (<= 64).
    // Staged rows: group words (2 x W) plus per-row tile-column ORs (2 x GW).
    auto pool_smem = [&](int rows) { return 2ull * rows * (p.W + p.GW) * 4; };
    int rpc = 1;
    while (rpc < 64 && rpc < p.GH && pool_smem(((rpc + 1) * p.BH - 1) * p.S + p.K) <= 48 * 1024) ++rpc;
    p.max_rows_in = std::min(p.H, (rpc * p.BH - 1) * p.S + p.K);
    const size_t psmem = pool_smem(p.max_rows_in);
    const int chunks = (p.GH + rpc - 1) / rpc;
    if (psmem > 48 * 1024 &&
        cudaFuncSetAttribute(pool_tiles_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem) != cudaSuccess)
      return SF_ERR_CUDA;
    pool_tiles_kernel<<<p.N * chunks, kPoolThreads, psmem, st>>>(p, rpc);
    if (cudaGetLastError() != cudaSuccess) return SF_ERR_CUDA;
    if (active_ids == nullptr) return SF_OK;
    const int nrows = p.N * p.GH;
    const int rows_per_block = std::max(1, kCompactTiles / p.GW);
    compact_ids_kernel<<<(nrows + rows_per_block - 1) / rows_per_block, kCompactThreads, 0, st>>>(
        tile_class, p.row_count, nrows, p.GW, rows_per_block, active_ids, active_count);
    return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
  }
  sf_status s2 = SF_ERR_INVALID_ARG;
  switch (d->dtype) {
    case SF_DTYPE_F32: s2 = launch_t<float>(p, d->layout, vec, smem, st); break;
    case SF_DTYPE_F16: s2 = launch_t<__half>(p, d->layout, vec, smem, st); break;
    case SF_DTYPE_BF16: s2 = launch_t<__nv_bfloat16>(p, d->layout, vec, smem, st); break;
  }
  return s2;
}

extern "C" sf_status sf_prescan2d_status(void* workspace, void* stream) {
  if (!workspace) return SF_ERR_INVALID_ARG;
  uint32_t err = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&err, static_cast<char*>(workspace) + 12, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return SF_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return SF_ERR_CUDA;
  return err ? SF_ERR_DEVICE_TIMEOUT : SF_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of sf_prescan2d.
//
// Some callers cannot allocate device memory when they run the prescan:
// code inside a host runtime that owns all allocations (an engine with a
// fixed arena, a plugin whose host forbids cudaMalloc while it executes), or
// a hot path where an allocation would synchronise the device. For them the
// look-back workspace lives in this file-scope device array instead of a
// caller buffer. It is sized for SF_PRESCAN_STATIC_MAX_ROWS tile rows
// (n * ceil(h_out / block_h)); every GPU that loads this library holds it
// until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

constexpr size_t kStaticWsBytes = 16 + 8 * (size_t)SF_PRESCAN_STATIC_MAX_ROWS;
static __device__ __align__(256) unsigned char g_prescan_static_ws[kStaticWsBytes];

std::mutex g_static_ws_mu;
void* g_static_ws_ptr[64] = {nullptr};

// Device address of g_prescan_static_ws on the current device, looked up
// once per device (the host-side symbol is not a device address).
sf_status static_ws_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SF_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_static_ws_mu);
  if (g_static_ws_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_prescan_static_ws) != cudaSuccess || ptr == nullptr) return SF_ERR_CUDA;
    g_static_ws_ptr[dev] = ptr;
  }
  *out = g_static_ws_ptr[dev];
  return SF_OK;
}

}  // namespace

extern "C" sf_status sf_prescan2d_static_ws(const void* x, const sf_prescan_desc* d, int32_t* ag_mask,
                                            int32_t* tile_class, int32_t* active_ids, int32_t* active_count,
                                            void* stream) {
  const sf_status v = validate_prescan(d);
  if (v != SF_OK) return v;
  const size_t need = prescan_min_workspace(d);
  if (need > kStaticWsBytes) return SF_ERR_WORKSPACE;  // more than SF_PRESCAN_STATIC_MAX_ROWS tile rows
  void* ws = nullptr;
  sf_status s = static_ws_for_current_device(&ws);
  if (s != SF_OK) return s;
  // The array keeps the previous call's contents. The ticket and done
  // counters (bytes 0-7) and the error word (bytes 12-15) must start at zero;
  // the epoch word (bytes 8-11) must not be reset, since it keeps the
  // previous call's look-back status words from being read as current.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(ws, 0, 8, st) != cudaSuccess) return SF_ERR_CUDA;
  if (cudaMemsetAsync(static_cast<char*>(ws) + 12, 0, 4, st) != cudaSuccess) return SF_ERR_CUDA;
  // Passing exactly the look-back size selects the one-pass kernel for every
  // shape: the two-pass path would write per-pixel group words over the
  // status words that a later one-pass call reads as predecessor state.
  return sf_prescan2d(x, d, ag_mask, tile_class, active_ids, active_count, ws, need, stream);
}

extern "C" sf_status sf_prescan2d_static_ws_status(void* stream) {
  uint32_t err = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyFromSymbolAsync(&err, g_prescan_static_ws, 4, 12, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return SF_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return SF_ERR_CUDA;
  return err ? SF_ERR_DEVICE_TIMEOUT : SF_OK;
}
