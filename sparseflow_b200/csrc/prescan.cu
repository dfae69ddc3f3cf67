// Stage 1: receptive-field prescan (single pass over x, HBM-bound).
//
// Semantics follow Kernels/_prescan_common.py:32-189 of the reference:
//   group_max[n,ih,iw,g] = amax_{c in g} |half(x)|             (:32-45)
//   rf_max   = max_pool2d(group_max, k, s, p)                   (:169-177)
//   tile_max = max_pool2d(rf_max, (BH,BW), ceil_mode=True)      (:182-187)
//   active   = tile_max > half(threshold)   (compared in half)  (:188)
//   ag_mask  = sum_g active_g << g ; class ZERO/SPARSE/DENSEISH (:48-109)
// and Kernels/conv2d.py:113-123 (ids of non-ZERO tiles, ascending).
//
// B200 design: one CTA per (image, tile row). The CTA streams the tile row's
// receptive-field rows of every channel once with 16-byte vector loads, folds
// them into a per-input-pixel group bitmap in shared memory (plus a NaN bitmap:
// a NaN anywhere in a pooling window makes the reference's max NaN and the
// comparison false), then ORs each tile's receptive-field rectangle with one
// warp per tile. Active tile ids are compacted in global order with a
// decoupled look-back scan over CTAs that take logical indices from a ticket
// counter, so no second launch and no host sync is needed.
#include <cmath>
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
      // Decoupled look-back over logical blocks.
      const uint64_t tag = (uint64_t)((epoch + 1u) & 0x3fffffffu) << 34;
      if (lane == 0) {
        int excl = 0;
        if (b == 0) {
          st_release_u64(&p.status[0], tag | (2ull << 32) | (uint32_t)local);
        } else {
          st_release_u64(&p.status[b], tag | (1ull << 32) | (uint32_t)local);
          int j = b - 1;
          bool failed = false;
          while (j >= 0) {
            uint64_t w = 0;
            uint32_t spins = 0;
            while (true) {
              w = ld_acquire_u64(&p.status[j]);
              if ((w & ~((1ull << 34) - 1)) == tag && ((w >> 32) & 3ull) != 0ull) break;
              if (++spins > kSpinLimit) { failed = true; break; }
            }
            if (failed) break;
            excl += (int)(uint32_t)(w & 0xffffffffull);
            if (((w >> 32) & 3ull) == 2ull) break;
            --j;
          }
          if (failed) atomicExch(&p.ws->error, 1u);
          st_release_u64(&p.status[b], tag | (2ull << 32) | (uint32_t)(excl + local));
        }
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

extern "C" size_t sf_prescan2d_workspace_size(const sf_prescan_desc* d) {
  if (validate_prescan(d) != SF_OK) return 0;
  const size_t blocks = (size_t)d->n * ((d->h_out + d->block_h - 1) / d->block_h);
  return 16 + 8 * blocks;
}

extern "C" sf_status sf_prescan2d(const void* x, const sf_prescan_desc* d, int32_t* ag_mask,
                                  int32_t* tile_class, int32_t* active_ids, int32_t* active_count,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  sf_status s = validate_prescan(d);
  if (s != SF_OK) return s;
  if (!x || !ag_mask || !tile_class) return SF_ERR_INVALID_ARG;
  if ((active_ids == nullptr) != (active_count == nullptr)) return SF_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < sf_prescan2d_workspace_size(d)) return SF_ERR_WORKSPACE;
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

  const size_t esz = dtype_size(d->dtype);
  const int V = (int)(16 / esz);
  int vec = 1;
  if (aligned16(x)) {
    if (d->layout == SF_LAYOUT_NCHW && d->w % V == 0) vec = V;
    if (d->layout == SF_LAYOUT_NHWC && d->c % V == 0) vec = V;
  }
  const size_t smem = 2ull * p.max_rows_in * p.W * 4ull;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
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
  switch (d->dtype) {
    case SF_DTYPE_F32: return launch_t<float>(p, d->layout, vec, smem, st);
    case SF_DTYPE_F16: return launch_t<__half>(p, d->layout, vec, smem, st);
    case SF_DTYPE_BF16: return launch_t<__nv_bfloat16>(p, d->layout, vec, smem, st);
  }
  return SF_ERR_INVALID_ARG;
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
  const size_t need = sf_prescan2d_workspace_size(d);
  if (need == 0) return validate_prescan(d) != SF_OK ? validate_prescan(d) : SF_ERR_INVALID_ARG;
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
  return sf_prescan2d(x, d, ag_mask, tile_class, active_ids, active_count, ws, kStaticWsBytes, stream);
}
