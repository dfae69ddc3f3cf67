// C-ABI entry points of stage 2 (sparse conv) and of the fused conv+LIF
// kernel: argument checks, launch planning, weight packing. The kernel itself
// is in conv_kernel.cuh.
#include <cstdlib>
#include <cstring>
#include <cudaTypedefs.h>
#include "conv_kernel.cuh"

namespace sf {
namespace conv {
namespace {

// Set when a bounded wait in the conv kernel runs out (read by
// sf_sparse_conv2d_status); a static device word, so no allocation is needed.
__device__ uint32_t g_conv_error = 0;

template <typename WT>
__global__ void pack_weights_kernel(const void* __restrict__ w, int src_dtype, WT* __restrict__ out, int Co,
                                    int Ci, int KK, int Co_pad) {
  const size_t total = (size_t)Ci * KK * Co_pad;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int co = (int)(i % Co_pad);
    const size_t r = i / Co_pad;
    const int t = (int)(r % KK);
    const int ci = (int)(r / KK);
    float v = 0.f;
    if (co < Co) {
      const size_t src = ((size_t)co * Ci + ci) * KK + t;
      if (src_dtype == SF_DTYPE_F32)
        v = static_cast<const float*>(w)[src];
      else if (src_dtype == SF_DTYPE_F16)
        v = __half2float(static_cast<const __half*>(w)[src]);
      else
        v = __bfloat162float(static_cast<const __nv_bfloat16*>(w)[src]);
    }
    if constexpr (sizeof(WT) == 4)
      out[i] = v;
    else
      out[i] = __float2bfloat16_rn(v);
  }
}

int env_int(const char* name) {
  const char* v = getenv(name);
  return v ? atoi(v) : 0;
}

// Launch plan: output channels per lane (CPL), row-segment length R, band
// height TH (one row segment per compute warp), channels per chunk (cc),
// stages, and whether the packed weights live in shared memory. The
// environment variables SF_CONV_CC / SF_CONV_TH / SF_CONV_NSTAGE /
// SF_CONV_NO_WSMEM / SF_CONV_NO_TMA pin choices for tuning sweeps.
bool make_plan(int K, int S, int P, int C, int H, int W, int Co, int Ho, int Wo, int esz, int wsz, bool lif,
               Plan& pl) {
  (void)H; (void)P; (void)lif;
  const int force_cc = env_int("SF_CONV_CC"), force_th = env_int("SF_CONV_TH"), force_ns = env_int("SF_CONV_NSTAGE");
  // A 4-D tensor map needs a 16-byte row pitch and box extents <= 256.
  const bool tmap_ok = (W * esz) % 16 == 0 && W <= 256 && env_int("SF_CONV_NO_TMA") == 0;
  pl.CPL = Co <= 32 ? 1 : (Co <= 64 ? 2 : 4);
  pl.R = pl.CPL == 4 ? 4 : 8;
  const int tpr = (Wo + pl.R - 1) / pl.R;
  const int tpu = std::min(tpr, kComputeWarps);  // wider rows are split into column blocks
  const int th_max = std::min(Ho, kComputeWarps / tpu);
  const int ncob = (Co + co_block(Co) - 1) / co_block(Co);
  const int w_bytes = C * K * K * co_padded(Co) * wsz;
  const bool ws_ok = ncob == 1 && env_int("SF_CONV_NO_WSMEM") == 0;
  const int cb_bytes = ((kMaxStages * kCbStride * 4 + 127) / 128) * 128;
  const int bar_bytes = (2 * kMaxStages + 1) * 8;
  for (int wsmem = ws_ok ? 1 : 0; wsmem >= 0; --wsmem) {
    const int w_region = wsmem ? ((w_bytes + 127) / 128) * 128 : 0;
    for (int cc = std::min(kCC, ((C + 7) / 8) * 8); cc >= 8; cc /= 2) {
      if (force_cc && cc != force_cc) continue;
      for (int TH = th_max; TH >= 1; --TH) {
        if (force_th && TH != force_th) continue;
        const int th_in = (TH - 1) * S + K;
        // Tensor copies land densely (channel pitch th_in*W); bulk copies need
        // 16 bytes of slack for the aligned-out byte range.
        const int slot_bytes = tmap_ok ? th_in * W * esz : ((th_in * W * esz + 15) / 16) * 16 + 16;
        const int stage_bytes = ((cc * slot_bytes + 127) / 128) * 128;
        const int fixed = w_region + cb_bytes + bar_bytes;
        if (fixed >= kSmemLimit) continue;
        int nstage = std::min(kMaxStages, (kSmemLimit - fixed) / stage_bytes);
        if (force_ns) {
          if (force_ns > nstage) continue;
          nstage = force_ns;
        }
        if (nstage < 2) continue;
        // Stage pitch must stay a whole number of slots.
        if (stage_bytes != cc * slot_bytes) continue;
        pl.wsmem = wsmem;
        pl.cc = cc;
        pl.use_tmap = tmap_ok ? 1 : 0;
        pl.TH = TH;
        pl.th_in = th_in;
        pl.nstage = nstage;
        pl.slot_elems = slot_bytes / esz;
        pl.w_off = nstage * stage_bytes;
        pl.cb_off = pl.w_off + w_region;
        pl.bar_off = pl.cb_off + cb_bytes;
        pl.smem = pl.bar_off + bar_bytes;
        return true;
      }
    }
  }
  return false;
}

int g_num_sms[64] = {0};

}  // namespace
}  // namespace conv

int num_sms_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (conv::g_num_sms[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    conv::g_num_sms[dev] = v;
  }
  return conv::g_num_sms[dev];
}

namespace conv {
namespace {

sf_status dispatch(bool lif, int xdt, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& tm,
                   const Plan& pl, cudaStream_t st) {
  if (xdt == SF_DTYPE_F32) return dispatch_f32(lif, wdt, K, S, p, tm, pl, st);
  if (xdt == SF_DTYPE_F16) return dispatch_f16(lif, wdt, K, S, p, tm, pl, st);
  if (xdt == SF_DTYPE_BF16) return dispatch_bf16(lif, wdt, K, S, p, tm, pl, st);
  return SF_ERR_UNSUPPORTED;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// x viewed as 4-D (W, H, C, T*N), box (W, th_in, cc, 1), zero fill outside.
sf_status encode_x_map(CUtensorMap* m, const void* x, int xdt, int W, int H, int C, long long nimg, int th_in,
                       int cc) {
  auto fn = tensor_map_encoder();
  if (!fn) return SF_ERR_CUDA;
  const CUtensorMapDataType dt = xdt == SF_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : xdt == SF_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t esz = dtype_size(xdt);
  const cuuint64_t dims[4] = {(cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)C, (cuuint64_t)nimg};
  const cuuint64_t strides[3] = {W * esz, (cuuint64_t)H * W * esz, (cuuint64_t)C * H * W * esz};
  const cuuint32_t box[4] = {(cuuint32_t)W, (cuuint32_t)th_in, (cuuint32_t)cc, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUresult r = fn(m, dt, 4, const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SF_OK : SF_ERR_CUDA;
}

sf_status conv_common(const void* x, const void* w_packed, const float* bias, void* y, int T, int N, int C,
                      int H, int W, int Co, int Ho, int Wo, int K, int S, int P, int xdt, int wdt, bool lif,
                      ConvParams& p, Plan& pl, CUtensorMap& tm) {
  if (!x || !w_packed || !y) return SF_ERR_INVALID_ARG;
  if (T <= 0 || N <= 0 || C <= 0 || H <= 0 || W <= 0 || Co <= 0 || Ho <= 0 || Wo <= 0) return SF_ERR_INVALID_ARG;
  if (!((K == 1 && S == 1 && P == 0) || (K == 3 && S == 1 && P == 1) || (K == 3 && S == 2 && P == 1)))
    return SF_ERR_UNSUPPORTED;
  if ((H + 2 * P - K) / S + 1 != Ho || (W + 2 * P - K) / S + 1 != Wo) return SF_ERR_INVALID_ARG;
  const size_t esz = dtype_size(xdt);
  if (esz == 0 || (wdt != SF_DTYPE_F32 && wdt != SF_DTYPE_BF16)) return SF_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_packed)) return SF_ERR_ALIGNMENT;
  if (!make_plan(K, S, P, C, H, W, Co, Ho, Wo, (int)esz, (int)dtype_size(wdt), lif, pl)) return SF_ERR_UNSUPPORTED;
  p.x = x;
  p.wp = w_packed;
  p.bias = bias;
  p.y = y;
  p.v = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p.err), g_conv_error) != cudaSuccess) return SF_ERR_CUDA;
  p.T = T; p.N = N; p.C = C; p.H = H; p.W = W; p.Co = Co; p.Ho = Ho; p.Wo = Wo; p.P = P;
  p.Co_pad = co_padded(Co);
  p.TH = pl.TH;
  p.nbands = (Ho + pl.TH - 1) / pl.TH;
  const int COB = 32 * pl.CPL;
  p.ncob = (Co + COB - 1) / COB;
  p.tpr = (Wo + pl.R - 1) / pl.R;
  p.tpu = std::min(p.tpr, kComputeWarps);
  p.ncolb = (p.tpr + p.tpu - 1) / p.tpu;
  const long long units = (long long)N * p.nbands * p.ncolb * p.ncob;
  if (units >= (1ll << 31)) return SF_ERR_UNSUPPORTED;
  p.n_units = (int)units;
  p.th_in = pl.th_in;
  p.slot_elems = pl.slot_elems;
  p.cc = pl.cc;
  p.nchunks = (C + pl.cc - 1) / pl.cc;
  p.nstage = pl.nstage;
  p.w_off = pl.w_off;
  p.w_bytes = (uint32_t)((size_t)C * K * K * p.Co_pad * dtype_size(wdt));
  p.cb_off = pl.cb_off;
  p.bar_off = pl.bar_off;
  p.tau = 1.f; p.vth = 1.f; p.vreset = 0.f; p.hard_reset = 1; p.decay_input = 1;
  p.use_tmap = pl.use_tmap;
  p.box_bytes = (uint32_t)((size_t)W * pl.th_in * pl.cc * esz);
  memset(&tm, 0, sizeof(tm));
  if (pl.use_tmap) {
    sf_status s = encode_x_map(&tm, x, xdt, W, H, C, (long long)T * N, pl.th_in, pl.cc);
    if (s != SF_OK) return s;
  }
  return SF_OK;
}

}  // namespace
}  // namespace conv
}  // namespace sf

using namespace sf;
using namespace sf::conv;

extern "C" size_t sf_packed_weight_bytes(int32_t c_out, int32_t c_in, int32_t kernel, int32_t w_dst_dtype) {
  if (c_out <= 0 || c_in <= 0 || kernel <= 0) return 0;
  const size_t esz = dtype_size(w_dst_dtype);
  const size_t co_pad = (size_t)co_padded(c_out);
  return (size_t)c_in * kernel * kernel * co_pad * esz;
}

extern "C" sf_status sf_pack_weights(const void* w_oihw, int32_t w_src_dtype, int32_t c_out, int32_t c_in,
                                     int32_t kernel, int32_t w_dst_dtype, void* w_packed, void* stream) {
  if (!w_oihw || !w_packed || c_out <= 0 || c_in <= 0 || kernel <= 0) return SF_ERR_INVALID_ARG;
  if (dtype_size(w_src_dtype) == 0) return SF_ERR_INVALID_ARG;
  if (w_dst_dtype != SF_DTYPE_F32 && w_dst_dtype != SF_DTYPE_BF16) return SF_ERR_UNSUPPORTED;
  const int co_pad = co_padded(c_out);
  const int KK = kernel * kernel;
  const size_t total = (size_t)c_in * KK * co_pad;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w_dst_dtype == SF_DTYPE_F32)
    pack_weights_kernel<float><<<blocks, 256, 0, st>>>(w_oihw, w_src_dtype, static_cast<float*>(w_packed), c_out,
                                                       c_in, KK, co_pad);
  else
    pack_weights_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        w_oihw, w_src_dtype, static_cast<__nv_bfloat16*>(w_packed), c_out, c_in, KK, co_pad);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

extern "C" sf_status sf_sparse_conv2d(const void* x, const void* w_packed, const float* bias, void* y,
                                      const sf_conv_desc* d, void* stream) {
  if (!d) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  ConvParams p;
  Plan pl;
  CUtensorMap tm;
  sf_status s = conv_common(x, w_packed, d->has_bias ? bias : nullptr, y, 1, d->n, d->c_in, d->h, d->w, d->c_out,
                            d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype, d->w_dtype, false, p, pl, tm);
  if (s != SF_OK) return s;
  return dispatch(false, d->x_dtype, d->w_dtype, d->kernel, d->stride, p, tm, pl, static_cast<cudaStream_t>(stream));
}

extern "C" sf_status sf_fused_conv_lif(const void* x, const void* w_packed, const float* bias, float* v_inout,
                                       void* spikes_out, const sf_lif_desc* d, void* stream) {
  if (!d || !v_inout) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  if (!(d->tau > 0.f)) return SF_ERR_INVALID_ARG;
  ConvParams p;
  Plan pl;
  CUtensorMap tm;
  sf_status s = conv_common(x, w_packed, d->has_bias ? bias : nullptr, spikes_out, d->t_steps, d->n, d->c_in, d->h,
                            d->w, d->c_out, d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype,
                            d->w_dtype, true, p, pl, tm);
  if (s != SF_OK) return s;
  p.v = v_inout;
  p.tau = d->tau;
  p.vth = d->v_threshold;
  p.vreset = d->hard_reset ? d->v_reset : 0.f;
  p.hard_reset = d->hard_reset;
  p.decay_input = d->decay_input;
  return dispatch(true, d->x_dtype, d->w_dtype, d->kernel, d->stride, p, tm, pl, static_cast<cudaStream_t>(stream));
}

extern "C" sf_status sf_sparse_conv2d_status(void* stream) {
  uint32_t err = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyFromSymbolAsync(&err, g_conv_error, 4, 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return SF_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return SF_ERR_CUDA;
  return err ? SF_ERR_DEVICE_TIMEOUT : SF_OK;
}

extern "C" int32_t sf_abi_version(void) { return SF_ABI_VERSION; }

extern "C" const char* sf_status_string(sf_status s) {
  switch (s) {
    case SF_OK: return "ok";
    case SF_ERR_INVALID_ARG: return "invalid argument";
    case SF_ERR_UNSUPPORTED: return "unsupported configuration";
    case SF_ERR_ALIGNMENT: return "pointer or size not 16-byte aligned";
    case SF_ERR_WORKSPACE: return "workspace missing or too small";
    case SF_ERR_CUDA: return "CUDA runtime error";
    case SF_ERR_DEVICE_TIMEOUT: return "bounded device wait expired";
  }
  return "unknown status";
}
