// C-ABI entry points of the sparse convolution (stage 1 event extraction +
// stage 2 gather) and of the fused conv+LIF kernel: argument checks, launch
// planning, weight packing. The kernels are in events.cu and conv_kernel.cuh.
#include <cstdlib>
#include <cstring>
#include "conv_kernel.cuh"
#include "events.cuh"

namespace sf {
namespace conv {
namespace {

// Set when a bounded wait in the conv kernel runs out (read by
// sf_sparse_conv2d_status); a static device word, so no allocation is needed.
__device__ uint32_t g_conv_error = 0;

// [co][ci][kk] (any dtype) -> [slice][ci][kk][32] (fp32 or bf16), zero padded.
template <typename WT>
__global__ void pack_weights_kernel(const void* __restrict__ w, int src_dtype, WT* __restrict__ out, int Co, int Ci,
                                    int KK, int slices) {
  const size_t total = (size_t)slices * Ci * KK * 32;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int l = (int)(i & 31);
    size_t r = i >> 5;
    const int t = (int)(r % KK);
    r /= KK;
    const int ci = (int)(r % Ci);
    const int sl = (int)(r / Ci);
    const int co = sl * 32 + l;
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

// Launch plan: 32-channel slices per lane (CPL), row-segment length R, band
// height TH (one row segment per compute warp), mask stages, and whether a
// block of packed weights lives in shared memory. SF_CONV_CPL / SF_CONV_TH /
// SF_CONV_NSTAGE / SF_CONV_NO_WSMEM (environment) pin choices for tuning.
bool make_plan(int K, int S, int C, int W, int Co, int Ho, int Wo, int nw, int wsz, Plan& pl) {
  const int force_cpl = env_int("SF_CONV_CPL"), force_th = env_int("SF_CONV_TH"), force_ns = env_int("SF_CONV_NSTAGE");
  const int slices = (Co + 31) / 32;
  const int bar_bytes = (2 * kMaxStages + 1) * 8;
  for (int wsmem = env_int("SF_CONV_NO_WSMEM") ? 0 : 1; wsmem >= 0; --wsmem) {
    for (int cpl = 4; cpl >= 1; cpl /= 2) {
      if (force_cpl && cpl != force_cpl) continue;
      if (!force_cpl && cpl > 1 && cpl > slices) continue;  // no wider block than the layer
      const int R = cpl == 4 ? 4 : 8;
      const int tpr = (Wo + R - 1) / R;
      const int tpu = std::min(tpr, kComputeWarps);
      const size_t w_bytes = (size_t)C * K * K * 32 * cpl * wsz;
      const int w_region = wsmem ? (int)std::min<size_t>(((w_bytes + 127) / 128) * 128, 1u << 30) : 0;
      for (int TH = std::min(Ho, kComputeWarps / tpu); TH >= 1; --TH) {
        if (force_th && TH != force_th) continue;
        const int th_in = (TH - 1) * S + K;
        const int slot_words = ((th_in * W * nw + 2) + 1) & ~1;
        const int stage_bytes = slot_words * 8;
        const long long fixed = (long long)w_region + bar_bytes;
        if (fixed + 2ll * stage_bytes > kSmemLimit) continue;
        int nstage = (int)std::min<long long>(kMaxStages, (kSmemLimit - fixed) / stage_bytes);
        if (force_ns) {
          if (force_ns > nstage) continue;
          nstage = force_ns;
        }
        pl.CPL = cpl;
        pl.R = R;
        pl.wsmem = wsmem;
        pl.TH = TH;
        pl.th_in = th_in;
        pl.nstage = nstage;
        pl.slot_words = slot_words;
        pl.w_off = nstage * stage_bytes;
        pl.bar_off = pl.w_off + w_region;
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

sf_status dispatch(bool lif, int xdt, int wdt, int K, int S, const ConvParams& p, int grid, const Plan& pl,
                   cudaStream_t st) {
  if (xdt == SF_DTYPE_F32) return dispatch_f32(lif, wdt, K, S, p, grid, pl, st);
  if (xdt == SF_DTYPE_F16) return dispatch_f16(lif, wdt, K, S, p, grid, pl, st);
  if (xdt == SF_DTYPE_BF16) return dispatch_bf16(lif, wdt, K, S, p, grid, pl, st);
  return SF_ERR_UNSUPPORTED;
}

sf_status check_geometry(int T, int N, int C, int H, int W, int Co, int Ho, int Wo, int K, int S, int P, int xdt,
                         int wdt) {
  if (T <= 0 || N <= 0 || C <= 0 || H <= 0 || W <= 0 || Co <= 0 || Ho <= 0 || Wo <= 0) return SF_ERR_INVALID_ARG;
  if (!((K == 1 && S == 1 && P == 0) || (K == 3 && S == 1 && P == 1) || (K == 3 && S == 2 && P == 1)))
    return SF_ERR_UNSUPPORTED;
  if ((H + 2 * P - K) / S + 1 != Ho || (W + 2 * P - K) / S + 1 != Wo) return SF_ERR_INVALID_ARG;
  if (dtype_size(xdt) == 0 || (wdt != SF_DTYPE_F32 && wdt != SF_DTYPE_BF16)) return SF_ERR_INVALID_ARG;
  if ((long long)T * N >= 65536) return SF_ERR_UNSUPPORTED;
  return SF_OK;
}

// Stage 1 + stage 2 for T*N images; the LIF variant when lif is set.
sf_status run_conv(const void* x, const void* w_packed, const float* bias, void* y, float* v, int T, int N, int C,
                   int H, int W, int Co, int Ho, int Wo, int K, int S, int P, int xdt, int wdt, bool lif,
                   const sf_lif_desc* lifd, void* workspace, size_t ws_bytes, cudaStream_t st) {
  sf_status s = check_geometry(T, N, C, H, W, Co, Ho, Wo, K, S, P, xdt, wdt);
  if (s != SF_OK) return s;
  if (!x || !w_packed || !y) return SF_ERR_INVALID_ARG;
  if (!workspace) return SF_ERR_WORKSPACE;
  if (!aligned16(w_packed)) return SF_ERR_ALIGNMENT;
  const int nw = (C + 63) / 64;
  Plan pl;
  if (!make_plan(K, S, C, W, Co, Ho, Wo, nw, (int)dtype_size(wdt), pl)) return SF_ERR_UNSUPPORTED;

  EventBuffers ev;
  s = extract_events(x, xdt, (long long)T * N, C, H * W, workspace, ws_bytes, ev, st);
  if (s != SF_OK) return s;

  ConvParams p;
  memset(&p, 0, sizeof(p));
  p.x = x;
  p.wp = w_packed;
  p.bias = bias;
  p.y = y;
  p.v = v;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p.err), g_conv_error) != cudaSuccess) return SF_ERR_CUDA;
  p.masks = ev.masks;
  p.flags = ev.flags;
  p.nw = nw;
  p.tau = 1.f;
  p.vth = 1.f;
  p.vreset = 0.f;
  p.hard_reset = 1;
  p.decay_input = 1;
  if (lif) {
    p.tau = lifd->tau;
    p.vth = lifd->v_threshold;
    p.vreset = lifd->hard_reset ? lifd->v_reset : 0.f;
    p.hard_reset = lifd->hard_reset;
    p.decay_input = lifd->decay_input;
  }
  p.T = T; p.N = N; p.C = C; p.H = H; p.W = W; p.Co = Co; p.Ho = Ho; p.Wo = Wo; p.P = P;
  p.TH = pl.TH;
  p.nbands = (Ho + pl.TH - 1) / pl.TH;
  p.tpr = (Wo + pl.R - 1) / pl.R;
  p.tpu = std::min(p.tpr, kComputeWarps);
  p.ncolb = (p.tpr + p.tpu - 1) / p.tpu;
  p.ncob = ((Co + 31) / 32 + pl.CPL - 1) / pl.CPL;
  const long long units = (long long)N * p.nbands * p.ncolb * p.ncob;
  if (units >= (1ll << 31)) return SF_ERR_UNSUPPORTED;
  p.n_units = (int)units;
  const int grid = std::max(1, std::min(p.n_units, num_sms_current_device()));
  p.units_per_cta = (p.n_units + grid - 1) / grid;
  p.th_in = pl.th_in;
  p.slot_words = pl.slot_words;
  p.nstage = pl.nstage;
  p.w_cob_bytes = (uint32_t)((size_t)C * K * K * 32 * pl.CPL * dtype_size(wdt));
  p.w_off = pl.w_off;
  p.bar_off = pl.bar_off;
  const int grid_used = (p.n_units + p.units_per_cta - 1) / p.units_per_cta;
  return dispatch(lif, xdt, wdt, K, S, p, grid_used, pl, st);
}

}  // namespace
}  // namespace conv
}  // namespace sf

using namespace sf;
using namespace sf::conv;

extern "C" size_t sf_packed_weight_bytes(int32_t c_out, int32_t c_in, int32_t kernel, int32_t w_dst_dtype) {
  if (c_out <= 0 || c_in <= 0 || kernel <= 0) return 0;
  return (size_t)co_slices_padded(c_out) * 32 * c_in * kernel * kernel * dtype_size(w_dst_dtype);
}

extern "C" sf_status sf_pack_weights(const void* w_oihw, int32_t w_src_dtype, int32_t c_out, int32_t c_in,
                                     int32_t kernel, int32_t w_dst_dtype, void* w_packed, void* stream) {
  if (!w_oihw || !w_packed || c_out <= 0 || c_in <= 0 || kernel <= 0) return SF_ERR_INVALID_ARG;
  if (dtype_size(w_src_dtype) == 0) return SF_ERR_INVALID_ARG;
  if (w_dst_dtype != SF_DTYPE_F32 && w_dst_dtype != SF_DTYPE_BF16) return SF_ERR_UNSUPPORTED;
  const int slices = co_slices_padded(c_out);
  const int KK = kernel * kernel;
  const size_t total = (size_t)slices * c_in * KK * 32;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w_dst_dtype == SF_DTYPE_F32)
    pack_weights_kernel<float><<<blocks, 256, 0, st>>>(w_oihw, w_src_dtype, static_cast<float*>(w_packed), c_out,
                                                       c_in, KK, slices);
  else
    pack_weights_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        w_oihw, w_src_dtype, static_cast<__nv_bfloat16*>(w_packed), c_out, c_in, KK, slices);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

extern "C" size_t sf_sparse_conv2d_workspace_size(const sf_conv_desc* d) {
  if (!d || d->n <= 0 || d->c_in <= 0 || d->h <= 0 || d->w <= 0) return 0;
  return event_workspace_bytes(d->n, d->c_in, d->h * d->w);
}

extern "C" sf_status sf_sparse_conv2d(const void* x, const void* w_packed, const float* bias, void* y,
                                      const sf_conv_desc* d, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (!d) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  return run_conv(x, w_packed, d->has_bias ? bias : nullptr, y, nullptr, 1, d->n, d->c_in, d->h, d->w, d->c_out,
                  d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype, d->w_dtype, false, nullptr,
                  workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" size_t sf_fused_conv_lif_workspace_size(const sf_lif_desc* d) {
  if (!d || d->t_steps <= 0 || d->n <= 0 || d->c_in <= 0 || d->h <= 0 || d->w <= 0) return 0;
  return event_workspace_bytes((long long)d->t_steps * d->n, d->c_in, d->h * d->w);
}

extern "C" sf_status sf_fused_conv_lif(const void* x, const void* w_packed, const float* bias, float* v_inout,
                                       void* spikes_out, const sf_lif_desc* d, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (!d || !v_inout) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  if (!(d->tau > 0.f)) return SF_ERR_INVALID_ARG;
  if (d->kernel == 3 && d->stride != 1) return SF_ERR_UNSUPPORTED;
  return run_conv(x, w_packed, d->has_bias ? bias : nullptr, spikes_out, v_inout, d->t_steps, d->n, d->c_in, d->h,
                  d->w, d->c_out, d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype, d->w_dtype, true,
                  d, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
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
