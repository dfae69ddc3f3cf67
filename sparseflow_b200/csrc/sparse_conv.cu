// C-ABI entry points of the sparse convolution (stage 1 event extraction +
// stage 2 gather) and of the fused conv+LIF kernel: argument checks, launch
// planning, weight packing. The kernels are in events.cu and conv_kernel.cuh.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>
#include <cudaTypedefs.h>
#include "conv_kernel.cuh"
#include "policy.cuh"
#include "events.cuh"
#include "lif.cuh"
#include "conv3x3_tc.cuh"

namespace sf {
namespace pwtc {
sf_status run_pointwise_tc(const void* x, const void* w_packed, const float* bias, void* y, uint32_t* err, int N,
                           int C, int H, int W, int Co, int xdt, int wdt, cudaStream_t st,
                           const unsigned long long* masks = nullptr);
}  // namespace pwtc
namespace pw {
sf_status run_pointwise(const void* x, const void* w_packed, const float* bias, void* y, int N, int C, int H,
                        int W, int Co, int Ho, int Wo, int S, int xdt, int wdt, cudaStream_t st);
}  // namespace pw
namespace conv {
namespace {

// Set when a bounded wait in the conv kernel runs out (read by
// sf_sparse_conv2d_status); a static device word, so no allocation is needed.
__device__ uint32_t g_conv_error = 0;
// All-binary flags for convolutions whose events come from a fused conv + LIF
// (spikes are 0/1 by construction); zero-initialised when the module loads.
constexpr int kZeroFlags = 65536;
__device__ uint32_t g_zero_flags[kZeroFlags];

// [co][ci][kk] (any dtype) -> [block][ci][kk][32][cpl] (fp32 or bf16), zero padded.
template <typename WT>
__global__ void pack_weights_kernel(const void* __restrict__ w, int src_dtype, WT* __restrict__ out, int Co, int Ci,
                                    int KK, int blocks, int cpl) {
  const size_t total = (size_t)blocks * Ci * KK * 32 * cpl;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % cpl);
    size_t r = i / cpl;
    const int l = (int)(r & 31);
    r >>= 5;
    const int t = (int)(r % KK);
    r /= KK;
    const int ci = (int)(r % Ci);
    const int b = (int)(r / Ci);
    const int co = (b * cpl + j) * 32 + l;
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

// Tuning overrides for development builds only (-DSF_DEV_KNOBS): they pin
// plan choices from the environment. Release builds read no environment.
int dev_knob(const char* name) {
#ifdef SF_DEV_KNOBS
  const char* v = getenv(name);
  return v ? atoi(v) : 0;
#else
  (void)name;
  return 0;
#endif
}

// Launch plan: 32-channel slices per lane (CPL, fixed by the weight packing),
// row-segment length R, band height TH (one row segment per compute warp),
// mask stages, and whether a block of packed weights lives in shared memory.
// Development builds can pin these choices (dev_knob).
bool make_plan(int K, int S, int C, int W, int Co, int Ho, int Wo, int nw, int wsz, int esz, bool y_tma_ok,
               bool lif, Plan& pl) {
  const int B = lif ? 1 : kRowsPerWarp;  // output rows per compute warp (matches the kernel)
  const int force_th = dev_knob("SF_CONV_TH"), force_ns = dev_knob("SF_CONV_NSTAGE");
  const int bar_bytes = (2 * kMaxStages + 1) * 8;
  const int cpl = weight_block_cpl(C, K, Co, wsz);
  const size_t w_bytes = (size_t)C * K * K * 32 * cpl * wsz;
  const bool ws_ok = w_bytes <= kWsmemMax && dev_knob("SF_CONV_NO_WSMEM") == 0;
  const int R = cpl == 4 ? 4 : 8;
  // TMA tensor stores need 16-byte row pitch and 16-byte tile rows.
  // Off unless SF_CONV_TMA_STORE=1: plain sector-complete stores measured faster.
  const bool tma_ok = y_tma_ok && (Wo * esz) % 16 == 0 && (R * esz) % 16 == 0 && dev_knob("SF_CONV_TMA_STORE") == 1;
  for (int combo = 0; combo < 4; ++combo) {
    const int wsmem = (combo < 2) ? (ws_ok ? 1 : -1) : 0;  // prefer weights in smem, then TMA stores
    const int tma = (combo % 2 == 0) ? (tma_ok ? 1 : -1) : 0;
    if (wsmem < 0 || tma < 0) continue;
    const int tpr = (Wo + R - 1) / R;
    const int tpu = std::min(tpr, kComputeWarps);
    const int w_region = wsmem ? (int)(((w_bytes + 127) / 128) * 128) : 0;
    const int stg_region = tma ? kComputeWarps * 32 * cpl * R * esz : 0;
    for (int TH = std::min(Ho, B * (kComputeWarps / tpu)); TH >= 1; --TH) {
      if (force_th && TH != force_th) continue;
      const int th_in = (TH - 1) * S + K;
      // 128-byte aligned stages keep every region after them 128-byte aligned.
      const int slot_words = ((th_in * W * nw + 2) + 15) & ~15;
      const int stage_bytes = slot_words * 8;
      const long long fixed = (long long)w_region + stg_region + bar_bytes;
      if (fixed + 2ll * stage_bytes > kSmemLimit) continue;
      int nstage = (int)std::min<long long>(kMaxStages, (kSmemLimit - fixed) / stage_bytes);
      if (force_ns) {
        if (force_ns > nstage) continue;
        nstage = force_ns;
      }
      pl.CPL = cpl;
      pl.R = R;
      pl.wsmem = wsmem;
      pl.tma_store = tma;
      pl.TH = TH;
      pl.th_in = th_in;
      pl.nstage = nstage;
      pl.slot_words = slot_words;
      pl.w_off = nstage * stage_bytes;
      pl.stg_off = pl.w_off + w_region;
      pl.bar_off = pl.stg_off + stg_region;
      pl.smem = pl.bar_off + bar_bytes;
      return true;
    }
  }
  return false;
}

int g_num_sms[64] = {0};

}  // namespace
}  // namespace conv

bool allow_max_smem(const void* kernel) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
    return false;
  done.insert({kernel, dev});
  return true;
}

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

sf_status dispatch(int mode, int xdt, int wdt, int K, int S, const ConvParams& p, const CUtensorMap& ym, int grid,
                   const Plan& pl, cudaStream_t st) {
  if (xdt == SF_DTYPE_F32) return dispatch_f32(mode, wdt, K, S, p, ym, grid, pl, st);
  if (xdt == SF_DTYPE_F16) return dispatch_f16(mode, wdt, K, S, p, ym, grid, pl, st);
  if (xdt == SF_DTYPE_BF16) return dispatch_bf16(mode, wdt, K, S, p, ym, grid, pl, st);
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

// y viewed as 4-D (W_out, H_out, C_out, T*N), box (R, 1, 32*CPL, 1).
sf_status encode_y_map(CUtensorMap* m, void* y, int xdt, int Wo, int Ho, int Co, long long nimg, int R, int cpl) {
  auto fn = tensor_map_encoder();
  if (!fn) return SF_ERR_CUDA;
  const CUtensorMapDataType dt = xdt == SF_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : xdt == SF_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t esz = dtype_size(xdt);
  const cuuint64_t dims[4] = {(cuuint64_t)Wo, (cuuint64_t)Ho, (cuuint64_t)Co, (cuuint64_t)nimg};
  const cuuint64_t strides[3] = {Wo * esz, (cuuint64_t)Ho * Wo * esz, (cuuint64_t)Co * Ho * Wo * esz};
  const cuuint32_t box[4] = {(cuuint32_t)R, 1u, (cuuint32_t)(32 * cpl), 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUresult r = fn(m, dt, 4, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SF_OK : SF_ERR_CUDA;
}

sf_status check_geometry(int T, int N, int C, int H, int W, int Co, int Ho, int Wo, int K, int S, int P, int xdt,
                         int wdt) {
  if (T <= 0 || N <= 0 || C <= 0 || H <= 0 || W <= 0 || Co <= 0 || Ho <= 0 || Wo <= 0) return SF_ERR_INVALID_ARG;
  if (!((K == 1 && S == 1 && P == 0) || (K == 1 && S == 2 && P == 0) || (K == 3 && S == 1 && P == 1) ||
        (K == 3 && S == 2 && P == 1)))
    return SF_ERR_UNSUPPORTED;
  if ((H + 2 * P - K) / S + 1 != Ho || (W + 2 * P - K) / S + 1 != Wo) return SF_ERR_INVALID_ARG;
  if (dtype_size(xdt) == 0 || (wdt != SF_DTYPE_F32 && wdt != SF_DTYPE_BF16)) return SF_ERR_INVALID_ARG;
  if ((long long)T * N >= 65536) return SF_ERR_UNSUPPORTED;
  return SF_OK;
}

// Bytes of the gather layout alone; the tensor-core section (3x3 layers the
// tcgen05 kernel takes) follows it at the next 256-byte boundary.
size_t gather_bytes(int c_out, int c_in, int kernel, int wsz) {
  const int cpl = weight_block_cpl(c_in, kernel, c_out, wsz);
  return (size_t)weight_blocks(c_out, cpl) * cpl * 32 * c_in * kernel * kernel * wsz;
}
size_t tc_section_offset(int c_out, int c_in, int kernel, int wsz) {
  return (gather_bytes(c_out, c_in, kernel, wsz) + 255) & ~(size_t)255;
}

// Device address of g_conv_error for the current device, looked up once per
// device (the host-side symbol is not a device address).
uint32_t* conv_error_word() {
  static uint32_t* cache[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_conv_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<uint32_t*>(ptr);
  }
  return cache[dev];
}

// A second stream of the calling thread on the current device, with a fork
// and a join event: the two gated routes of a 3x3 call run side by side, so
// the kernels of the route the gate closes overlap the open route's instead
// of queueing behind them. Created once per thread and device.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
// Null when there is none yet and `may_create` is false (a stream being
// captured into a CUDA graph: creating streams there is not allowed in every
// capture mode).
const SideStream* side_stream(bool may_create) {
  thread_local SideStream cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  SideStream& ss = cache[dev];
  if (ss.stream == nullptr) {
    if (!may_create) return nullptr;
    SideStream n;
    if (cudaStreamCreateWithFlags(&n.stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    if (cudaEventCreateWithFlags(&n.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&n.join, cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
    ss = n;
  }
  return &ss;
}

// Spike density below which the gather kernel beats the tensor-core kernel
// for 3x3/s1 layers of C_in input channels (0: the tensor cores always win).
// Crossovers measured with both paths forced (1024 images of 14x14, 28x28
// and 56x56, one B200): C_in 64 none (tensor cores 2.8-4.5x cuDNN at every
// density); C_in 128 near 0.4 % (0.3 % at 28x28, 0.7 % at 14x14); C_in 256
// near 0.8 %; C_in 512 near 1 %.
double tc3_min_density(int C) {
  if (C <= c3tc::kTcResidentMaxC) return 0.0;
  if (C <= 160) return 0.004;
  return C <= 320 ? 0.008 : 0.01;
}
// The same for the fused conv + LIF: the tensor-core route writes the
// preactivations and runs the LIF over them in place, 8 bytes per output
// element more than the fused gather kernel; emitting the next layer's event
// masks costs the gather kernel more than the LIF kernel. Crossovers (T16
// N64, one B200, both routes forced, ms gather / tensor cores):
//   C_in 64 56x56:  masks 0.735 / 0.735 at 0.1 %, 0.809 / 0.734 at 0.3 %;
//                   none  0.646 / 0.666 at 0.1 %, 0.705 / 0.664 at 0.3 %
//   C_in 128 28x28: masks 0.649 / 0.668 at 0.3 %, 0.688 / 0.667 at 0.4 %;
//                   none  0.561 / 0.590 at 0.3 %, 0.592 / 0.590 at 0.4 %,
//                         0.624 / 0.589 at 0.5 % (LIF in the epilogue)
//   C_in 256 14x14: masks 0.553 / 0.550 at 0.6 %; none 0.548 / 0.528 at 0.6 %
double tc3_lif_min_density(int C, bool masks) {
  if (C <= c3tc::kTcResidentMaxC) return masks ? 0.0 : 0.002;
  if (C <= 160) return masks ? 0.0035 : 0.004;
  return C <= 320 ? 0.0055 : 0.01;
}
constexpr int kDensitySamples = kMaxDensitySamples;
constexpr size_t kMasksOrXWorkspace = 256;  // the sampled count of sf_sparse_conv2d_masks_or_x

// Stage 1 + stage 2 for T*N images; the LIF variant when lif is set.
// masks_in: events of x precomputed by a fused conv + LIF (binary spikes;
// x itself is then not read, or may be null, except by the tensor-core 3x3
// route when x is given too). mask_out: LIF only, the output spikes' events.
sf_status run_conv(const void* x, const void* w_packed, const float* bias, void* y, float* v, int T, int N, int C,
                   int H, int W, int Co, int Ho, int Wo, int K, int S, int P, int xdt, int wdt, bool lif,
                   const sf_lif_desc* lifd, void* workspace, size_t ws_bytes, cudaStream_t st,
                   const unsigned long long* masks_in = nullptr, uint32_t* mask_out = nullptr) {
  sf_status s = check_geometry(T, N, C, H, W, Co, Ho, Wo, K, S, P, xdt, wdt);
  if (s != SF_OK) return s;
  if ((!x && !masks_in) || !w_packed || !y) return SF_ERR_INVALID_ARG;
  if (!workspace && !masks_in) return SF_ERR_WORKSPACE;
  if (!aligned16(w_packed)) return SF_ERR_ALIGNMENT;
  // 1x1 stride 1: tcgen05 GEMM tiles over x streamed once (pointwise_tc.cu).
  // With the spikes' event masks handed over (masks_in), the same kernel
  // builds A from the masks and never reads x: with bf16 weights (one digit
  // plane) that beats the gather kernel from the masks (C2 cell: 0.23-0.25 ms
  // against 0.26-0.27 ms); with fp32 weights (three bf16 planes) it does not
  // (0.33 against 0.26 ms), so those run the gather kernel.
  if (!lif && K == 1 && S == 1 && P == 0 && policy(SF_POLICY_CONV1X1_PATH) == 0 &&
      !(masks_in && wdt == SF_DTYPE_F32)) {
    uint32_t* err = nullptr;
    if ((err = conv_error_word()) == nullptr) return SF_ERR_CUDA;
    s = pwtc::run_pointwise_tc(x, w_packed, bias, y, err, T * N, C, H, W, Co, xdt, wdt, st, masks_in);
    if (s != SF_ERR_UNSUPPORTED) return s;
  }
  // 3x3 stride 1: integer tcgen05 implicit GEMM over x streamed once
  // (conv3x3_tc.cu), unless the policy asks for the gather kernel. Its cost
  // does not depend on the spike density; the gather kernel's does. For
  // C_in <= 64 the tensor-core kernel is faster at every density; above, the
  // gather kernel wins on sparse enough inputs, so a sampled nonzero count
  // picks one of the two paths on the device (both are launched; the other
  // returns at entry). The fused conv + LIF makes the same choice at its own
  // densities.
  const int pol3 = (int)policy(SF_POLICY_CONV3X3_PATH);
  Gate gate{nullptr, 0u, 0};
  bool tc_after = false;
  // With masks handed over and x too (sf_sparse_conv2d_masks_or_x), the gate
  // picks the gather kernel from the masks or the tensor cores from x.
  const bool tc_shape = (!masks_in || x) && K == 3 && S == 1 && P == 1 && pol3 != 1 && c3tc::tc3_packs(Co, C, K) &&
                        (wdt == SF_DTYPE_F32 || wdt == SF_DTYPE_BF16) &&
                        c3tc::tc3_supported(T * N, C, H, W, Co);
  // Fused conv + LIF: the tensor-core kernel with the multi-step LIF in its
  // epilogue; when the caller wants the spikes' event masks, the kernel
  // writes the fp32 preactivations into the spike buffer and the multi-step
  // LIF with mask emission runs over them in place (v, spikes and event masks
  // as the fused gather kernel writes them). fp32 spikes only: a 16-bit
  // buffer would round the preactivations.
  const bool lif_tc = lif && tc_shape && xdt == SF_DTYPE_F32;
  auto tc_then_lif = [&](const Gate& g, cudaStream_t sx) -> sf_status {
    const int wsz = (int)dtype_size(wdt);
    const void* section = static_cast<const char*>(w_packed) + tc_section_offset(Co, C, K, wsz);
    const int epi = (int)policy(SF_POLICY_LIF_TC_EPILOGUE);
    if (lif && !mask_out && epi != 1) {
      // One launch: the LIF runs in the tensor-core kernel's epilogue (unit
      // by unit over t = 0..T-1, the membrane read and written by the same
      // thread each step, kept in L2 between steps), so the preactivations
      // never reach memory.
      const c3tc::TcLif tl{T, v, lifd->tau, lifd->v_threshold, lifd->v_reset, lifd->hard_reset, lifd->decay_input,
                           epi == 2};
      sf_status r = c3tc::run_conv3x3_tc(x, w_packed, weight_block_cpl(C, K, Co, wsz), section, bias, y,
                                         conv_error_word(), T * N, C, H, W, Co, xdt, wdt, sx, g, &tl);
      if (r != SF_ERR_UNSUPPORTED) return r;
    }
    sf_status r = c3tc::run_conv3x3_tc(x, w_packed, weight_block_cpl(C, K, Co, wsz), section, bias, y,
                                       conv_error_word(), T * N, C, H, W, Co, xdt, wdt, sx, g);
    if (r != SF_OK || !lif) return r;
    return lif_after_conv(static_cast<const float*>(y), v, static_cast<float*>(y), mask_out, T, N, Co, Ho * Wo,
                          lifd->tau, lifd->v_threshold, lifd->v_reset, lifd->hard_reset, lifd->decay_input, g, sx);
  };
  if ((!lif && tc_shape) || lif_tc) {
    if (conv_error_word() == nullptr) return SF_ERR_CUDA;
    const double rho = lif ? tc3_lif_min_density(C, mask_out != nullptr) : tc3_min_density(C);
    if (pol3 == 2 || rho <= 0.0) return tc_then_lif(Gate{nullptr, 0u, 0}, st);
    const long long nimg = (long long)T * N;
    uint32_t* count = nullptr;
    if (masks_in) {
      if (!workspace || ws_bytes < kMasksOrXWorkspace) return SF_ERR_WORKSPACE;
      count = static_cast<uint32_t*>(workspace);
    } else {
      if (ws_bytes < event_workspace_bytes(nimg, C, H * W)) return SF_ERR_WORKSPACE;
      count = event_count_word(workspace, nimg, C, H * W);
    }
    s = sample_nonzeros(x, xdt, nimg * C * H * W, kDensitySamples, count, st);
    if (s != SF_OK) return s;
    gate = Gate{count, (uint32_t)std::ceil(rho * kDensitySamples), 1};
    tc_after = true;
  }
  // The gather path (mask pass + gather kernel), or the one-pass 1x1/s2
  // kernel; gated by `gate` when the tensor-core kernel follows.
  auto gather_path = [&]() -> sf_status {
  sf_status s = SF_OK;
  // 1x1 stride 2: one pass over x with masks built in shared memory
  // (pointwise.cu). For stride 1 that kernel measured slower than the two
  // stages (0.74 vs 0.54 ms on the C2 cell; both issue-bound), so it runs
  // only when the SF_POLICY_CONV1X1_PATH policy asks for it.
  if (!lif && !masks_in && K == 1 && (S == 2 || policy(SF_POLICY_CONV1X1_PATH) == 2)) {
    s = pw::run_pointwise(x, w_packed, bias, y, T * N, C, H, W, Co, Ho, Wo, S, xdt, wdt, st);
    if (s != SF_ERR_UNSUPPORTED) return s;
  }
  if (K == 1 && S != 1) return SF_ERR_UNSUPPORTED;
  const int nw = (C + 63) / 64;
  Plan pl;
  const bool y_tma_ok = aligned16(y) && tensor_map_encoder() != nullptr;
  if (!make_plan(K, S, C, W, Co, Ho, Wo, nw, (int)dtype_size(wdt), (int)dtype_size(xdt), y_tma_ok, lif, pl))
    return SF_ERR_UNSUPPORTED;

  EventBuffers ev;
  if (masks_in) {
    if ((long long)T * N > kZeroFlags) return SF_ERR_UNSUPPORTED;
    ev.masks = const_cast<unsigned long long*>(masks_in);
    ev.nw = nw;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ev.flags), g_zero_flags) != cudaSuccess) return SF_ERR_CUDA;
  } else {
    s = extract_events(x, xdt, (long long)T * N, C, H * W, workspace, ws_bytes, ev, st, gate);
    if (s != SF_OK) return s;
  }
  if (mask_out && Co % 64 != 0) {
    // Halves past C_out are never written by the kernel.
    const size_t mbytes = (size_t)T * N * Ho * Wo * ((Co + 63) / 64) * 8;
    if (cudaMemsetAsync(mask_out, 0, mbytes, st) != cudaSuccess) return SF_ERR_CUDA;
  }

  ConvParams p;
  memset(&p, 0, sizeof(p));
  p.x = x;
  p.wp = w_packed;
  p.bias = bias;
  p.y = y;
  p.v = v;
  if ((p.err = conv_error_word()) == nullptr) return SF_ERR_CUDA;
  p.masks = ev.masks;
  p.flags = ev.flags;
  p.mask_out = mask_out;
  p.nw_out = (Co + 63) / 64;
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
  p.stg_off = pl.stg_off;
  p.bar_off = pl.bar_off;
  p.tma_store = pl.tma_store;
  CUtensorMap ym;
  memset(&ym, 0, sizeof(ym));
  if (pl.tma_store) {
    s = encode_y_map(&ym, y, xdt, Wo, Ho, Co, (long long)T * N, pl.R, pl.CPL);
    if (s != SF_OK) return s;
  }
  const int grid_used = (p.n_units + p.units_per_cta - 1) / p.units_per_cta;
  int mode = 0;
  if (lif) {
    int e = 0;
    const float m = std::frexp(p.tau, &e);
    const bool pow2 = m == 0.5f && e > -125 && e < 126;  // tau = 2^(e-1), 1/tau a normal float
    p.inv_tau = pow2 ? 1.f / p.tau : 0.f;
    mode = (mask_out ? 2 : 1) + (pow2 ? 2 : 0);
  }
  p.gate = gate;
  return dispatch(mode, xdt, wdt, K, S, p, ym, grid_used, pl, st);
  };
  if (!tc_after) return gather_path();
  // Both routes, each gated: the gather route on the caller's stream, the
  // tensor-core route (and LIF) on the side stream between a fork after the
  // sampler and a join before whatever the caller queues next.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return SF_ERR_CUDA;
  const SideStream* side = side_stream(cap == cudaStreamCaptureStatusNone);
  if (side == nullptr) {
    // No side stream: both routes in order on the caller's stream.
    s = gather_path();
    return tc_then_lif(s == SF_OK ? Gate{gate.count, gate.thr, 2} : Gate{nullptr, 0u, 0}, st);
  }
  if (cudaEventRecord(side->fork, st) != cudaSuccess || cudaStreamWaitEvent(side->stream, side->fork, 0) != cudaSuccess)
    return SF_ERR_CUDA;
  s = gather_path();
  // Gated too when the gather route launched; ungated (it alone computes y)
  // when that route could not.
  const sf_status r =
      tc_then_lif(s == SF_OK ? Gate{gate.count, gate.thr, 2} : Gate{nullptr, 0u, 0}, side->stream);
  if (cudaEventRecord(side->join, side->stream) != cudaSuccess || cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess)
    return SF_ERR_CUDA;
  return r;
}

}  // namespace
}  // namespace conv
}  // namespace sf

using namespace sf;
using namespace sf::conv;

extern "C" size_t sf_packed_weight_bytes(int32_t c_out, int32_t c_in, int32_t kernel, int32_t w_dst_dtype) {
  if (c_out <= 0 || c_in <= 0 || kernel <= 0) return 0;
  const int wsz = (int)dtype_size(w_dst_dtype);
  if (wsz == 0) return 0;
  if (c3tc::tc3_packs(c_out, c_in, kernel))
    return tc_section_offset(c_out, c_in, kernel, wsz) + c3tc::tc3_section_bytes(c_out, c_in);
  return gather_bytes(c_out, c_in, kernel, wsz);
}

extern "C" sf_status sf_pack_weights(const void* w_oihw, int32_t w_src_dtype, int32_t c_out, int32_t c_in,
                                     int32_t kernel, int32_t w_dst_dtype, void* w_packed, void* stream) {
  if (!w_oihw || !w_packed || c_out <= 0 || c_in <= 0 || kernel <= 0) return SF_ERR_INVALID_ARG;
  if (dtype_size(w_src_dtype) == 0) return SF_ERR_INVALID_ARG;
  if (w_dst_dtype != SF_DTYPE_F32 && w_dst_dtype != SF_DTYPE_BF16) return SF_ERR_UNSUPPORTED;
  const int cpl = weight_block_cpl(c_in, kernel, c_out, (int)dtype_size(w_dst_dtype));
  const int blocks_w = weight_blocks(c_out, cpl);
  const int KK = kernel * kernel;
  const size_t total = (size_t)blocks_w * c_in * KK * 32 * cpl;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w_dst_dtype == SF_DTYPE_F32)
    pack_weights_kernel<float><<<blocks, 256, 0, st>>>(w_oihw, w_src_dtype, static_cast<float*>(w_packed), c_out,
                                                       c_in, KK, blocks_w, cpl);
  else
    pack_weights_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        w_oihw, w_src_dtype, static_cast<__nv_bfloat16*>(w_packed), c_out, c_in, KK, blocks_w, cpl);
  if (cudaGetLastError() != cudaSuccess) return SF_ERR_CUDA;
  if (c3tc::tc3_packs(c_out, c_in, kernel)) {
    const size_t off = tc_section_offset(c_out, c_in, kernel, (int)dtype_size(w_dst_dtype));
    return c3tc::tc3_pack(w_oihw, w_src_dtype, c_out, c_in, static_cast<char*>(w_packed) + off, st);
  }
  return SF_OK;
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
                                       void* spikes_out, void* spike_masks_out, const sf_lif_desc* d,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!d || !v_inout) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  if (!(d->tau > 0.f)) return SF_ERR_INVALID_ARG;
  if (d->kernel == 3 && d->stride != 1) return SF_ERR_UNSUPPORTED;
  if (spike_masks_out && (reinterpret_cast<uintptr_t>(spike_masks_out) & 7u) != 0) return SF_ERR_ALIGNMENT;
  return run_conv(x, w_packed, d->has_bias ? bias : nullptr, spikes_out, v_inout, d->t_steps, d->n, d->c_in, d->h,
                  d->w, d->c_out, d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype, d->w_dtype, true,
                  d, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), nullptr,
                  static_cast<uint32_t*>(spike_masks_out));
}

extern "C" size_t sf_event_masks_bytes(int64_t n_images, int32_t channels, int32_t h, int32_t w) {
  if (n_images <= 0 || channels <= 0 || h <= 0 || w <= 0) return 0;
  return (size_t)n_images * h * w * ((channels + 63) / 64) * 8;
}

extern "C" sf_status sf_sparse_conv2d_from_masks(const void* event_masks, const void* w_packed, const float* bias,
                                                 void* y, const sf_conv_desc* d, void* stream) {
  if (!d || !event_masks) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(event_masks) & 15u) != 0) return SF_ERR_ALIGNMENT;
  return run_conv(nullptr, w_packed, d->has_bias ? bias : nullptr, y, nullptr, 1, d->n, d->c_in, d->h, d->w,
                  d->c_out, d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype, d->w_dtype, false,
                  nullptr, nullptr, 0, static_cast<cudaStream_t>(stream),
                  static_cast<const unsigned long long*>(event_masks));
}

extern "C" size_t sf_sparse_conv2d_masks_or_x_workspace_size(void) { return kMasksOrXWorkspace; }

extern "C" sf_status sf_sparse_conv2d_masks_or_x(const void* x, const void* event_masks, const void* w_packed,
                                                 const float* bias, void* y, const sf_conv_desc* d, void* workspace,
                                                 size_t workspace_bytes, void* stream) {
  if (!d || !event_masks || !x) return SF_ERR_INVALID_ARG;
  if (d->has_bias && !bias) return SF_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(event_masks) & 15u) != 0) return SF_ERR_ALIGNMENT;
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 3u) != 0) return SF_ERR_ALIGNMENT;
  return run_conv(x, w_packed, d->has_bias ? bias : nullptr, y, nullptr, 1, d->n, d->c_in, d->h, d->w, d->c_out,
                  d->h_out, d->w_out, d->kernel, d->stride, d->padding, d->x_dtype, d->w_dtype, false, nullptr,
                  workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                  static_cast<const unsigned long long*>(event_masks));
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
