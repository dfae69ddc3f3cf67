// Multi-step LIF neuron over [T, numel] (HBM-bound elementwise).
//
// The update is the reference's multi-step LIF (Ops/sparse_fused_conv_lif.py:
// 271-293, spikingjelly LIFNode with step_mode 'm'):
//   decay_input: h = v + (x - (v - v_reset)) / tau
//   otherwise:   h = v - (v - v_reset) / tau + x
//   spike = h >= v_threshold
//   hard reset:  v = spike ? v_reset : h;   soft reset: v = h - spike * v_threshold
// with the same operation order and IEEE division, so spikes equal the
// PyTorch formula bit for bit. A torch LIFNode runs about eight elementwise
// kernels per step and moves v through HBM every step; here each thread owns
// VEC elements, keeps their v in registers across all T steps, and reads x /
// writes spikes once: bytes = T * numel * (|x| + |spike|) + 8 * numel.
#include "common.cuh"

namespace sf {
namespace {

template <typename T, int V>
struct alignas(sizeof(T) * V) LVec {
  T v[V];
};

struct LifParams {
  float tau, vth, vr;
  int hard, decay_input;
};

__device__ __forceinline__ float lif_update(float& v, float x, const LifParams& q) {
  float h;
  if (q.decay_input)
    h = v + (x - (v - q.vr)) / q.tau;
  else
    h = v - (v - q.vr) / q.tau + x;
  const bool s = h >= q.vth;
  v = q.hard ? (s ? q.vr : h) : (h - (s ? q.vth : 0.f));
  return s ? 1.f : 0.f;
}

template <typename XT, typename ST, int VEC>
__global__ void __launch_bounds__(256) lif_multistep_kernel(const XT* __restrict__ x, float* __restrict__ v,
                                                            ST* __restrict__ s, long long numel, int T,
                                                            LifParams q) {
  const long long nvec = numel / VEC;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    LVec<float, VEC> vv = reinterpret_cast<const LVec<float, VEC>*>(v)[i];
    // Loads of step t+1 do not depend on step t's state: unrolling keeps
    // several in flight.
#pragma unroll 4
    for (int t = 0; t < T; ++t) {
      const LVec<XT, VEC> xv = reinterpret_cast<const LVec<XT, VEC>*>(x + (size_t)t * numel)[i];
      LVec<ST, VEC> sv;
#pragma unroll
      for (int e = 0; e < VEC; ++e) sv.v[e] = DT<ST>::from_f(lif_update(vv.v[e], DT<XT>::to_f(xv.v[e]), q));
      reinterpret_cast<LVec<ST, VEC>*>(s + (size_t)t * numel)[i] = sv;
    }
    reinterpret_cast<LVec<float, VEC>*>(v)[i] = vv;
  }
}

template <typename XT, typename ST>
sf_status launch(const void* x, float* v, void* s, long long numel, int T, const LifParams& q, cudaStream_t st) {
  const bool vec = numel % 4 == 0 && aligned16(v) && (reinterpret_cast<uintptr_t>(x) % (4 * sizeof(XT))) == 0 &&
                   (reinterpret_cast<uintptr_t>(s) % (4 * sizeof(ST))) == 0;
  const int V = vec ? 4 : 1;
  const long long nvec = numel / V;
  const long long blocks = std::min<long long>((nvec + 255) / 256, (long long)num_sms_current_device() * 8);
  if (blocks <= 0) return SF_OK;
  if (vec)
    lif_multistep_kernel<XT, ST, 4><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const XT*>(x), v,
                                                                     static_cast<ST*>(s), numel, T, q);
  else
    lif_multistep_kernel<XT, ST, 1><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const XT*>(x), v,
                                                                     static_cast<ST*>(s), numel, T, q);
  return cudaGetLastError() == cudaSuccess ? SF_OK : SF_ERR_CUDA;
}

template <typename XT>
sf_status dispatch_s(int sdt, const void* x, float* v, void* s, long long numel, int T, const LifParams& q,
                     cudaStream_t st) {
  switch (sdt) {
    case SF_DTYPE_F32: return launch<XT, float>(x, v, s, numel, T, q, st);
    case SF_DTYPE_F16: return launch<XT, __half>(x, v, s, numel, T, q, st);
    case SF_DTYPE_BF16: return launch<XT, __nv_bfloat16>(x, v, s, numel, T, q, st);
  }
  return SF_ERR_INVALID_ARG;
}

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" sf_status sf_lif_multistep(const void* x, float* v_inout, void* spikes_out, const sf_lif_ms_desc* d,
                                      void* stream) {
  if (!d || !x || !v_inout || !spikes_out) return SF_ERR_INVALID_ARG;
  if (d->numel < 0 || d->t_steps < 0 || !(d->tau != 0.f)) return SF_ERR_INVALID_ARG;
  if (dtype_size(d->x_dtype) == 0 || dtype_size(d->s_dtype) == 0) return SF_ERR_INVALID_ARG;
  if (d->numel == 0 || d->t_steps == 0) return SF_OK;
  LifParams q;
  q.tau = d->tau;
  q.vth = d->v_threshold;
  q.vr = d->hard_reset ? d->v_reset : 0.f;
  q.hard = d->hard_reset;
  q.decay_input = d->decay_input;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (d->x_dtype) {
    case SF_DTYPE_F32: return dispatch_s<float>(d->s_dtype, x, v_inout, spikes_out, d->numel, d->t_steps, q, st);
    case SF_DTYPE_F16: return dispatch_s<__half>(d->s_dtype, x, v_inout, spikes_out, d->numel, d->t_steps, q, st);
    case SF_DTYPE_BF16:
      return dispatch_s<__nv_bfloat16>(d->s_dtype, x, v_inout, spikes_out, d->numel, d->t_steps, q, st);
  }
  return SF_ERR_INVALID_ARG;
}

// ---------------------------------------------------------------------------
// Bounded-wait self test (diagnostics): an mbarrier that never completes.
// ---------------------------------------------------------------------------
namespace sf {
namespace {
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, uint32_t* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none is ever made
    fence_mbar_init();
    *out = mbar_wait_ns(&bar, 0u, limit_ns) ? 1u : 2u;  // 2: gave up, as it must
  }
}
}  // namespace
}  // namespace sf

extern "C" sf_status sf_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* d = nullptr;
  uint32_t h = 0;
  if (cudaMallocAsync(reinterpret_cast<void**>(&d), 4, st) != cudaSuccess) return SF_ERR_CUDA;
  sf::bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns, d);
  const bool ok = cudaGetLastError() == cudaSuccess &&
                  cudaMemcpyAsync(&h, d, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
                  cudaFreeAsync(d, st) == cudaSuccess && cudaStreamSynchronize(st) == cudaSuccess;
  if (!ok) return SF_ERR_CUDA;
  return h == 2u ? SF_ERR_DEVICE_TIMEOUT : (h == 1u ? SF_OK : SF_ERR_CUDA);
}
