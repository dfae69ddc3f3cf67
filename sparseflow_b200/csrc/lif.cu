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

// Streaming (evict-first) vector loads and stores: x is read once and the
// spikes are written once, so neither should displace v or other data in L2.
template <typename T, int V>
__device__ __forceinline__ LVec<T, V> ld_stream(const LVec<T, V>* p) {
  if constexpr (sizeof(LVec<T, V>) == 16) {
    const float4 f = __ldcs(reinterpret_cast<const float4*>(p));
    return *reinterpret_cast<const LVec<T, V>*>(&f);
  } else if constexpr (sizeof(LVec<T, V>) == 8) {
    const float2 f = __ldcs(reinterpret_cast<const float2*>(p));
    return *reinterpret_cast<const LVec<T, V>*>(&f);
  } else {
    return *p;
  }
}
template <typename T, int V>
__device__ __forceinline__ void st_stream(LVec<T, V>* p, const LVec<T, V>& v) {
  if constexpr (sizeof(LVec<T, V>) == 16)
    __stcs(reinterpret_cast<float4*>(p), *reinterpret_cast<const float4*>(&v));
  else if constexpr (sizeof(LVec<T, V>) == 8)
    __stcs(reinterpret_cast<float2*>(p), *reinterpret_cast<const float2*>(&v));
  else
    *p = v;
}

// Steps whose x is loaded ahead of their updates: the loads of a group do not
// depend on the membrane state, so all of them are in flight together.
constexpr int kLifPrefetch = 8;

template <typename XT, typename ST, int VEC>
__global__ void __launch_bounds__(256) lif_multistep_kernel(const XT* __restrict__ x, float* __restrict__ v,
                                                            ST* __restrict__ s, long long numel, int T,
                                                            LifParams q) {
  const long long nvec = numel / VEC;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    LVec<float, VEC> vv = reinterpret_cast<const LVec<float, VEC>*>(v)[i];
    for (int t0 = 0; t0 < T; t0 += kLifPrefetch) {
      LVec<XT, VEC> xb[kLifPrefetch];
#pragma unroll
      for (int k = 0; k < kLifPrefetch; ++k)
        if (t0 + k < T) xb[k] = ld_stream(reinterpret_cast<const LVec<XT, VEC>*>(x + (size_t)(t0 + k) * numel) + i);
#pragma unroll
      for (int k = 0; k < kLifPrefetch; ++k) {
        if (t0 + k < T) {
          LVec<ST, VEC> sv;
#pragma unroll
          for (int e = 0; e < VEC; ++e) sv.v[e] = DT<ST>::from_f(lif_update(vv.v[e], DT<XT>::to_f(xb[k].v[e]), q));
          st_stream(reinterpret_cast<LVec<ST, VEC>*>(s + (size_t)(t0 + k) * numel) + i, sv);
        }
      }
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
  // One vector per thread where the grid allows (no tail of uneven loop trips).
  const long long blocks = std::min<long long>((nvec + 255) / 256, 1ll << 30);
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
