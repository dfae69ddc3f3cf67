// Shared device helpers for the sm_100a kernels: dtype traits, mbarrier and
// bulk-copy (TMA, non-tensor form) wrappers with bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/sparseflow_b200.h"

namespace sf {

// Bounded spin limits. A wait that runs out sets an error word and returns
// instead of hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 24;

template <typename T> struct DT;
template <> struct DT<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ bool nonzero(float v) { return v != 0.0f; }
  static __device__ __forceinline__ uint32_t nz_bit(float v) { return (__float_as_uint(v) << 1) != 0u; }
  static __device__ __forceinline__ uint32_t not_one(float v) { return __float_as_uint(v) != 0x3f800000u; }
};
template <> struct DT<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ bool nonzero(__half v) {
    return (__half_as_ushort(v) & 0x7fffu) != 0u;
  }
  static __device__ __forceinline__ uint32_t nz_bit(__half v) { return (__half_as_ushort(v) & 0x7fffu) != 0u; }
  static __device__ __forceinline__ uint32_t not_one(__half v) { return __half_as_ushort(v) != 0x3c00u; }
};
template <> struct DT<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ bool nonzero(__nv_bfloat16 v) {
    return (__bfloat16_as_ushort(v) & 0x7fffu) != 0u;
  }
  static __device__ __forceinline__ uint32_t nz_bit(__nv_bfloat16 v) {
    return (__bfloat16_as_ushort(v) & 0x7fffu) != 0u;
  }
  static __device__ __forceinline__ uint32_t not_one(__nv_bfloat16 v) { return __bfloat16_as_ushort(v) != 0x3f80u; }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Returns false when the wait ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// As mbar_wait_bounded, but bounded by wall time (the %globaltimer
// nanosecond clock) rather than by the number of try_wait calls, each of
// which may suspend for a system-dependent time.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u && global_ns() - t0 > limit_ns) return false;
  }
}

// Contiguous global -> shared bulk copy completing on an mbarrier.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled tensor load (TMA) into shared memory, completing on an mbarrier.
// No multicast. The innermost coordinate c0 must keep c0 * element size a
// multiple of 16 bytes (callers pass 0).
__device__ __forceinline__ void tma_load_4d(void* dst_smem, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(dst_smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled tensor store (TMA) from shared memory, bulk-group completion.
// Elements outside the tensor are not written. c0 * element size must be a
// multiple of 16 bytes and stays >= 0.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src_smem, int c0, int c1, int c2,
                                             int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src_smem)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the shared-memory sources of all committed bulk stores have been read.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

inline size_t dtype_size(int32_t dt) {
  return dt == SF_DTYPE_F32 ? 4 : ((dt == SF_DTYPE_F16 || dt == SF_DTYPE_BF16) ? 2 : 0);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms_current_device();

// Opts a kernel in to the full 227 KB of dynamic shared memory once per
// (kernel, device) instead of on every launch (a driver call each time).
bool allow_max_smem(const void* kernel);

// Device-side choice between two kernel paths launched back to back: a
// sampling kernel writes a nonzero count to *count, and each gated kernel
// returns at entry unless the count selects it (side 1: count < thr; side 2:
// count >= thr). side 0: not gated.
struct Gate {
  const uint32_t* count;
  uint32_t thr;
  int side;
};
__device__ __forceinline__ bool gate_open(const Gate& g) {
  if (g.side == 0) return true;
  const uint32_t c = *reinterpret_cast<const volatile uint32_t*>(g.count);
  return g.side == 1 ? c < g.thr : c >= g.thr;
}

}  // namespace sf
