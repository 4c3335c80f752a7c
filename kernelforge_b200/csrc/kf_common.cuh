// Shared device/host helpers for the sm_100a kernels of kernelforge_b200.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kernelforge_b200.h"

#define KF_API extern "C" __attribute__((visibility("default")))

namespace kf {

// ------------------------------------------------------------------------------------------
// Element conversions. Rounding to 16-bit types is round-to-nearest-even, as torch's casts.
// ------------------------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ float round_f(float v) { return v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round_f(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round_f(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};

inline size_t dtype_size(int dtype) {
  return dtype == KF_DTYPE_F32 ? 4 : 2;
}
inline bool dtype_valid(int dtype) {
  return dtype == KF_DTYPE_F32 || dtype == KF_DTYPE_F16 || dtype == KF_DTYPE_BF16;
}
inline bool aligned(const void* p, size_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// ------------------------------------------------------------------------------------------
// Cache-hinted 16-byte global accesses. x is streamed once: no L1 allocation on load and an
// evict-first store for the output.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ld_cached_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Nanosecond wall clock for bounded waits.
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace kf

// Host-side check helper used by the C-ABI wrappers.
#define KF_CUDA_TRY(expr)                      \
  do {                                         \
    cudaError_t kf_err__ = (expr);             \
    if (kf_err__ != cudaSuccess) {             \
      (void)cudaGetLastError();                \
      return KF_ERR_CUDA;                      \
    }                                          \
  } while (0)

#define KF_LAUNCH_CHECK()                      \
  do {                                         \
    cudaError_t kf_err__ = cudaGetLastError(); \
    if (kf_err__ != cudaSuccess) return KF_ERR_CUDA; \
  } while (0)
