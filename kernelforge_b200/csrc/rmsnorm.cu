// One-pass RMSNorm forward for sm_100a.
//
// Computes RMSNorm.forward of the reference (rmsnorm/original.py:40-52) with the rounding
// points of its one-pass kernel (rmsnorm/custom.py:63-73):
//   r    = 1 / sqrt(sum(x^2) / dim + eps)                (fp32)
//   y    = cast(float(cast(x * r)) * float(w))           (two roundings for 16-bit types)
//
// Design (HBM-bound: 2 bytes read + 2 bytes written per bf16 element):
//   * a row is split over TPR = 32..256 threads (one CTA holds 256 / TPR rows); every thread keeps NV 16-byte vectors of
//     the row in registers, so x is read from HBM exactly once;
//   * loads bypass L1 (ld.global.nc.L1::no_allocate), stores are evict-first (st.global.cs);
//   * the weight vector is re-read per row through L1 (it is shared by every row and stays
//     cache resident), keeping registers for in-flight row data; the grid is persistent and
//     sized from the occupancy of the chosen variant;
//   * sum of squares: fp32, warp shuffle, then (TPR > 32) a fixed-order sum of the row's
//     warp partials through shared memory -- deterministic for a given launch shape;
//   * any dim / alignment not fitting the vector path goes to a generic kernel (one CTA per
//     row, two passes over the row through L2).
#include "kf_common.cuh"

#include <algorithm>

namespace {

constexpr int kBlock = 256;
constexpr int kMaxNV = 8;

template <typename T> struct Pack;
template <> struct Pack<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct Pack<__half> {
  static constexpr int kPerVec = 8;
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct Pack<float> {
  static constexpr int kPerVec = 4;
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};

// Row scale with IEEE division and square root (matches 1/sqrt on the CPU).
__device__ __forceinline__ float row_scale(float sum_sq, int dim, float eps) {
  return 1.0f / sqrtf(sum_sq / static_cast<float>(dim) + eps);
}

template <typename T, int NV, bool kHasWeight>
__global__ void __launch_bounds__(kBlock)
rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                   int64_t rows, int nvec, int dim, int64_t x_stride, int64_t y_stride, float eps,
                   int tpr_log2) {
  using P = Pack<T>;
  constexpr int E = P::kPerVec;
  const int tpr = 1 << tpr_log2;
  const int lane = threadIdx.x & (tpr - 1);
  const int row_in_cta = threadIdx.x >> tpr_log2;
  const int rows_per_cta = kBlock >> tpr_log2;
  const int warps_per_row = tpr >> 5;
  __shared__ float partial[kBlock / 32];

  const int64_t step = static_cast<int64_t>(gridDim.x) * rows_per_cta;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * rows_per_cta; base < rows; base += step) {
    const int64_t row = base + row_in_cta;
    const bool active = row < rows;
    const T* xr = x + row * x_stride;
    uint4 xv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = lane + i * tpr;
      xv[i] = (active && v < nvec) ? kf::ld_stream_v4(xr + static_cast<int64_t>(v) * E)
                                   : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float f[E];
      P::unpack(xv[i], f);
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(f[e], f[e], ss);
    }
    ss = kf::warp_sum(ss);
    if (warps_per_row > 1) {
      if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
      __syncthreads();
      const int first = row_in_cta * warps_per_row;
      ss = 0.f;
      for (int k = 0; k < warps_per_row; ++k) ss += partial[first + k];
      __syncthreads();
    }
    const float r = row_scale(ss, dim, eps);
    if (active) {
      T* yr = y + row * y_stride;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int v = lane + i * tpr;
        if (v < nvec) {
          float f[E];
          P::unpack(xv[i], f);
          if constexpr (kHasWeight) {
            // The weight row is tiny and shared by every row: it stays L1/L2 resident.
            float g[E];
            P::unpack(kf::ld_cached_v4(w + static_cast<int64_t>(v) * E), g);
#pragma unroll
            for (int e = 0; e < E; ++e) f[e] = kf::Elem<T>::round_f(f[e] * r) * g[e];
          } else {
#pragma unroll
            for (int e = 0; e < E; ++e) f[e] = f[e] * r;
          }
          kf::st_stream_v4(yr + static_cast<int64_t>(v) * E, P::pack(f));
        }
      }
    }
  }
}

// Any dim, any alignment: one CTA per row, two passes (the second mostly hits L2).
template <typename T>
__global__ void __launch_bounds__(kBlock)
rmsnorm_generic_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                       int64_t rows, int64_t dim, int64_t x_stride, int64_t y_stride, float eps) {
  __shared__ float partial[kBlock / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * x_stride;
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < dim; c += kBlock) {
      const float v = kf::Elem<T>::to_f(xr[c]);
      ss = fmaf(v, v, ss);
    }
    ss = kf::warp_sum(ss);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
    for (int k = 0; k < kBlock / 32; ++k) ss += partial[k];
    __syncthreads();
    const float r = row_scale(ss, static_cast<int>(dim), eps);
    T* yr = y + row * y_stride;
    for (int64_t c = threadIdx.x; c < dim; c += kBlock) {
      float v = kf::Elem<T>::to_f(xr[c]) * r;
      if (w != nullptr) v = kf::Elem<T>::round_f(v) * kf::Elem<T>::to_f(w[c]);
      yr[c] = kf::Elem<T>::from_f(v);
    }
  }
}

struct DeviceInfo {
  int sms = 0;
};

int device_sms() {
  static DeviceInfo info[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (info[dev].sms == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    info[dev].sms = sms;
  }
  return info[dev].sms;
}

template <typename T, int NV, bool kW>
int launch_vec_nv(const T* x, const T* w, T* y, int64_t rows, int nvec, int dim, int64_t xs,
                  int64_t ys, float eps, int tpr_log2, cudaStream_t stream) {
  auto kernel = rmsnorm_vec_kernel<T, NV, kW>;
  static int occ_cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = (dev >= 0 && dev < 64) ? occ_cache[dev] : 0;
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kBlock, 0) != cudaSuccess || occ <= 0) {
      (void)cudaGetLastError();
      occ = 4;
    }
    if (dev >= 0 && dev < 64) occ_cache[dev] = occ;
  }
  const int rows_per_cta = kBlock >> tpr_log2;
  const int64_t needed = (rows + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = static_cast<int64_t>(device_sms()) * occ;
  const int grid = static_cast<int>(std::min<int64_t>(needed, cap));
  kernel<<<grid, kBlock, 0, stream>>>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

template <typename T, bool kW>
int launch_vec(const T* x, const T* w, T* y, int64_t rows, int nvec, int dim, int64_t xs,
               int64_t ys, float eps, int tpr_log2, int nv, cudaStream_t s) {
  switch (nv) {
    case 1: return launch_vec_nv<T, 1, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    case 2: return launch_vec_nv<T, 2, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    case 3: return launch_vec_nv<T, 3, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    case 4: return launch_vec_nv<T, 4, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    case 5: return launch_vec_nv<T, 5, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    case 6: return launch_vec_nv<T, 6, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    case 7: return launch_vec_nv<T, 7, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
    default: return launch_vec_nv<T, 8, kW>(x, w, y, rows, nvec, dim, xs, ys, eps, tpr_log2, s);
  }
}

template <typename T>
int run_rmsnorm(const void* xp, const void* wp, void* yp, int64_t rows, int64_t dim, int64_t xs,
                int64_t ys, float eps, cudaStream_t stream) {
  const T* x = static_cast<const T*>(xp);
  const T* w = static_cast<const T*>(wp);
  T* y = static_cast<T*>(yp);
  constexpr int E = Pack<T>::kPerVec;
  const bool vec_ok = (dim % E == 0) && (xs % E == 0) && (ys % E == 0) && kf::aligned(x, 16) &&
                      kf::aligned(y, 16) && (w == nullptr || kf::aligned(w, 16)) &&
                      dim / E <= kBlock * kMaxNV;
  if (vec_ok) {
    const int nvec = static_cast<int>(dim / E);
    // Threads per row: grow from a warp to the CTA while a thread would hold > 4 vectors;
    // rows wider than 256 x 4 vectors use up to kMaxNV vectors per thread.
    int tpr_log2 = 5;
    while ((1 << tpr_log2) * 4 < nvec && (1 << tpr_log2) < kBlock) ++tpr_log2;
    const int tpr = 1 << tpr_log2;
    const int nv = (nvec + tpr - 1) / tpr;
    if (w != nullptr)
      return launch_vec<T, true>(x, w, y, rows, nvec, static_cast<int>(dim), xs, ys, eps, tpr_log2, nv, stream);
    return launch_vec<T, false>(x, w, y, rows, nvec, static_cast<int>(dim), xs, ys, eps, tpr_log2, nv, stream);
  }
  const int64_t cap = static_cast<int64_t>(device_sms()) * 8;
  const int grid = static_cast<int>(std::min<int64_t>(rows, cap));
  rmsnorm_generic_kernel<T><<<grid, kBlock, 0, stream>>>(x, w, y, rows, dim, xs, ys, eps);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

}  // namespace

KF_API int kf_rmsnorm_fwd(const void* x, const void* weight, void* y, int64_t rows, int64_t dim,
                          int64_t x_row_stride, int64_t y_row_stride, float eps, int dtype,
                          void* stream) {
  if (!kf::dtype_valid(dtype)) return KF_ERR_UNSUPPORTED;
  if (rows < 0 || dim <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (rows == 0) return KF_OK;
  if (x == nullptr || y == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (rows > 1 && (x_row_stride < dim || y_row_stride < dim)) return KF_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  if (dim > (int64_t(1) << 30)) return KF_ERR_UNSUPPORTED;
  const size_t es = kf::dtype_size(dtype);
  if (!kf::aligned(x, es) || !kf::aligned(y, es) || (weight && !kf::aligned(weight, es)))
    return KF_ERR_MISALIGNED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case KF_DTYPE_F32: return run_rmsnorm<float>(x, weight, y, rows, dim, x_row_stride, y_row_stride, eps, s);
    case KF_DTYPE_F16: return run_rmsnorm<__half>(x, weight, y, rows, dim, x_row_stride, y_row_stride, eps, s);
    default: return run_rmsnorm<__nv_bfloat16>(x, weight, y, rows, dim, x_row_stride, y_row_stride, eps, s);
  }
}
