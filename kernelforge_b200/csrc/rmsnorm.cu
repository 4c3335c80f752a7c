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

namespace {

// ------------------------------------------------------------------------------------------
// Backward. The reference ships RMSNorm forward only (rmsnorm/README.md:5); this is the gradient
// of its forward y = cast(cast(x r) w), r = 1 / sqrt(mean(x^2) + eps), with the casts taken as
// identities (as torch autograd treats .type_as):
//   g   = dy w                                       (fp32)
//   dx  = r g - x r^3 (g . x) / dim
//   dw  = sum over rows of dy cast(x r)
// One pass per row over x and dy (both in registers, like the forward), dx written once. Every
// thread keeps the dw partial of its columns in registers across the rows it visits; each CTA
// writes one fp32 partial row to the workspace and a second launch sums the partial rows in CTA
// order (deterministic for a given launch shape) and rounds them to the weight's dtype.
// HBM-bound: 6 bytes per bf16 element (x, dy read; dx written) + 4 bytes x dim per CTA.
// ------------------------------------------------------------------------------------------
constexpr int kMaxBwdParts = 320;  // CTAs of a backward launch, and dw partial rows
constexpr int kMaxBwdNV = 4;       // vectors per thread per row on the vector path

template <typename T, int NV, bool kW>
__global__ void __launch_bounds__(kBlock, 2)
rmsnorm_bwd_vec_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ dy,
                       T* __restrict__ dx, float* __restrict__ part, int64_t rows, int nvec, int dim,
                       int64_t x_stride, int64_t dy_stride, int64_t dx_stride, float eps, int tpr_log2) {
  using P = Pack<T>;
  constexpr int E = P::kPerVec;
  const int tpr = 1 << tpr_log2;
  const int lane = threadIdx.x & (tpr - 1);
  const int row_in_cta = threadIdx.x >> tpr_log2;
  const int rows_per_cta = kBlock >> tpr_log2;
  const int warps_per_row = tpr >> 5;
  __shared__ float partial[2][kBlock / 32];
  // dw partials, [row group][dim]: each thread owns its columns in its row group's row (no two
  // threads touch one slot until the final sum). Shared memory rather than registers keeps two
  // CTAs per SM without spills.
  extern __shared__ float dw_rows[];

  // This thread's columns are the same in every row: its weight vectors stay in registers.
  uint4 wv[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = lane + i * tpr;
    wv[i] = (kW && v < nvec) ? kf::ld_cached_v4(w + static_cast<int64_t>(v) * E) : make_uint4(0, 0, 0, 0);
    if (kW && v < nvec)
#pragma unroll
      for (int e = 0; e < E; e += 4)
        *reinterpret_cast<float4*>(dw_rows + row_in_cta * dim + v * E + e) = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  const int64_t step = static_cast<int64_t>(gridDim.x) * rows_per_cta;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * rows_per_cta; base < rows; base += step) {
    const int64_t row = base + row_in_cta;
    const bool active = row < rows;
    const T* xr = x + row * x_stride;
    const T* dyr = dy + row * dy_stride;
    uint4 xv[NV], dv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = lane + i * tpr;
      const bool in = active && v < nvec;
      xv[i] = in ? kf::ld_stream_v4(xr + static_cast<int64_t>(v) * E) : make_uint4(0, 0, 0, 0);
      dv[i] = in ? kf::ld_stream_v4(dyr + static_cast<int64_t>(v) * E) : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float xf[E], df[E], wf[E];
      P::unpack(xv[i], xf);
      P::unpack(dv[i], df);
      P::unpack(wv[i], wf);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        ss = fmaf(xf[e], xf[e], ss);
        dot = fmaf(kW ? df[e] * wf[e] : df[e], xf[e], dot);
      }
    }
    ss = kf::warp_sum(ss);
    dot = kf::warp_sum(dot);
    if (warps_per_row > 1) {
      if ((threadIdx.x & 31) == 0) {
        partial[0][threadIdx.x >> 5] = ss;
        partial[1][threadIdx.x >> 5] = dot;
      }
      __syncthreads();
      const int first = row_in_cta * warps_per_row;
      ss = 0.f;
      dot = 0.f;
      for (int k = 0; k < warps_per_row; ++k) {
        ss += partial[0][first + k];
        dot += partial[1][first + k];
      }
      __syncthreads();
    }
    const float r = row_scale(ss, dim, eps);
    const float c = r * r * r * dot / static_cast<float>(dim);
    if (active) {
      T* dxr = dx + row * dx_stride;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int v = lane + i * tpr;
        if (v < nvec) {
          float xf[E], df[E], wf[E], out[E];
          P::unpack(xv[i], xf);
          P::unpack(dv[i], df);
          P::unpack(wv[i], wf);
#pragma unroll
          for (int e = 0; e < E; ++e) out[e] = r * (kW ? df[e] * wf[e] : df[e]) - xf[e] * c;
          kf::st_stream_v4(dxr + static_cast<int64_t>(v) * E, P::pack(out));
          if (kW) {
            float* acc = dw_rows + row_in_cta * dim + v * E;
#pragma unroll
            for (int e = 0; e < E; e += 4) {
              float4 a = *reinterpret_cast<float4*>(acc + e);
              a.x = fmaf(df[e], kf::Elem<T>::round_f(xf[e] * r), a.x);
              a.y = fmaf(df[e + 1], kf::Elem<T>::round_f(xf[e + 1] * r), a.y);
              a.z = fmaf(df[e + 2], kf::Elem<T>::round_f(xf[e + 2] * r), a.z);
              a.w = fmaf(df[e + 3], kf::Elem<T>::round_f(xf[e + 3] * r), a.w);
              *reinterpret_cast<float4*>(acc + e) = a;
            }
          }
        }
      }
    }
  }
  if (!kW) return;
  // This CTA's partial row: the row groups' partials summed in group order.
  float* prow = part + static_cast<int64_t>(blockIdx.x) * dim;
  __syncthreads();
  for (int col = threadIdx.x; col < dim; col += kBlock) {
    float s = 0.f;
    for (int g = 0; g < rows_per_cta; ++g) s += dw_rows[g * dim + col];
    prow[col] = s;
  }
}

// Any dim, any alignment: one CTA per row at a time, two passes over the row. Thread t owns
// columns t, t + 256, ... of this CTA's dw partial row, kept in the workspace.
template <typename T, bool kW>
__global__ void __launch_bounds__(kBlock)
rmsnorm_bwd_generic_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ dy,
                           T* __restrict__ dx, float* __restrict__ part, int64_t rows, int64_t dim,
                           int64_t x_stride, int64_t dy_stride, int64_t dx_stride, float eps) {
  __shared__ float partial[2][kBlock / 32];
  float* prow = part + static_cast<int64_t>(blockIdx.x) * dim;
  if (kW)
    for (int64_t col = threadIdx.x; col < dim; col += kBlock) prow[col] = 0.f;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * x_stride;
    const T* dyr = dy + row * dy_stride;
    float ss = 0.f, dot = 0.f;
    for (int64_t col = threadIdx.x; col < dim; col += kBlock) {
      const float xf = kf::Elem<T>::to_f(xr[col]);
      const float g = kf::Elem<T>::to_f(dyr[col]) * (kW ? kf::Elem<T>::to_f(w[col]) : 1.f);
      ss = fmaf(xf, xf, ss);
      dot = fmaf(g, xf, dot);
    }
    ss = kf::warp_sum(ss);
    dot = kf::warp_sum(dot);
    if ((threadIdx.x & 31) == 0) {
      partial[0][threadIdx.x >> 5] = ss;
      partial[1][threadIdx.x >> 5] = dot;
    }
    __syncthreads();
    ss = 0.f;
    dot = 0.f;
    for (int k = 0; k < kBlock / 32; ++k) {
      ss += partial[0][k];
      dot += partial[1][k];
    }
    __syncthreads();
    const float r = row_scale(ss, static_cast<int>(dim), eps);
    const float c = r * r * r * dot / static_cast<float>(dim);
    T* dxr = dx + row * dx_stride;
    for (int64_t col = threadIdx.x; col < dim; col += kBlock) {
      const float xf = kf::Elem<T>::to_f(xr[col]);
      const float df = kf::Elem<T>::to_f(dyr[col]);
      const float g = df * (kW ? kf::Elem<T>::to_f(w[col]) : 1.f);
      dxr[col] = kf::Elem<T>::from_f(r * g - xf * c);
      if (kW) prow[col] = fmaf(df, kf::Elem<T>::round_f(xf * r), prow[col]);
    }
  }
}

// dw[c] = sum of the `parts` partial rows at column c, in row order.
template <typename T>
__global__ void __launch_bounds__(kBlock)
rmsnorm_dw_reduce_kernel(const float* __restrict__ part, int parts, int64_t dim, T* __restrict__ dw) {
  const int64_t col = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
  if (col >= dim) return;
  float s = 0.f;
#pragma unroll 8
  for (int p = 0; p < parts; ++p) s += __ldcg(part + p * dim + col);
  dw[col] = kf::Elem<T>::from_f(s);
}

template <typename T, int NV, bool kW>
int launch_bwd_vec_nv(const T* x, const T* w, const T* dy, T* dx, float* part, int64_t rows, int nvec, int dim,
                      int64_t xs, int64_t dys, int64_t dxs, float eps, int tpr_log2, cudaStream_t stream,
                      int* parts) {
  auto kernel = rmsnorm_bwd_vec_kernel<T, NV, kW>;
  const int rows_per_cta = kBlock >> tpr_log2;
  const int smem = kW ? rows_per_cta * dim * 4 : 0;  // <= 32 KB: nvec <= 4 x tpr, or tpr = 256 and NV <= 4
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kBlock, smem) != cudaSuccess || occ <= 0) {
    (void)cudaGetLastError();
    occ = 1;
  }
  const int64_t needed = (rows + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = std::min<int64_t>(kMaxBwdParts, static_cast<int64_t>(device_sms()) * occ);
  const int grid = static_cast<int>(std::min<int64_t>(needed, cap));
  kernel<<<grid, kBlock, smem, stream>>>(x, w, dy, dx, part, rows, nvec, dim, xs, dys, dxs, eps, tpr_log2);
  KF_LAUNCH_CHECK();
  *parts = grid;
  return KF_OK;
}

template <typename T, bool kW>
int launch_bwd_vec(const T* x, const T* w, const T* dy, T* dx, float* part, int64_t rows, int nvec, int dim,
                   int64_t xs, int64_t dys, int64_t dxs, float eps, int tpr_log2, int nv, cudaStream_t s,
                   int* parts) {
  switch (nv) {
    case 1: return launch_bwd_vec_nv<T, 1, kW>(x, w, dy, dx, part, rows, nvec, dim, xs, dys, dxs, eps, tpr_log2, s, parts);
    case 2: return launch_bwd_vec_nv<T, 2, kW>(x, w, dy, dx, part, rows, nvec, dim, xs, dys, dxs, eps, tpr_log2, s, parts);
    case 3: return launch_bwd_vec_nv<T, 3, kW>(x, w, dy, dx, part, rows, nvec, dim, xs, dys, dxs, eps, tpr_log2, s, parts);
    default: return launch_bwd_vec_nv<T, 4, kW>(x, w, dy, dx, part, rows, nvec, dim, xs, dys, dxs, eps, tpr_log2, s, parts);
  }
}

template <typename T>
int run_rmsnorm_bwd(const void* xp, const void* wp, const void* dyp, void* dxp, void* dwp, float* part,
                    int64_t rows, int64_t dim, int64_t xs, int64_t dys, int64_t dxs, float eps, cudaStream_t stream) {
  const T* x = static_cast<const T*>(xp);
  const T* w = static_cast<const T*>(wp);
  const T* dy = static_cast<const T*>(dyp);
  T* dx = static_cast<T*>(dxp);
  constexpr int E = Pack<T>::kPerVec;
  const bool vec_ok = (dim % E == 0) && (xs % E == 0) && (dys % E == 0) && (dxs % E == 0) && kf::aligned(x, 16) &&
                      kf::aligned(dy, 16) && kf::aligned(dx, 16) && (w == nullptr || kf::aligned(w, 16)) &&
                      dim / E <= kBlock * kMaxBwdNV && kf::aligned(part, 16);
  int parts = 0;
  int st = KF_OK;
  if (vec_ok) {
    const int nvec = static_cast<int>(dim / E);
    // Threads per row as in the forward: from a warp up to the CTA while a thread would hold
    // more than 4 vectors.
    int tpr_log2 = 5;
    while ((1 << tpr_log2) * 4 < nvec && (1 << tpr_log2) < kBlock) ++tpr_log2;
    const int tpr = 1 << tpr_log2;
    const int nv = (nvec + tpr - 1) / tpr;
    st = w != nullptr
             ? launch_bwd_vec<T, true>(x, w, dy, dx, part, rows, nvec, static_cast<int>(dim), xs, dys, dxs, eps,
                                       tpr_log2, nv, stream, &parts)
             : launch_bwd_vec<T, false>(x, w, dy, dx, part, rows, nvec, static_cast<int>(dim), xs, dys, dxs, eps,
                                        tpr_log2, nv, stream, &parts);
  } else {
    const int64_t cap = std::min<int64_t>(kMaxBwdParts, static_cast<int64_t>(device_sms()) * 2);
    parts = static_cast<int>(std::min<int64_t>(rows, cap));
    if (w != nullptr)
      rmsnorm_bwd_generic_kernel<T, true><<<parts, kBlock, 0, stream>>>(x, w, dy, dx, part, rows, dim, xs, dys, dxs, eps);
    else
      rmsnorm_bwd_generic_kernel<T, false><<<parts, kBlock, 0, stream>>>(x, w, dy, dx, part, rows, dim, xs, dys, dxs, eps);
    KF_LAUNCH_CHECK();
  }
  if (st != KF_OK || w == nullptr) return st;
  const int grid = static_cast<int>((dim + kBlock - 1) / kBlock);
  rmsnorm_dw_reduce_kernel<T><<<grid, kBlock, 0, stream>>>(part, parts, dim, static_cast<T*>(dwp));
  KF_LAUNCH_CHECK();
  return KF_OK;
}

}  // namespace

KF_API size_t kf_rmsnorm_bwd_workspace_size(int64_t dim) {
  if (dim <= 0 || dim > (int64_t(1) << 30)) return 0;
  return static_cast<size_t>(kMaxBwdParts) * static_cast<size_t>(dim) * sizeof(float);
}

KF_API int kf_rmsnorm_bwd(const void* x, const void* weight, const void* dy, void* dx, void* dweight,
                          void* workspace, size_t workspace_bytes, int64_t rows, int64_t dim,
                          int64_t x_row_stride, int64_t dy_row_stride, int64_t dx_row_stride, float eps,
                          int dtype, void* stream) {
  if (!kf::dtype_valid(dtype)) return KF_ERR_UNSUPPORTED;
  if (rows < 0 || dim <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (dim > (int64_t(1) << 30)) return KF_ERR_UNSUPPORTED;
  if ((weight == nullptr) != (dweight == nullptr)) return KF_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  const size_t es = kf::dtype_size(dtype);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (dweight != nullptr) KF_CUDA_TRY(cudaMemsetAsync(dweight, 0, static_cast<size_t>(dim) * es, s));
    return KF_OK;
  }
  if (x == nullptr || dy == nullptr || dx == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (rows > 1 && (x_row_stride < dim || dy_row_stride < dim || dx_row_stride < dim)) return KF_ERR_INVALID_ARGUMENT;
  if (weight != nullptr) {
    if (workspace == nullptr) return KF_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < kf_rmsnorm_bwd_workspace_size(dim)) return KF_ERR_WORKSPACE;
    if (!kf::aligned(workspace, 16)) return KF_ERR_MISALIGNED;
  }
  if (!kf::aligned(x, es) || !kf::aligned(dy, es) || !kf::aligned(dx, es) || (weight && !kf::aligned(weight, es)) ||
      (dweight && !kf::aligned(dweight, es)))
    return KF_ERR_MISALIGNED;
  float* part = static_cast<float*>(workspace);
  switch (dtype) {
    case KF_DTYPE_F32:
      return run_rmsnorm_bwd<float>(x, weight, dy, dx, dweight, part, rows, dim, x_row_stride, dy_row_stride,
                                    dx_row_stride, eps, s);
    case KF_DTYPE_F16:
      return run_rmsnorm_bwd<__half>(x, weight, dy, dx, dweight, part, rows, dim, x_row_stride, dy_row_stride,
                                     dx_row_stride, eps, s);
    default:
      return run_rmsnorm_bwd<__nv_bfloat16>(x, weight, dy, dx, dweight, part, rows, dim, x_row_stride,
                                            dy_row_stride, dx_row_stride, eps, s);
  }
}
