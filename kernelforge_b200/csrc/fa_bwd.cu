// FlashAttention backward (reverse-mode VJP) from the saved O and LSE: the row statistics.
//
// Replaces the flash_attn binary's _flash_attn_backward that FlashAttentionFunction.backward
// calls (flash_attention_jvp/custom.py:255-266), for every shape the forward supports: head
// dims 8..256 (multiple of 8), causal (bottom-right aligned), GQA / MQA, fp16 / bf16.
//
//   delta_i = sum_d dO[i, d] O[i, d]
//   P  = exp(gamma S - LSE),  S = Q K^T      (masked keys: P = 0)
//   dP = dO V^T,  dS = P * (dP - delta)
//   dQ = gamma dS K,  dK = gamma dS^T Q,  dV = P^T dO
//
// fa_bwd_rowstat_kernel here, one warp per (batch, head, query) row, writes -LSE log2(e) and
// -delta into the padded row-statistics arrays (and zeroes the row's dq_acc sums when the fused
// kernel runs); the tcgen05 kernels of fa_bwd_sm100.cu consume them: one fused kernel whose dQ
// partials are summed at L2, then fa_bwd_dq_convert_kernel here (head dims up to 128, not
// deterministic), or separate dQ and dK / dV kernels with no atomics (deterministic).
#include "fa_common.cuh"

namespace {

using kf::fa::BwdArgs;

constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------------------------------
// Row statistics, fp32 [B, Hq, NqP]: row_nlse = -LSE log2(e), row_ndelta = -rowsum(dO * O);
// padding rows (query >= Nq) get -inf and 0.
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) fa_bwd_rowstat_kernel(const BwdArgs p) {
  const int64_t rows = static_cast<int64_t>(p.B) * p.Hq * p.NqP;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);  // (b, h, i)
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int i = static_cast<int>(row % p.NqP);
  const int64_t bh = row / p.NqP;
  if (p.dq_acc != nullptr) {  // the fused kernel adds its dQ partials into zeroed rows
    float4* acc = reinterpret_cast<float4*>(p.dq_acc + row * p.Dp);
    for (int c = lane; c < p.Dp / 4; c += 32) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (i >= p.Nq) {
    if (lane == 0) {
      p.row_nlse[row] = -__int_as_float(0x7f800000);
      p.row_ndelta[row] = 0.f;
    }
    return;
  }
  const int h = static_cast<int>(bh % p.Hq), b = static_cast<int>(bh / p.Hq);
  const int64_t off = ((static_cast<int64_t>(b) * p.Nq + i) * p.Hq + h) * p.D;
  const T* o = static_cast<const T*>(p.o) + off;
  const T* d = static_cast<const T*>(p.dout) + off;
  float sum = 0.f;
  for (int c = lane * 8; c < p.D; c += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + c);
    const uint4 g = *reinterpret_cast<const uint4*>(d + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = kf::Mma<T>::to_f2(aw[e]), y = kf::Mma<T>::to_f2(gw[e]);
      sum += x.x * y.x + x.y * y.y;
    }
  }
  sum = kf::warp_sum(sum);
  if (lane == 0) {
    p.row_nlse[row] = -p.lse[bh * p.Nq + i] * kLog2e;
    p.row_ndelta[row] = -sum;
  }
}

// ------------------------------------------------------------------------------------------
// dq [B, Nq, Hq, D] = gamma dq_acc [B, Hq, NqP, Dp] (the fused kernel's fp32 sums), rounded to
// T; one thread per 8 head-dim values, grid-stride.
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) fa_bwd_dq_convert_kernel(const BwdArgs p) {
  const int d8 = p.D / 8;
  const int64_t n = static_cast<int64_t>(p.B) * p.Nq * p.Hq * d8;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; idx < n;
       idx += static_cast<int64_t>(gridDim.x) * 256) {
    const int c = static_cast<int>(idx % d8);
    const int64_t bih = idx / d8;
    const int h = static_cast<int>(bih % p.Hq);
    const int64_t bi = bih / p.Hq;
    const int i = static_cast<int>(bi % p.Nq), b = static_cast<int>(bi / p.Nq);
    const float4* src =
        reinterpret_cast<const float4*>(p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + h) * p.NqP + i) * p.Dp + c * 8);
    const float4 x = src[0], y = src[1];
    const float g = p.scale;
    *reinterpret_cast<uint4*>(static_cast<T*>(p.dq) + idx * 8) =
        make_uint4(kf::Mma<T>::from_f2(x.x * g, x.y * g), kf::Mma<T>::from_f2(x.z * g, x.w * g),
                   kf::Mma<T>::from_f2(y.x * g, y.y * g), kf::Mma<T>::from_f2(y.z * g, y.w * g));
  }
}

template <typename T>
int launch_t(const BwdArgs& a, int dtype, cudaStream_t s) {
  if (!kf::fa::sm100_bwd_supported(a)) return KF_ERR_UNSUPPORTED;
  {
    const int64_t rows = static_cast<int64_t>(a.B) * a.Hq * a.NqP;
    fa_bwd_rowstat_kernel<T><<<static_cast<unsigned int>((rows + 7) / 8), 256, 0, s>>>(a);
    KF_LAUNCH_CHECK();
  }
  const int st = kf::fa::launch_sm100_bwd(a, dtype, s);
  if (st != KF_OK || a.dq_acc == nullptr) return st;
  const int64_t n = static_cast<int64_t>(a.B) * a.Nq * a.Hq * (a.D / 8);
  const int64_t blocks = (n + 255) / 256;
  fa_bwd_dq_convert_kernel<T><<<static_cast<unsigned int>(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(a);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

}  // namespace

namespace kf::fa {

int launch_bwd(const BwdArgs& a, int dtype, cudaStream_t s) {
  return dtype == KF_DTYPE_F16 ? launch_t<__half>(a, dtype, s) : launch_t<__nv_bfloat16>(a, dtype, s);
}

}  // namespace kf::fa
