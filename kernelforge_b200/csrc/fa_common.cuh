// Shared declarations of the FlashAttention forward / JVP kernels.
#pragma once

#include "kf_sm100.cuh"

namespace kf::fa {

enum : int { kModeFwd = 0, kModeJvp = 1, kModeFwdJvp = 2 };

// Device pointers and sizes of one call. Tensors are contiguous [B, N, H, D]; LSE is fp32
// [B, Hq, Nq] in natural-log units. Tangent pointers may be null (zero tangent).
struct FaArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* tq;
  const void* tk;
  const void* tv;
  const void* o_in;      // kModeJvp: cached O
  const float* lse_in;   // kModeJvp: cached LSE
  void* o_out;           // kModeFwd / kModeFwdJvp
  float* lse_out;        // kModeFwd / kModeFwdJvp
  void* to_out;          // kModeJvp / kModeFwdJvp
  int B, Nq, Nk, Hq, Hkv, D;
  float scale;       // softmax scale (gamma)
  float scale_log2;  // gamma * log2(e)
  int causal;
};

// mma.sync path: any D in 8..256 (multiple of 8), fp16 / bf16.
int launch_general(const FaArgs& a, int mode, int dtype, cudaStream_t stream);

// tcgen05 / TMEM / TMA path of the standalone JVP: D in {64, 128}, at least one tangent.
bool sm100_jvp_supported(const FaArgs& a);
int launch_sm100_jvp(const FaArgs& a, int dtype, cudaStream_t stream);

// tcgen05 / TMEM / TMA path of the forward (kModeFwd) and one-pass forward + JVP
// (kModeFwdJvp): D in {64, 128}; the one-pass mode needs at least one tangent.
bool sm100_fused_supported(const FaArgs& a, int mode);
int launch_sm100_fused(const FaArgs& a, int mode, int dtype, cudaStream_t stream);

}  // namespace kf::fa
