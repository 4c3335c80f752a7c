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

// Inputs and outputs of the backward (reverse-mode VJP) from the saved O and LSE. Tensors are
// contiguous [B, N, H, D]; LSE is fp32 [B, Hq, Nq] (natural log). The first kernel fills two fp32
// row-statistics arrays of the workspace, each [B, Hq, NqP] with NqP = Nq rounded up to
// kBwdRowPad: row_nlse = -LSE log2(e) and row_ndelta = -rowsum(dO * O); padding rows hold -inf
// and 0, so that they contribute P = 0 and dS = 0 wherever a tile reads past Nq.
constexpr int kBwdRowPad = 128;
struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  float* row_nlse;
  float* row_ndelta;
  float* dq_acc;  // non-deterministic schedule: fp32 dQ sums [B, Hq, NqP, Dp], else null
  int Dp;         // head dim of the dq_acc rows (the kernel's zero-padded head dim)
  void* dq;
  void* dk;
  void* dv;
  int B, Nq, Nk, Hq, Hkv, D;
  int NqP;
  float scale;
  float scale_log2;
  int causal;
};

// Row statistics, then dQ, dK, dV on the tcgen05 kernels: head dims up to 256, zero-padded to
// 64, 128 or 256. With dq_acc set (head dims up to 128), one kernel computes all three and adds
// its dQ partials into dq_acc at L2 (summation order varies from run to run), then a conversion
// pass writes dq; otherwise separate dQ and dK / dV kernels, no atomics (deterministic).
int launch_bwd(const BwdArgs& a, int dtype, cudaStream_t stream);
bool sm100_bwd_supported(const BwdArgs& a);
int launch_sm100_bwd(const BwdArgs& a, int dtype, cudaStream_t stream);

// 4-D TMA map of a contiguous [B, N, H, D] 16-bit tensor with 128-byte swizzle: boxes of 64
// head-dim elements x 1 head x `rows` tokens x 1 batch.
inline bool encode_bnhd(CUtensorMap* map, const void* base, int dtype, int B, int N, int H, int D, int rows) {
  const uint64_t es = 2;
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H), static_cast<uint64_t>(N),
                            static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {D * es, static_cast<uint64_t>(H) * D * es,
                               static_cast<uint64_t>(N) * H * D * es};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(rows), 1};
  return kf_host::encode_tiled(map, kf_host::map_type(dtype), 4, base, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
}

// tcgen05 / TMEM / TMA path of the standalone JVP: D up to 256 (zero-padded to 64, 128 or 256),
// at least one tangent.
bool sm100_jvp_supported(const FaArgs& a);
int launch_sm100_jvp(const FaArgs& a, int dtype, cudaStream_t stream);

// tcgen05 / TMEM / TMA path of the forward (kModeFwd, D up to 256) and one-pass forward + JVP
// (kModeFwdJvp, D up to 128, at least one tangent).
bool sm100_fused_supported(const FaArgs& a, int mode);
int launch_sm100_fused(const FaArgs& a, int mode, int dtype, cudaStream_t stream);

}  // namespace kf::fa
