// C ABI of the FlashAttention forward / forward-mode JVP kernels: validation and dispatch.
#include "fa_common.cuh"

#include <cmath>

namespace {

using kf::fa::FaArgs;

int validate(const void* q, const void* k, const void* v, int64_t B, int64_t Nq, int64_t Nk,
             int64_t Hq, int64_t Hkv, int64_t D, float scale, int dtype) {
  if (dtype != KF_DTYPE_F16 && dtype != KF_DTYPE_BF16) return KF_ERR_UNSUPPORTED;
  if (q == nullptr || k == nullptr || v == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (B <= 0 || Nq <= 0 || Nk <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (Hq % Hkv != 0 || D % 8 != 0 || D > 256) return KF_ERR_UNSUPPORTED;
  if (!(std::isfinite(scale) && scale > 0.f)) return KF_ERR_INVALID_ARGUMENT;
  if (B > 65535 || Hq > 65535 || Nq > (int64_t(1) << 30) || Nk > (int64_t(1) << 30))
    return KF_ERR_UNSUPPORTED;
  return KF_OK;
}

bool aligned16(const void* p) { return p == nullptr || kf::aligned(p, 16); }

// A JVP with every tangent missing is the zero tangent: tO = 0 exactly, no kernel needed.
int zero_tangent(const FaArgs& a, cudaStream_t stream) {
  const size_t bytes = static_cast<size_t>(a.B) * a.Nq * a.Hq * a.D * 2;
  return cudaMemsetAsync(a.to_out, 0, bytes, stream) == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

FaArgs make_args(const void* q, const void* k, const void* v, const void* tq, const void* tk,
                 const void* tv, int64_t B, int64_t Nq, int64_t Nk, int64_t Hq, int64_t Hkv,
                 int64_t D, float scale, int causal) {
  FaArgs a = {};
  a.q = q; a.k = k; a.v = v; a.tq = tq; a.tk = tk; a.tv = tv;
  a.B = static_cast<int>(B); a.Nq = static_cast<int>(Nq); a.Nk = static_cast<int>(Nk);
  a.Hq = static_cast<int>(Hq); a.Hkv = static_cast<int>(Hkv); a.D = static_cast<int>(D);
  a.scale = scale;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  return a;
}

}  // namespace

KF_API int kf_fa_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
                     int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads,
                     int64_t kv_heads, int64_t head_dim, float softmax_scale, int causal,
                     int dtype, void* stream) {
  int st = validate(q, k, v, batch, q_len, k_len, q_heads, kv_heads, head_dim, softmax_scale, dtype);
  if (st != KF_OK) return st;
  if (out == nullptr || lse == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !kf::aligned(lse, 4))
    return KF_ERR_MISALIGNED;
  FaArgs a = make_args(q, k, v, nullptr, nullptr, nullptr, batch, q_len, k_len, q_heads, kv_heads,
                       head_dim, softmax_scale, causal);
  a.o_out = out;
  a.lse_out = lse;
  if (kf::fa::sm100_fused_supported(a, kf::fa::kModeFwd))
    return kf::fa::launch_sm100_fused(a, kf::fa::kModeFwd, dtype, static_cast<cudaStream_t>(stream));
  return KF_ERR_UNSUPPORTED;
}

KF_API int kf_fa_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
                     const void* tv, const void* out, const float* lse, void* tangent_out,
                     int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads,
                     int64_t kv_heads, int64_t head_dim, float softmax_scale, int causal,
                     int dtype, void* stream) {
  int st = validate(q, k, v, batch, q_len, k_len, q_heads, kv_heads, head_dim, softmax_scale, dtype);
  if (st != KF_OK) return st;
  if (out == nullptr || lse == nullptr || tangent_out == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(tq) || !aligned16(tk) ||
      !aligned16(tv) || !aligned16(out) || !aligned16(tangent_out) || !kf::aligned(lse, 4))
    return KF_ERR_MISALIGNED;
  FaArgs a = make_args(q, k, v, tq, tk, tv, batch, q_len, k_len, q_heads, kv_heads, head_dim,
                       softmax_scale, causal);
  a.o_in = out;
  a.lse_in = lse;
  a.to_out = tangent_out;
  if (tq == nullptr && tk == nullptr && tv == nullptr) return zero_tangent(a, static_cast<cudaStream_t>(stream));
  if (kf::fa::sm100_jvp_supported(a))
    return kf::fa::launch_sm100_jvp(a, dtype, static_cast<cudaStream_t>(stream));
  return KF_ERR_UNSUPPORTED;
}

KF_API int kf_fa_fwd_jvp(const void* q, const void* k, const void* v, const void* tq,
                         const void* tk, const void* tv, void* out, float* lse, void* tangent_out,
                         int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads,
                         int64_t kv_heads, int64_t head_dim, float softmax_scale, int causal,
                         int dtype, void* stream) {
  int st = validate(q, k, v, batch, q_len, k_len, q_heads, kv_heads, head_dim, softmax_scale, dtype);
  if (st != KF_OK) return st;
  if (out == nullptr || lse == nullptr || tangent_out == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(tq) || !aligned16(tk) ||
      !aligned16(tv) || !aligned16(out) || !aligned16(tangent_out) || !kf::aligned(lse, 4))
    return KF_ERR_MISALIGNED;
  FaArgs a = make_args(q, k, v, tq, tk, tv, batch, q_len, k_len, q_heads, kv_heads, head_dim,
                       softmax_scale, causal);
  a.o_out = out;
  a.lse_out = lse;
  a.to_out = tangent_out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kf::fa::sm100_fused_supported(a, kf::fa::kModeFwdJvp)) return kf::fa::launch_sm100_fused(a, kf::fa::kModeFwdJvp, dtype, s);
  if (!kf::fa::sm100_fused_supported(a, kf::fa::kModeFwd)) return KF_ERR_UNSUPPORTED;
  // Otherwise the forward (O, LSE) runs first: every tangent missing (tO = 0), or head dims
  // 136..256, where tensor memory holds one D = 256 accumulator, not O and tO together, and the
  // standalone JVP reads O and LSE back.
  st = kf::fa::launch_sm100_fused(a, kf::fa::kModeFwd, dtype, s);
  if (st != KF_OK) return st;
  if (tq == nullptr && tk == nullptr && tv == nullptr) return zero_tangent(a, s);
  a.o_in = out;
  a.lse_in = lse;
  return kf::fa::sm100_jvp_supported(a) ? kf::fa::launch_sm100_jvp(a, dtype, s) : KF_ERR_UNSUPPORTED;
}

namespace {

// Head dim of the fused kernel's dq_acc rows, or 0 when the separate (deterministic) kernels run.
int64_t fused_dq_cols(int64_t head_dim, int deterministic) {
  if (deterministic || head_dim > 128) return 0;
  return head_dim <= 64 ? 64 : 128;
}

}  // namespace

KF_API size_t kf_fa_bwd_workspace_size(int64_t batch, int64_t q_heads, int64_t q_len, int64_t head_dim,
                                       int deterministic) {
  if (batch <= 0 || q_heads <= 0 || q_len <= 0 || head_dim <= 0) return 0;
  const int64_t padded = (q_len + kf::fa::kBwdRowPad - 1) / kf::fa::kBwdRowPad * kf::fa::kBwdRowPad;
  const int64_t cols = 2 + fused_dq_cols(head_dim, deterministic);
  return static_cast<size_t>(cols) * batch * q_heads * padded * sizeof(float);
}

KF_API int kf_fa_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout,
                     const float* lse, void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
                     int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads, int64_t kv_heads,
                     int64_t head_dim, float softmax_scale, int causal, int deterministic, int dtype,
                     void* stream) {
  int st = validate(q, k, v, batch, q_len, k_len, q_heads, kv_heads, head_dim, softmax_scale, dtype);
  if (st != KF_OK) return st;
  if (out == nullptr || dout == nullptr || lse == nullptr || dq == nullptr || dk == nullptr || dv == nullptr ||
      workspace == nullptr)
    return KF_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < kf_fa_bwd_workspace_size(batch, q_heads, q_len, head_dim, deterministic))
    return KF_ERR_WORKSPACE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(dout) ||
      !aligned16(dq) || !aligned16(dk) || !aligned16(dv) || !kf::aligned(lse, 4) || !aligned16(workspace))
    return KF_ERR_MISALIGNED;
  kf::fa::BwdArgs a = {};
  a.q = q; a.k = k; a.v = v; a.o = out; a.dout = dout; a.lse = lse;
  a.dq = dq; a.dk = dk; a.dv = dv;
  a.B = static_cast<int>(batch); a.Nq = static_cast<int>(q_len); a.Nk = static_cast<int>(k_len);
  a.Hq = static_cast<int>(q_heads); a.Hkv = static_cast<int>(kv_heads); a.D = static_cast<int>(head_dim);
  a.NqP = (a.Nq + kf::fa::kBwdRowPad - 1) / kf::fa::kBwdRowPad * kf::fa::kBwdRowPad;
  const int64_t rows = static_cast<int64_t>(a.B) * a.Hq * a.NqP;
  a.row_nlse = static_cast<float*>(workspace);
  a.row_ndelta = a.row_nlse + rows;
  a.Dp = static_cast<int>(fused_dq_cols(head_dim, deterministic));
  a.dq_acc = a.Dp > 0 ? a.row_ndelta + rows : nullptr;  // 512-byte aligned: NqP is a multiple of 128
  a.scale = softmax_scale;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  return kf::fa::launch_bwd(a, dtype, static_cast<cudaStream_t>(stream));
}
