// FlashAttention forward / forward-mode JVP, general path (any head dim <= 256, multiple of 8).
//
// Three modes share one kernel template (per CTA: 64 query rows of one (batch, head); per warp:
// 16 rows; key tiles of BN rows streamed through a two-stage cp.async ring):
//
//  kModeFwd     O, LSE                       S = QK^T, online softmax, U += E V
//  kModeJvp     tO from cached O and LSE     (flash_attention_jvp/custom.py:12-120)
//                 P = exp(gamma S - LSE), H = P * gamma (tQ K^T + Q tK^T), c += rowsum(H)
//                 tO = P tV + H V - c * O
//  kModeFwdJvp  O, LSE and tO in one pass   (flash-attention-jvp-derivation.md, sec. 7-8)
//                 m, l, U, r, G online: E = exp(S - m), H = E * dS, l += rowsum(E),
//                 U += E V, r += rowsum(H), G += H V + E tV;  O = U/l, tO = G/l - (r/l) O
//
// Masking follows FlashAttention: keys >= Nk are invalid; with `causal`, key j is visible to
// query i iff j <= i + Nk - Nq (bottom-right aligned). Rows without a visible key produce
// O = 0, tO = 0 and LSE = +inf. A NULL tangent pointer means a zero tangent and skips its
// GEMM. All tensors are contiguous [B, N, H, D]; LSE is fp32 [B, Hq, Nq] (natural log).
//
// This path covers every shape the reference harness uses; the tcgen05 kernels
// (fa_sm100.cu) take the head dims the benchmark runs.
#include "fa_common.cuh"

namespace {

using kf::fa::FaArgs;
using kf::fa::kModeFwd;
using kf::fa::kModeFwdJvp;
using kf::fa::kModeJvp;

constexpr int kBM = 64;  // query rows per CTA (16 per warp)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

using namespace kf::fa::tile;

template <typename T, int DP, int BN, int DSPLIT, int MODE>
__global__ void __launch_bounds__(128 * DSPLIT)
fa_general_kernel(const FaArgs p) {
  constexpr int kThreads = 128 * DSPLIT;
  constexpr int kPitch = Pitch<DP>::value;
  constexpr bool kJvp = MODE != kModeFwd;
  constexpr bool kFwd = MODE != kModeJvp;
  constexpr int kDPW = DP / DSPLIT;  // output columns per warp
  constexpr int kNT = BN / 8;        // score n-tiles
  constexpr int kDT = kDPW / 8;      // output n-tiles
  constexpr int kQTile = kBM * kPitch * 2;
  constexpr int kKTile = BN * kPitch * 2;
  constexpr int kKV = kJvp ? 4 : 2;  // K, V (+ tK, tV) tiles per stage
  static_assert(DP % 16 == 0 && kDPW % 16 == 0 && BN % 16 == 0, "tile shapes");

  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s_q = kf::smem_u32(smem);
  const uint32_t s_tq = s_q + kQTile;
  const uint32_t s_kv = s_q + (kJvp ? 2 : 1) * kQTile;  // stage s, tensor t: s_kv + (s*kKV + t)*kKTile

  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wrow = (warp & 3) * 16;         // warp's first row within the CTA tile
  const int col0 = (warp >> 2) * kDPW;      // warp's first output column
  const int gid = lane >> 2, tig = lane & 3;
  const int q0 = qtile * kBM;
  const int kvh = h / (p.Hq / p.Hkv);
  const int D = p.D;
  const int64_t q_stride = static_cast<int64_t>(p.Hq) * D;   // between tokens
  const int64_t k_stride = static_cast<int64_t>(p.Hkv) * D;
  const int64_t q_off = (static_cast<int64_t>(b) * p.Nq * p.Hq + h) * D;
  const int64_t k_off = (static_cast<int64_t>(b) * p.Nk * p.Hkv + kvh) * D;
  const T* Q = static_cast<const T*>(p.q) + q_off;
  const T* K = static_cast<const T*>(p.k) + k_off;
  const T* V = static_cast<const T*>(p.v) + k_off;
  const T* TQ = p.tq ? static_cast<const T*>(p.tq) + q_off : nullptr;
  const T* TK = p.tk ? static_cast<const T*>(p.tk) + k_off : nullptr;
  const T* TV = p.tv ? static_cast<const T*>(p.tv) + k_off : nullptr;

  int k_end = p.Nk;
  if (p.causal) k_end = min(p.Nk, max(0, q0 + kBM + p.Nk - p.Nq));
  const int ntiles = (k_end + BN - 1) / BN;

  const int q_valid = min(kBM, p.Nq - q0);
  load_tile<T, DP, kThreads>(s_q, Q + q0 * q_stride, q_stride, kBM, q_valid, D);
  if (kJvp && TQ) load_tile<T, DP, kThreads>(s_tq, TQ + q0 * q_stride, q_stride, kBM, q_valid, D);
  cp_async_commit();
  auto load_kv = [&](int tile, int stage) {
    const int k0 = tile * BN;
    const int valid = min(BN, p.Nk - k0);
    const uint32_t base = s_kv + stage * kKV * kKTile;
    load_tile<T, DP, kThreads>(base, K + k0 * k_stride, k_stride, BN, valid, D);
    load_tile<T, DP, kThreads>(base + kKTile, V + k0 * k_stride, k_stride, BN, valid, D);
    if (kJvp && TK) load_tile<T, DP, kThreads>(base + 2 * kKTile, TK + k0 * k_stride, k_stride, BN, valid, D);
    if (kJvp && TV) load_tile<T, DP, kThreads>(base + 3 * kKTile, TV + k0 * k_stride, k_stride, BN, valid, D);
  };
  if (ntiles > 0) load_kv(0, 0);
  cp_async_commit();

  // Per-lane rows: r_lo = wrow + gid, r_hi = r_lo + 8 (global q0 + ...).
  const int row_g[2] = {q0 + wrow + gid, q0 + wrow + gid + 8};
  float lse_l2[2] = {0.f, 0.f};
  if constexpr (MODE == kModeJvp) {
#pragma unroll
    for (int i = 0; i < 2; ++i)
      lse_l2[i] = row_g[i] < p.Nq ? p.lse_in[(static_cast<int64_t>(b) * p.Hq + h) * p.Nq + row_g[i]] * kLog2e
                                  : __int_as_float(0x7f800000);
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f}, r_run[2] = {0.f, 0.f};
  float acc_o[kFwd ? kDT : 1][4];
  float acc_t[kJvp ? kDT : 1][4];
#pragma unroll
  for (int i = 0; i < (kFwd ? kDT : 1); ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc_o[i][j] = 0.f;
#pragma unroll
  for (int i = 0; i < (kJvp ? kDT : 1); ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc_t[i][j] = 0.f;

  const bool has_tq = kJvp && TQ != nullptr;
  const bool has_tk = kJvp && TK != nullptr;
  const bool has_tv = kJvp && TV != nullptr;

  for (int j = 0; j < ntiles; ++j) {
    if (j + 1 < ntiles) load_kv(j + 1, (j + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t st = s_kv + (j & 1) * kKV * kKTile;
    const uint32_t s_k = st, s_v = st + kKTile, s_tk = st + 2 * kKTile, s_tv = st + 3 * kKTile;

    // ---- scores S = Q K^T and score tangents dS = tQ K^T + Q tK^T (unscaled)
    float s[kNT][4], ts[kJvp ? kNT : 1][4];
#pragma unroll
    for (int i = 0; i < kNT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
    for (int i = 0; i < (kJvp ? kNT : 1); ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) ts[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DP / 16; ++ks) {
      const int arow = wrow + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int achunk = 2 * ks + (lane >> 4);
      uint32_t qa[4], tqa[4];
      kf::ldsm_x4(s_q + tile_off<kPitch>(arow, achunk), qa[0], qa[1], qa[2], qa[3]);
      if (has_tq) kf::ldsm_x4(s_tq + tile_off<kPitch>(arow, achunk), tqa[0], tqa[1], tqa[2], tqa[3]);
#pragma unroll
      for (int np = 0; np < kNT / 2; ++np) {
        const int brow = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int bchunk = 2 * ks + ((lane >> 3) & 1);
        uint32_t kb[4];
        kf::ldsm_x4(s_k + tile_off<kPitch>(brow, bchunk), kb[0], kb[1], kb[2], kb[3]);
        kf::Mma<T>::run(s[2 * np], qa, kb);
        kf::Mma<T>::run(s[2 * np + 1], qa, kb + 2);
        if constexpr (kJvp) {
          if (has_tq) {
            kf::Mma<T>::run(ts[2 * np], tqa, kb);
            kf::Mma<T>::run(ts[2 * np + 1], tqa, kb + 2);
          }
          if (has_tk) {
            uint32_t tkb[4];
            kf::ldsm_x4(s_tk + tile_off<kPitch>(brow, bchunk), tkb[0], tkb[1], tkb[2], tkb[3]);
            kf::Mma<T>::run(ts[2 * np], qa, tkb);
            kf::Mma<T>::run(ts[2 * np + 1], qa, tkb + 2);
          }
        }
      }
    }

    // ---- masking and probabilities (in log2 units: x = gamma * log2(e) * S)
    const int k0 = j * BN;
    float alpha[2] = {1.f, 1.f};
    if constexpr (MODE != kModeJvp) {
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + nt * 8 + tig * 2 + (e & 1);
          const int ri = e >> 1;
          const bool valid = key < p.Nk && (!p.causal || key <= row_g[ri] + p.Nk - p.Nq);
          const float x = valid ? s[nt][e] * p.scale_log2 : -INFINITY;
          s[nt][e] = x;
          mx[ri] = fmaxf(mx[ri], x);
        }
#pragma unroll
      for (int ri = 0; ri < 2; ++ri) {
        mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
        mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
        const float m_new = fmaxf(m_run[ri], mx[ri]);
        const float m_ref = m_new == -INFINITY ? 0.f : m_new;  // no (-inf) - (-inf)
        alpha[ri] = exp2f(m_run[ri] - m_ref);
        m_run[ri] = m_new;
        mx[ri] = m_ref;
      }
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] = exp2f(s[nt][e] - mx[e >> 1]);  // exp2(-inf) = 0
    } else {
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + nt * 8 + tig * 2 + (e & 1);
          const int ri = e >> 1;
          const bool valid = key < p.Nk && (!p.causal || key <= row_g[ri] + p.Nk - p.Nq);
          s[nt][e] = valid ? exp2f(s[nt][e] * p.scale_log2 - lse_l2[ri]) : 0.f;
        }
    }
    // H = P * gamma * dS and the row sums (per lane; reduced over the quad at the end)
    float lsum[2] = {0.f, 0.f}, hsum[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        lsum[e >> 1] += s[nt][e];
        if constexpr (kJvp) {
          ts[nt][e] = s[nt][e] * ts[nt][e] * p.scale;
          hsum[e >> 1] += ts[nt][e];
        }
      }
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      l_run[ri] = alpha[ri] * l_run[ri] + lsum[ri];
      r_run[ri] = alpha[ri] * r_run[ri] + hsum[ri];
    }
    if constexpr (MODE != kModeJvp) {
#pragma unroll
      for (int dt = 0; dt < kDT; ++dt) {
        acc_o[dt][0] *= alpha[0]; acc_o[dt][1] *= alpha[0];
        acc_o[dt][2] *= alpha[1]; acc_o[dt][3] *= alpha[1];
        if constexpr (kJvp) {
          acc_t[dt][0] *= alpha[0]; acc_t[dt][1] *= alpha[0];
          acc_t[dt][2] *= alpha[1]; acc_t[dt][3] *= alpha[1];
        }
      }
    }

    // ---- output GEMMs: P / E and H (bf16 / fp16 A fragments) times V, tV
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t pa[4], ha[4];
      pa[0] = kf::Mma<T>::from_f2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = kf::Mma<T>::from_f2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = kf::Mma<T>::from_f2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = kf::Mma<T>::from_f2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      if constexpr (kJvp) {
        ha[0] = kf::Mma<T>::from_f2(ts[2 * kk][0], ts[2 * kk][1]);
        ha[1] = kf::Mma<T>::from_f2(ts[2 * kk][2], ts[2 * kk][3]);
        ha[2] = kf::Mma<T>::from_f2(ts[2 * kk + 1][0], ts[2 * kk + 1][1]);
        ha[3] = kf::Mma<T>::from_f2(ts[2 * kk + 1][2], ts[2 * kk + 1][3]);
      }
      const int vrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int dp = 0; dp < kDT / 2; ++dp) {
        const int vchunk = (col0 + dp * 16) / 8 + (lane >> 4);
        uint32_t vb[4];
        kf::ldsm_x4_t(s_v + tile_off<kPitch>(vrow, vchunk), vb[0], vb[1], vb[2], vb[3]);
        if constexpr (kFwd) {
          kf::Mma<T>::run(acc_o[2 * dp], pa, vb);
          kf::Mma<T>::run(acc_o[2 * dp + 1], pa, vb + 2);
        }
        if constexpr (kJvp) {
          kf::Mma<T>::run(acc_t[2 * dp], ha, vb);
          kf::Mma<T>::run(acc_t[2 * dp + 1], ha, vb + 2);
          if (has_tv) {
            uint32_t tvb[4];
            kf::ldsm_x4_t(s_tv + tile_off<kPitch>(vrow, vchunk), tvb[0], tvb[1], tvb[2], tvb[3]);
            kf::Mma<T>::run(acc_t[2 * dp], pa, tvb);
            kf::Mma<T>::run(acc_t[2 * dp + 1], pa, tvb + 2);
          }
        }
      }
    }
    __syncthreads();  // the next iteration's loads overwrite this stage
  }
  cp_async_wait<0>();

  // ---- epilogue
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    l_run[ri] += __shfl_xor_sync(0xffffffffu, l_run[ri], 1);
    l_run[ri] += __shfl_xor_sync(0xffffffffu, l_run[ri], 2);
    r_run[ri] += __shfl_xor_sync(0xffffffffu, r_run[ri], 1);
    r_run[ri] += __shfl_xor_sync(0xffffffffu, r_run[ri], 2);
  }
  const T* O_in = MODE == kModeJvp ? static_cast<const T*>(p.o_in) + q_off : nullptr;
  T* O_out = kFwd ? static_cast<T*>(p.o_out) + q_off : nullptr;
  T* TO = kJvp ? static_cast<T*>(p.to_out) + q_off : nullptr;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int row = row_g[ri];
    if (row >= p.Nq) continue;
    const int64_t roff = static_cast<int64_t>(row) * q_stride;
    const float inv_l = l_run[ri] > 0.f ? 1.f / l_run[ri] : 0.f;
    if constexpr (kFwd) {
      if (col0 == 0 && tig == 0)
        p.lse_out[(static_cast<int64_t>(b) * p.Hq + h) * p.Nq + row] =
            l_run[ri] > 0.f ? (m_run[ri] + log2f(l_run[ri])) * kLn2 : __int_as_float(0x7f800000);
    }
#pragma unroll
    for (int dt = 0; dt < kDT; ++dt) {
      const int col = col0 + dt * 8 + tig * 2;
      if (col >= D) continue;
      if constexpr (MODE == kModeFwd) {
        const float o0 = acc_o[dt][2 * ri] * inv_l, o1 = acc_o[dt][2 * ri + 1] * inv_l;
        *reinterpret_cast<uint32_t*>(O_out + roff + col) = kf::Mma<T>::from_f2(o0, o1);
      } else if constexpr (MODE == kModeJvp) {
        const float2 o = kf::Mma<T>::to_f2(*reinterpret_cast<const uint32_t*>(O_in + roff + col));
        const float t0 = acc_t[dt][2 * ri] - r_run[ri] * o.x;
        const float t1 = acc_t[dt][2 * ri + 1] - r_run[ri] * o.y;
        *reinterpret_cast<uint32_t*>(TO + roff + col) = kf::Mma<T>::from_f2(t0, t1);
      } else {
        const float o0 = acc_o[dt][2 * ri] * inv_l, o1 = acc_o[dt][2 * ri + 1] * inv_l;
        const float rl = r_run[ri] * inv_l;
        const float t0 = acc_t[dt][2 * ri] * inv_l - rl * o0;
        const float t1 = acc_t[dt][2 * ri + 1] * inv_l - rl * o1;
        *reinterpret_cast<uint32_t*>(O_out + roff + col) = kf::Mma<T>::from_f2(o0, o1);
        *reinterpret_cast<uint32_t*>(TO + roff + col) = kf::Mma<T>::from_f2(t0, t1);
      }
    }
  }
}

template <typename T, int DP, int MODE>
int launch_dp(const FaArgs& a, cudaStream_t stream) {
  constexpr int DSPLIT = DP > 128 ? 2 : 1;
  constexpr int kDPW = DP / DSPLIT;
  constexpr int BN = (DSPLIT == 2 || (MODE == kModeFwdJvp && kDPW > 64)) ? 32 : 64;
  constexpr int kPitch = Pitch<DP>::value;
  constexpr bool kJvp = MODE != kModeFwd;
  const int smem = (kJvp ? 2 : 1) * kBM * kPitch * 2 + 2 * (kJvp ? 4 : 2) * BN * kPitch * 2;
  auto kernel = fa_general_kernel<T, DP, BN, DSPLIT, MODE>;
  const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), 128 * DSPLIT, smem, nullptr);
  if (prep != KF_OK) return prep;
  const dim3 grid((a.Nq + kBM - 1) / kBM, a.Hq, a.B);
  kernel<<<grid, 128 * DSPLIT, smem, stream>>>(a);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

template <typename T, int MODE>
int launch_mode(const FaArgs& a, cudaStream_t s) {
  const int d = a.D;
  if (d <= 32) return launch_dp<T, 32, MODE>(a, s);
  if (d <= 64) return launch_dp<T, 64, MODE>(a, s);
  if (d <= 96) return launch_dp<T, 96, MODE>(a, s);
  if (d <= 128) return launch_dp<T, 128, MODE>(a, s);
  if (d <= 192) return launch_dp<T, 192, MODE>(a, s);
  return launch_dp<T, 256, MODE>(a, s);
}

}  // namespace

namespace kf::fa {

int launch_general(const FaArgs& a, int mode, int dtype, cudaStream_t s) {
  if (dtype == KF_DTYPE_F16) {
    switch (mode) {
      case kModeFwd: return launch_mode<__half, kModeFwd>(a, s);
      case kModeJvp: return launch_mode<__half, kModeJvp>(a, s);
      default: return launch_mode<__half, kModeFwdJvp>(a, s);
    }
  }
  switch (mode) {
    case kModeFwd: return launch_mode<__nv_bfloat16, kModeFwd>(a, s);
    case kModeJvp: return launch_mode<__nv_bfloat16, kModeJvp>(a, s);
    default: return launch_mode<__nv_bfloat16, kModeFwdJvp>(a, s);
  }
}

}  // namespace kf::fa
