// FlashAttention backward (reverse-mode VJP) from the saved O and LSE.
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
// Three kernels, deterministic (no atomics). The first is shared with the tcgen05 kernels of
// fa_bwd_sm100.cu (head dims up to 128); the other two serve head dims 136..256:
//   fa_bwd_rowstat_kernel one warp per (batch, head, query) row: -LSE log2(e) and -delta into
//                        the padded row-statistics arrays
//   fa_bwd_dq_kernel     query-stationary: 64 query rows per CTA, key tiles streamed through a
//                        two-stage cp.async ring; S and dP by mma.sync, then dQ += dS K
//   fa_bwd_dkdv_kernel   key-stationary: 64 keys per CTA, the query tiles of every query head
//                        of the KV group streamed in order (the group sum is sequential);
//                        S^T = K Q^T and dP^T = V dO^T, then dV += P^T dO and dK += dS^T Q
// Per warp, 16 rows (queries or keys) of the CTA tile; for large head dims the output columns
// are split over warp groups (each group recomputes the score tiles). The A operands of the
// second GEMMs (P, dS and their transposes) are the first GEMMs' accumulators converted in
// registers, as in the forward.
#include "fa_common.cuh"

namespace {

using kf::fa::BwdArgs;
using namespace kf::fa::tile;

constexpr int kBM = 64;  // query rows per dQ CTA, keys per dK/dV CTA
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

// Accumulator fragments of two m16n8 tiles (keys 16 kk .. 16 kk + 15 of this warp's rows) as the
// A operand of an m16n8k16 MMA.
template <typename T>
__device__ __forceinline__ void acc_to_a(const float (&lo)[4], const float (&hi)[4], uint32_t (&a)[4]) {
  a[0] = kf::Mma<T>::from_f2(lo[0], lo[1]);
  a[1] = kf::Mma<T>::from_f2(lo[2], lo[3]);
  a[2] = kf::Mma<T>::from_f2(hi[0], hi[1]);
  a[3] = kf::Mma<T>::from_f2(hi[2], hi[3]);
}

// ------------------------------------------------------------------------------------------
// dQ: 64 query rows of one (batch, head) per CTA
// ------------------------------------------------------------------------------------------
template <typename T, int DP, int BN, int DSPLIT>
__global__ void __launch_bounds__(128 * DSPLIT) fa_bwd_dq_kernel(const BwdArgs p) {
  constexpr int kThreads = 128 * DSPLIT;
  constexpr int kPitch = Pitch<DP>::value;
  constexpr int kDPW = DP / DSPLIT;  // dQ columns per warp
  constexpr int kNT = BN / 8;        // score n-tiles
  constexpr int kDT = kDPW / 8;      // dQ n-tiles
  constexpr int kQTile = kBM * kPitch * 2;
  constexpr int kKTile = BN * kPitch * 2;
  static_assert(DP % 16 == 0 && kDPW % 16 == 0 && BN % 16 == 0, "tile shapes");

  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s_q = kf::smem_u32(smem), s_do = s_q + kQTile;
  const uint32_t s_kv = s_q + 2 * kQTile;  // stage s: K at s_kv + 2 s kKTile, V after it

  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wrow = (warp & 3) * 16;
  const int col0 = (warp >> 2) * kDPW;
  const int gid = lane >> 2, tig = lane & 3;
  const int q0 = qtile * kBM;
  const int kvh = h / (p.Hq / p.Hkv);
  const int D = p.D;
  const int64_t q_stride = static_cast<int64_t>(p.Hq) * D, k_stride = static_cast<int64_t>(p.Hkv) * D;
  const int64_t q_off = (static_cast<int64_t>(b) * p.Nq * p.Hq + h) * D;
  const int64_t k_off = (static_cast<int64_t>(b) * p.Nk * p.Hkv + kvh) * D;
  const T* Q = static_cast<const T*>(p.q) + q_off;
  const T* dO = static_cast<const T*>(p.dout) + q_off;
  const T* K = static_cast<const T*>(p.k) + k_off;
  const T* V = static_cast<const T*>(p.v) + k_off;

  int k_end = p.Nk;
  if (p.causal) k_end = min(p.Nk, max(0, q0 + kBM + p.Nk - p.Nq));
  const int ntiles = (k_end + BN - 1) / BN;

  const int q_valid = min(kBM, p.Nq - q0);
  load_tile<T, DP, kThreads>(s_q, Q + q0 * q_stride, q_stride, kBM, q_valid, D);
  load_tile<T, DP, kThreads>(s_do, dO + q0 * q_stride, q_stride, kBM, q_valid, D);
  cp_async_commit();
  auto load_kv = [&](int tile, int stage) {
    const int k0 = tile * BN;
    const int valid = min(BN, p.Nk - k0);
    const uint32_t base = s_kv + stage * 2 * kKTile;
    load_tile<T, DP, kThreads>(base, K + k0 * k_stride, k_stride, BN, valid, D);
    load_tile<T, DP, kThreads>(base + kKTile, V + k0 * k_stride, k_stride, BN, valid, D);
  };
  if (ntiles > 0) load_kv(0, 0);
  cp_async_commit();

  // Rows past Nq read the padding (-inf: P = 0); row_g < q0 + 64 <= NqP.
  const int row_g[2] = {q0 + wrow + gid, q0 + wrow + gid + 8};
  float nlse[2], ndelta[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t idx = (static_cast<int64_t>(b) * p.Hq + h) * p.NqP + row_g[i];
    nlse[i] = p.row_nlse[idx];
    ndelta[i] = p.row_ndelta[idx];
  }
  float acc[kDT][4];
#pragma unroll
  for (int i = 0; i < kDT; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    if (j + 1 < ntiles) load_kv(j + 1, (j + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t s_k = s_kv + (j & 1) * 2 * kKTile, s_v = s_k + kKTile;

    // S = Q K^T and dP = dO V^T for this warp's 16 rows
    float s[kNT][4], dp[kNT][4];
#pragma unroll
    for (int i = 0; i < kNT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DP / 16; ++ks) {
      const int arow = wrow + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int achunk = 2 * ks + (lane >> 4);
      uint32_t qa[4], da[4];
      kf::ldsm_x4(s_q + tile_off<kPitch>(arow, achunk), qa[0], qa[1], qa[2], qa[3]);
      kf::ldsm_x4(s_do + tile_off<kPitch>(arow, achunk), da[0], da[1], da[2], da[3]);
#pragma unroll
      for (int np = 0; np < kNT / 2; ++np) {
        const int brow = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int bchunk = 2 * ks + ((lane >> 3) & 1);
        uint32_t kb[4], vb[4];
        kf::ldsm_x4(s_k + tile_off<kPitch>(brow, bchunk), kb[0], kb[1], kb[2], kb[3]);
        kf::ldsm_x4(s_v + tile_off<kPitch>(brow, bchunk), vb[0], vb[1], vb[2], vb[3]);
        kf::Mma<T>::run(s[2 * np], qa, kb);
        kf::Mma<T>::run(s[2 * np + 1], qa, kb + 2);
        kf::Mma<T>::run(dp[2 * np], da, vb);
        kf::Mma<T>::run(dp[2 * np + 1], da, vb + 2);
      }
    }
    // dS = P (dP - delta), P = exp2(S gamma log2 e - LSE log2 e) on visible keys
    const int k0 = j * BN;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nt * 8 + tig * 2 + (e & 1);
        const int ri = e >> 1;
        const bool valid = key < p.Nk && (!p.causal || key <= row_g[ri] + p.Nk - p.Nq);
        const float pr = valid ? exp2f(fmaf(s[nt][e], p.scale_log2, nlse[ri])) : 0.f;
        s[nt][e] = pr * (dp[nt][e] + ndelta[ri]);
      }
    // dQ += dS K (K as the B operand: keys along k, head dim along n)
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t a[4];
      acc_to_a<T>(s[2 * kk], s[2 * kk + 1], a);
      const int vrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int dq = 0; dq < kDT / 2; ++dq) {
        const int vchunk = (col0 + dq * 16) / 8 + (lane >> 4);
        uint32_t kb[4];
        kf::ldsm_x4_t(s_k + tile_off<kPitch>(vrow, vchunk), kb[0], kb[1], kb[2], kb[3]);
        kf::Mma<T>::run(acc[2 * dq], a, kb);
        kf::Mma<T>::run(acc[2 * dq + 1], a, kb + 2);
      }
    }
    __syncthreads();  // the next iteration's loads overwrite this stage
  }
  cp_async_wait<0>();

  T* dQ = static_cast<T*>(p.dq) + q_off;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int row = row_g[ri];
    if (row >= p.Nq) continue;
    const int64_t roff = static_cast<int64_t>(row) * q_stride;
#pragma unroll
    for (int dt = 0; dt < kDT; ++dt) {
      const int col = col0 + dt * 8 + tig * 2;
      if (col >= D) continue;
      *reinterpret_cast<uint32_t*>(dQ + roff + col) =
          kf::Mma<T>::from_f2(acc[dt][2 * ri] * p.scale, acc[dt][2 * ri + 1] * p.scale);
    }
  }
}

// ------------------------------------------------------------------------------------------
// dK, dV: 64 keys of one (batch, KV head) per CTA; all query heads of the group, in order
// ------------------------------------------------------------------------------------------
template <typename T, int DP, int BQ, int DSPLIT>
__global__ void __launch_bounds__(128 * DSPLIT) fa_bwd_dkdv_kernel(const BwdArgs p) {
  constexpr int kThreads = 128 * DSPLIT;
  constexpr int kPitch = Pitch<DP>::value;
  constexpr int kDPW = DP / DSPLIT;  // dK / dV columns per warp
  constexpr int kNT = BQ / 8;        // query n-tiles of the transposed scores
  constexpr int kDT = kDPW / 8;
  constexpr int kKTile = kBM * kPitch * 2;
  constexpr int kQTile = BQ * kPitch * 2;
  constexpr int kStageBytes = 2 * kQTile + 2 * BQ * 4;  // Q, dO tiles; LSE (log2), delta
  static_assert(DP % 16 == 0 && kDPW % 16 == 0 && BQ % 16 == 0, "tile shapes");

  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s_k = kf::smem_u32(smem), s_v = s_k + kKTile;
  uint8_t* const stages = smem + 2 * kKTile;

  const int ktile = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wrow = (warp & 3) * 16;
  const int col0 = (warp >> 2) * kDPW;
  const int gid = lane >> 2, tig = lane & 3;
  const int k0 = ktile * kBM;
  const int group = p.Hq / p.Hkv;
  const int D = p.D;
  const int64_t q_stride = static_cast<int64_t>(p.Hq) * D, k_stride = static_cast<int64_t>(p.Hkv) * D;
  const int64_t k_off = (static_cast<int64_t>(b) * p.Nk * p.Hkv + kvh) * D;
  const T* K = static_cast<const T*>(p.k) + k_off;
  const T* V = static_cast<const T*>(p.v) + k_off;

  // Query tiles that see at least one of these keys: key k is visible to query i iff
  // k <= i + Nk - Nq (causal), so queries below k0 - (Nk - Nq) see none of them.
  const int q_first = p.causal ? max(0, k0 - (p.Nk - p.Nq)) : 0;
  const int qt_first = q_first / BQ;
  const int qt_count = max(0, (p.Nq + BQ - 1) / BQ - qt_first);
  const int n_it = group * qt_count;

  const int k_valid = min(kBM, p.Nk - k0);
  load_tile<T, DP, kThreads>(s_k, K + k0 * k_stride, k_stride, kBM, k_valid, D);
  load_tile<T, DP, kThreads>(s_v, V + k0 * k_stride, k_stride, kBM, k_valid, D);
  cp_async_commit();
  auto load_stage = [&](int it, int stage) {
    const int h = kvh * group + it / qt_count;
    const int q0 = (qt_first + it % qt_count) * BQ;
    const int64_t q_off = (static_cast<int64_t>(b) * p.Nq * p.Hq + h) * D;
    uint8_t* st = stages + stage * kStageBytes;
    const uint32_t s_q = kf::smem_u32(st);
    const int valid = min(BQ, p.Nq - q0);
    load_tile<T, DP, kThreads>(s_q, static_cast<const T*>(p.q) + q_off + q0 * q_stride, q_stride, BQ, valid, D);
    load_tile<T, DP, kThreads>(s_q + kQTile, static_cast<const T*>(p.dout) + q_off + q0 * q_stride, q_stride, BQ,
                               valid, D);
    float* nlse_s = reinterpret_cast<float*>(st + 2 * kQTile);
    float* ndelta_s = nlse_s + BQ;
    for (int i = threadIdx.x; i < BQ; i += kThreads) {
      const int64_t idx = (static_cast<int64_t>(b) * p.Hq + h) * p.NqP + q0 + i;  // q0 + i < NqP
      nlse_s[i] = p.row_nlse[idx];
      ndelta_s[i] = p.row_ndelta[idx];
    }
  };
  if (n_it > 0) load_stage(0, 0);
  cp_async_commit();

  const int key_g[2] = {k0 + wrow + gid, k0 + wrow + gid + 8};
  float dk[kDT][4], dv[kDT][4];
#pragma unroll
  for (int i = 0; i < kDT; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  for (int it = 0; it < n_it; ++it) {
    if (it + 1 < n_it) load_stage(it + 1, (it + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    uint8_t* st = stages + (it & 1) * kStageBytes;
    const uint32_t s_q = kf::smem_u32(st), s_do = s_q + kQTile;
    const float* nlse_s = reinterpret_cast<const float*>(st + 2 * kQTile);
    const float* ndelta_s = nlse_s + BQ;
    const int q0 = (qt_first + it % qt_count) * BQ;

    // S^T = K Q^T and dP^T = V dO^T for this warp's 16 keys
    float sT[kNT][4], dpT[kNT][4];
#pragma unroll
    for (int i = 0; i < kNT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) sT[i][e] = dpT[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DP / 16; ++ks) {
      const int arow = wrow + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int achunk = 2 * ks + (lane >> 4);
      uint32_t ka[4], va[4];
      kf::ldsm_x4(s_k + tile_off<kPitch>(arow, achunk), ka[0], ka[1], ka[2], ka[3]);
      kf::ldsm_x4(s_v + tile_off<kPitch>(arow, achunk), va[0], va[1], va[2], va[3]);
#pragma unroll
      for (int np = 0; np < kNT / 2; ++np) {
        const int brow = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int bchunk = 2 * ks + ((lane >> 3) & 1);
        uint32_t qb[4], db[4];
        kf::ldsm_x4(s_q + tile_off<kPitch>(brow, bchunk), qb[0], qb[1], qb[2], qb[3]);
        kf::ldsm_x4(s_do + tile_off<kPitch>(brow, bchunk), db[0], db[1], db[2], db[3]);
        kf::Mma<T>::run(sT[2 * np], ka, qb);
        kf::Mma<T>::run(sT[2 * np + 1], ka, qb + 2);
        kf::Mma<T>::run(dpT[2 * np], va, db);
        kf::Mma<T>::run(dpT[2 * np + 1], va, db + 2);
      }
    }
    // P^T and dS^T = P^T (dP^T - delta) on visible (key, query) pairs
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + tig * 2 + (e & 1);
        const int q = q0 + qi;
        const int key = key_g[e >> 1];
        const bool valid = q < p.Nq && key < p.Nk && (!p.causal || key <= q + p.Nk - p.Nq);
        const float pr = valid ? exp2f(fmaf(sT[nt][e], p.scale_log2, nlse_s[qi])) : 0.f;
        sT[nt][e] = pr;
        dpT[nt][e] = pr * (dpT[nt][e] + ndelta_s[qi]);
      }
    // dV += P^T dO and dK += dS^T Q (dO, Q as B operands: queries along k, head dim along n)
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t pa[4], sa[4];
      acc_to_a<T>(sT[2 * kk], sT[2 * kk + 1], pa);
      acc_to_a<T>(dpT[2 * kk], dpT[2 * kk + 1], sa);
      const int vrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int dd = 0; dd < kDT / 2; ++dd) {
        const int vchunk = (col0 + dd * 16) / 8 + (lane >> 4);
        uint32_t ob[4], qb[4];
        kf::ldsm_x4_t(s_do + tile_off<kPitch>(vrow, vchunk), ob[0], ob[1], ob[2], ob[3]);
        kf::ldsm_x4_t(s_q + tile_off<kPitch>(vrow, vchunk), qb[0], qb[1], qb[2], qb[3]);
        kf::Mma<T>::run(dv[2 * dd], pa, ob);
        kf::Mma<T>::run(dv[2 * dd + 1], pa, ob + 2);
        kf::Mma<T>::run(dk[2 * dd], sa, qb);
        kf::Mma<T>::run(dk[2 * dd + 1], sa, qb + 2);
      }
    }
    __syncthreads();  // the next iteration's loads overwrite this stage
  }
  cp_async_wait<0>();

  T* dK = static_cast<T*>(p.dk) + k_off;
  T* dV = static_cast<T*>(p.dv) + k_off;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int key = key_g[ri];
    if (key >= p.Nk) continue;
    const int64_t roff = static_cast<int64_t>(key) * k_stride;
#pragma unroll
    for (int dt = 0; dt < kDT; ++dt) {
      const int col = col0 + dt * 8 + tig * 2;
      if (col >= D) continue;
      *reinterpret_cast<uint32_t*>(dK + roff + col) =
          kf::Mma<T>::from_f2(dk[dt][2 * ri] * p.scale, dk[dt][2 * ri + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dV + roff + col) = kf::Mma<T>::from_f2(dv[dt][2 * ri], dv[dt][2 * ri + 1]);
    }
  }
}

template <typename T, int DP>
int launch_dp(const BwdArgs& a, cudaStream_t stream) {
  constexpr int kPitch = Pitch<DP>::value;
  {
    constexpr int DSPLIT = DP > 128 ? 2 : 1;
    constexpr int BN = DP > 128 ? 32 : 64;
    const int smem = 2 * kBM * kPitch * 2 + 2 * 2 * BN * kPitch * 2;
    auto kernel = fa_bwd_dq_kernel<T, DP, BN, DSPLIT>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), 128 * DSPLIT, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3((a.Nq + kBM - 1) / kBM, a.Hq, a.B), 128 * DSPLIT, smem, stream>>>(a);
    KF_LAUNCH_CHECK();
  }
  {
    constexpr int DSPLIT = DP <= 64 ? 1 : (DP <= 128 ? 2 : 4);
    constexpr int BQ = DP > 128 ? 32 : 64;
    const int smem = 2 * kBM * kPitch * 2 + 2 * (2 * BQ * kPitch * 2 + 2 * BQ * 4);
    auto kernel = fa_bwd_dkdv_kernel<T, DP, BQ, DSPLIT>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), 128 * DSPLIT, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3((a.Nk + kBM - 1) / kBM, a.Hkv, a.B), 128 * DSPLIT, smem, stream>>>(a);
    KF_LAUNCH_CHECK();
  }
  return KF_OK;
}

template <typename T>
int launch_t(const BwdArgs& a, int dtype, cudaStream_t s) {
  {
    const int64_t rows = static_cast<int64_t>(a.B) * a.Hq * a.NqP;
    fa_bwd_rowstat_kernel<T><<<static_cast<unsigned int>((rows + 7) / 8), 256, 0, s>>>(a);
    KF_LAUNCH_CHECK();
  }
  if (kf::fa::sm100_bwd_supported(a)) return kf::fa::launch_sm100_bwd(a, dtype, s);
  const int d = a.D;
  // Head dims up to 128 went to the tcgen05 kernels above; these serve 136..256.
  if (d <= 192) return launch_dp<T, 192>(a, s);
  return launch_dp<T, 256>(a, s);
}

}  // namespace

namespace kf::fa {

int launch_bwd(const BwdArgs& a, int dtype, cudaStream_t s) {
  return dtype == KF_DTYPE_F16 ? launch_t<__half>(a, dtype, s) : launch_t<__nv_bfloat16>(a, dtype, s);
}

}  // namespace kf::fa
