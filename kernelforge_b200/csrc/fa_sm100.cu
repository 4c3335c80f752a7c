// FlashAttention forward-mode JVP and forward on the 5th-generation tensor cores (tcgen05 + TMEM
// + TMA), head dims up to 256.
//
// Standalone JVP from a cached O and LSE (flash_attention_jvp/custom.py:12-120):
//   P  = exp(gamma * Q K^T - LSE)                     (keys masked to 0)
//   H  = P * gamma * (tQ K^T + Q tK^T)
//   tO = P tV + H V - rowsum(H) * O
//
// One CTA owns 128 query rows of one (batch, head); in each softmax warpgroup one thread owns
// one row (= one TMEM lane). Warp roles:
//   warps 0..7  two softmax warpgroups; in the standalone JVP both work on every 64-key tile,
//               warpgroup g on keys [32 g, 32 g + 32): they turn scores into P, H (16-bit A
//               operands written back to TMEM) and row sums; at the end both add their row sums
//               and split the epilogue by columns
//   warp 8      TMA producer: Q, tQ once; rings of {K, tK} and {V, tV} tiles of 64 keys
//   warp 9      TMEM owner; one thread issues the score MMAs (runs ahead while buffers allow)
//   warp 10     one thread issues the output MMAs as each tile's P / H become ready
// Two issuing threads keep the tensor core's short instruction queue fed: while one waits on a
// barrier the other issues.
// Double-buffered S / dS in tensor memory let the tensor core compute tile j+1's scores while
// the softmax warps turn tile j into P and H. Per 64-key tile the MMA warp issues
//   [S | Q tK^T] = Q [K ; tK]^T   (D/16 x M128 N128 K16, operands from shared memory)
//   dS += tQ K^T                   (D/16 x M128 N64 K16)
//   tO += P tV + H V               (2 x 4 x M128 N=D K16, A from tensor memory, B MN-major)
// All operand tiles arrive by TMA with 128-byte swizzle; every wait is a bounded mbarrier
// wait that records KF_ERR_DEVICE_TIMEOUT in the module's error word and gives up.
#include "fa_common.cuh"
#include "kf_tcgen05.cuh"

namespace {

using kf::fa::FaArgs;
using kf::fa::encode_bnhd;

__device__ unsigned int g_fa_error = 0;

constexpr int kBM = 128;       // query rows per CTA (one TMEM lane each)
constexpr int kBN = 64;        // keys per tile
constexpr int kThreads = 352;  // 11 warps
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;     // TMEM owner; issues the score MMAs
constexpr int kPvWarp = 10;     // issues the output MMAs
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol = 0;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxScoreBufs = 3;

// Shared-memory plan: Q, tQ once; a ring of {K, tK} stages (a stage is free again once the
// tile's score MMAs complete: k_empty) and a separate ring of {V, tV} stages (free once the
// tile's output MMAs complete: v_empty), so K and V tiles stream in ahead of their use (a TMA
// load of a tile from L2 takes ~1000-1400 cycles, about one tile period). D = 64 has room for
// four stages of each; D = 128 (32 KB stages next to 64 KB of Q and tQ) for two.
// kTan: room for the tangents tQ, tK, tV next to Q, K, V (the forward alone has none, which
// leaves room for D = 256: 64 KB of Q and two stages of 32 KB K and V tiles). BN: keys per tile.
// The standalone JVP at D = 256 (128 KB of Q and tQ) takes 32-key tiles, two K stages and one V
// stage: 224 KB.
template <int D, bool kTan = true, int BN = kBN> struct Cfg {
  static constexpr int kKB = D / 64;                    // 128-byte boxes along the head dim
  static constexpr int kQBytes = kKB * kBM * 128;       // Q or tQ
  static constexpr int kTileBytes = kKB * BN * 128;     // K, tK, V or tV of one tile
  static constexpr int kKBox = BN * 128;                // one 128-byte box of a K or tK tile
  // A K stage holds the boxes of K and tK interleaved, [K box 0 | tK box 0 | K box 1 | ...]:
  // box kb of K and of tK together are the 128 rows of one N = 128 operand [K ; tK].
  static constexpr int kKPair = kTan ? 2 * kKBox : kKBox;  // K box kb to K box kb + 1
  static constexpr int kStageBytes = kTan ? 2 * kTileBytes : kTileBytes;  // {K, tK} or {V, tV}
  // The forward at D = 128 takes three K stages (the one-pass kernel's three score buffers need
  // as many: a buffer's "free" arrival for tile j + 3 lands in that tile's K stage).
  static constexpr int kKStages = D == 64 ? 4 : (D == 128 && !kTan ? 3 : 2);
  // The V ring needs as many stages as the one-pass kernel has score buffers: the softmax
  // threads' arrival for tile j lands on V stage j % kVStages, and what lets them reach tile
  // j + NB (the output MMAs of tile j) proves only that the V phases before tile j completed.
  static constexpr int kVStages = D == 64 ? 4 : (D == 128 && !kTan ? 3 : (D == 256 && kTan ? 1 : 2));
  static constexpr int kKOffset = kTan ? 2 * kQBytes : kQBytes;
  static constexpr int kVOffset = kKOffset + kKStages * kStageBytes;
  static constexpr int kBarOffset = kVOffset + kVStages * kStageBytes;
  // Tensor memory: S of score buffer b at kBufCol + 128 b, dS 64 columns further; the
  // accumulators below kBufCol.
  static constexpr uint32_t kBufCol = D <= 128 ? 128 : 256;
  static constexpr int kScratchOffset = kBarOffset + 512;  // row statistics
  // [2][kBM] row sums (standalone JVP) or [8][kBM] maxima and sums (one-pass kernel)
  static constexpr int kScratchBytes = (D == 256 && kTan ? 2 : 8) * kBM * 4;
  static constexpr int kSmemBytes = kScratchOffset + kScratchBytes + 64 + 1024;  // + abort flag, slack
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// Barriers, in shared memory after the operand tiles.
template <int D, bool kTan = true, int BN = kBN> struct Bars {
  uint64_t* q_full;
  uint64_t* k_full;   // [kKStages] K / tK of the stage's tile landed (+ k_extra arrivals)
  uint64_t* k_empty;  // [kKStages] the score MMAs of the stage's tile completed
  uint64_t* v_full;   // [kVStages] V / tV of the stage's tile landed (+ v_extra arrivals)
  uint64_t* v_empty;  // [kVStages] the output MMAs of the stage's tile completed
  uint64_t* s_full;   // [kMaxScoreBufs] scores of tile j complete
  uint64_t* p_full;   // [kMaxScoreBufs] P / H of tile j written
  uint64_t* pv_done;  // [kMaxScoreBufs] output MMAs of tile j complete
  uint64_t* acc_full;
  uint32_t* tmem_slot;
  __device__ explicit Bars(uint8_t* smem) {
    using C = Cfg<D, kTan, BN>;
    q_full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    k_full = q_full + 1;
    k_empty = k_full + C::kKStages;
    v_full = k_empty + C::kKStages;
    v_empty = v_full + C::kVStages;
    s_full = v_empty + C::kVStages;
    p_full = s_full + kMaxScoreBufs;
    pv_done = p_full + kMaxScoreBufs;
    acc_full = pv_done + kMaxScoreBufs;
    tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  }
  // k_extra / v_extra: arrivals besides the producer's that complete a K or V stage. The kernels
  // fold "score buffer j & 1 free" into the k_full phase of tile j and "P / H of tile j written"
  // into v_full, so each MMA thread waits on one barrier per tile.
  __device__ void init(int p_arrivals, int k_extra, int v_extra) const {
    using C = Cfg<D, kTan, BN>;
    kf::mbar_init(q_full, 1);
    for (int s = 0; s < C::kKStages; ++s) {
      kf::mbar_init(&k_full[s], 1 + k_extra);
      kf::mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::kVStages; ++s) {
      kf::mbar_init(&v_full[s], 1 + v_extra);
      kf::mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < kMaxScoreBufs; ++i) {
      kf::mbar_init(&s_full[i], 1);
      kf::mbar_init(&p_full[i], p_arrivals);
      kf::mbar_init(&pv_done[i], 1);
    }
    kf::mbar_init(acc_full, 1);
  }
};

// TMA producer (one thread): Q, tQ, then K tiles one ahead of V tiles -- the order in which
// the MMA warp consumes them -- each behind its ring's "empty" barrier.
template <int D, bool kTan, int BN>
__device__ void produce(const Bars<D, kTan, BN>& bars, uint8_t* smem, const CUtensorMap* tm_q, const CUtensorMap* tm_tq,
                        const CUtensorMap* tm_k, const CUtensorMap* tm_tk, const CUtensorMap* tm_v,
                        const CUtensorMap* tm_tv, bool has_tq, bool has_tk, bool need_v, bool has_tv,
                        int h, int kvh, int q0, int b, int ntiles, volatile int* abort) {
  using C = Cfg<D, kTan, BN>;
  kf::prefetch_tensormap(tm_q);
  kf::prefetch_tensormap(tm_k);
  kf::mbar_arrive_expect_tx(bars.q_full, C::kQBytes * (has_tq ? 2 : 1));
  for (int kb = 0; kb < C::kKB; ++kb) {
    kf::tma_load_4d(smem + kb * kBM * 128, tm_q, bars.q_full, kb * 64, h, q0, b);
    if (has_tq) kf::tma_load_4d(smem + C::kQBytes + kb * kBM * 128, tm_tq, bars.q_full, kb * 64, h, q0, b);
  }
  const uint32_t k_bytes = C::kTileBytes * (has_tk ? 2 : 1);
  const uint32_t v_bytes = C::kTileBytes * ((need_v ? 1 : 0) + (has_tv ? 1 : 0));
  auto load_k = [&](int j) -> bool {
    const int st = j % C::kKStages;  // last read by the score MMAs of tile j - kKStages
    if (j >= C::kKStages &&
        !kf::mbar_wait_or_abort<true>(&bars.k_empty[st], (j / C::kKStages - 1) & 1, &g_fa_error, abort))
      return false;
    uint8_t* base = smem + C::kKOffset + st * C::kStageBytes;
    kf::mbar_arrive_expect_tx(&bars.k_full[st], k_bytes);
    for (int kb = 0; kb < C::kKB; ++kb) {  // boxes interleaved: K kb, tK kb (kKPair bytes apart)
      kf::tma_load_4d(base + kb * C::kKPair, tm_k, &bars.k_full[st], kb * 64, kvh, j * BN, b);
      if (has_tk) kf::tma_load_4d(base + kb * C::kKPair + C::kKBox, tm_tk, &bars.k_full[st], kb * 64, kvh, j * BN, b);
    }
    return true;
  };
  auto load_v = [&](int j) -> bool {
    const int st = j % C::kVStages;  // last read by the output MMAs of tile j - kVStages
    if (j >= C::kVStages &&
        !kf::mbar_wait_or_abort<true>(&bars.v_empty[st], (j / C::kVStages - 1) & 1, &g_fa_error, abort))
      return false;
    uint8_t* base = smem + C::kVOffset + st * C::kStageBytes;
    kf::mbar_arrive_expect_tx(&bars.v_full[st], v_bytes);
    for (int kb = 0; kb < C::kKB; ++kb) {
      if (need_v) kf::tma_load_4d(base + kb * C::kKBox, tm_v, &bars.v_full[st], kb * 64, kvh, j * BN, b);
      if (has_tv) kf::tma_load_4d(base + C::kTileBytes + kb * C::kKBox, tm_tv, &bars.v_full[st], kb * 64, kvh, j * BN, b);
    }
    return true;
  };
  // K tiles run up to kKStages - 1 ahead of V tiles: the score MMAs of tile j+1 come before the
  // output MMAs of tile j.
  int kj = 0;
  for (int j = 0; j < ntiles; ++j) {
    for (; kj < ntiles && kj < j + C::kKStages; ++kj)
      if (!load_k(kj)) return;
    if (!load_v(j)) return;
  }
}

// 128-byte-swizzle descriptor of the matrix `off` bytes past `base`: the descriptor of `base`
// (loop-invariant, built once per tile) plus the offset, so each K step costs one add.
__device__ __forceinline__ uint64_t dsw(uint32_t base, uint32_t off, uint32_t lbo) {
  return kf::tc::desc_advance(kf::tc::desc_sw128(base, lbo, 1024), off);
}

// Score MMAs of tile j: S = Q K^T into s_col, then dS = tQ K^T + Q tK^T into ts_col.
template <int D, int kKPair>
__device__ __forceinline__ void issue_s(uint32_t q_addr, uint32_t k_base, uint32_t s_col, uint32_t idS) {
#pragma unroll
  for (int k = 0; k < D / 16; ++k) {
    const uint32_t off = (k >> 2) * kBM * 128 + (k & 3) * 32;
    const uint32_t koff = (k >> 2) * kKPair + (k & 3) * 32;
    kf::tc::mma_ss(s_col, dsw(q_addr, off, 16), dsw(k_base, koff, 16),
                   idS, k > 0);
  }
}
template <int D, int kKPair, int kKBox>
__device__ __forceinline__ void issue_ds(uint32_t q_addr, uint32_t tq_addr, uint32_t k_base,
                                         uint32_t ts_col, uint32_t idS, bool has_tq, bool has_tk) {
  uint32_t started = 0;
  if (has_tq) {
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      const uint32_t off = (k >> 2) * kBM * 128 + (k & 3) * 32;
      const uint32_t koff = (k >> 2) * kKPair + (k & 3) * 32;
      kf::tc::mma_ss(ts_col, dsw(tq_addr, off, 16),
                     dsw(k_base, koff, 16), idS, started);
      started = 1;
    }
  }
  if (has_tk) {
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      const uint32_t off = (k >> 2) * kBM * 128 + (k & 3) * 32;
      const uint32_t koff = (k >> 2) * kKPair + kKBox + (k & 3) * 32;
      kf::tc::mma_ss(ts_col, dsw(q_addr, off, 16),
                     dsw(k_base, koff, 16), idS, started);
      started = 1;
    }
  }
}

// S into s_col and dS into s_col + BN for one key tile. An N = 64 MMA with both operands in
// shared memory reads 6 KB per K step against 8 KB for N = 128 in twice the tensor time, so it
// is bound by shared-memory bandwidth at 2/3 of the tensor core's rate. With a tangent tK,
// [S | Q tK^T] = Q [K ; tK]^T is one N = 128 MMA per K step (box kb of K and of tK are adjacent
// in the stage) and tQ K^T is added to its second half.
template <int D, int kKPair, int kKBox, int BN>
__device__ __forceinline__ void issue_scores(uint32_t q_addr, uint32_t tq_addr, uint32_t k_base,
                                             uint32_t s_col, bool has_tq, bool has_tk, bool bf16) {
  const uint32_t idS = kf::tc::idesc_f16(bf16 ? 1 : 0, kBM, BN, false, false);
  if (has_tk) {
    const uint32_t idS2 = kf::tc::idesc_f16(bf16 ? 1 : 0, kBM, 2 * BN, false, false);
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      const uint32_t off = (k >> 2) * kBM * 128 + (k & 3) * 32;
      const uint32_t koff = (k >> 2) * kKPair + (k & 3) * 32;
      kf::tc::mma_ss(s_col, dsw(q_addr, off, 16), dsw(k_base, koff, 16), idS2, k > 0);
    }
    if (has_tq) {
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint32_t off = (k >> 2) * kBM * 128 + (k & 3) * 32;
        const uint32_t koff = (k >> 2) * kKPair + (k & 3) * 32;
        kf::tc::mma_ss(s_col + BN, dsw(tq_addr, off, 16), dsw(k_base, koff, 16), idS, 1);
      }
    }
    return;
  }
  issue_s<D, kKPair>(q_addr, k_base, s_col, idS);
  issue_ds<D, kKPair, kKBox>(q_addr, tq_addr, k_base, s_col + BN, idS, has_tq, has_tk);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  return bf16 ? kf::Mma<__nv_bfloat16>::from_f2(a, b) : kf::Mma<__half>::from_f2(a, b);
}

// 2^x with the MUFU instruction (flushes subnormal results to zero; exp2(-inf) = 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Named barrier over the two softmax warpgroups (256 threads).
__device__ __forceinline__ void softmax_groups_sync() {
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

// ============================================================================================
// Standalone JVP. Tensor memory (JvpLayout):
//   D <= 128: [0, D) tO accumulator | S_b at 128 + 128 b, dS_b at 192 + 128 b | P_b at
//             384 + 64 b, H_b + 32; 64-key tiles, softmax warpgroup g on keys [32 g, 32 g + 32)
//             (P and H at + 16 g)
//   D = 256:  [0, 256) tO | S_b at 256 + 64 b, dS_b + 32 | P_b at 384 + 32 b, H_b + 16; 32-key
//             tiles (the 128 KB of Q and tQ leave room for 32 KB K and V stages only), warpgroup
//             g on keys [16 g, 16 g + 16) (P and H at + 8 g)
// P and H have their own columns, so tile j+2's score MMAs never wait for tile j's output MMAs.
// ============================================================================================
template <int D> struct JvpLayout {
  static constexpr int kN = D <= 128 ? 64 : 32;          // keys per tile
  static constexpr int kKeysG = kN / 2;                   // keys per softmax warpgroup
  static constexpr uint32_t kS = D <= 128 ? 128 : 256;    // S of buffer b at kS + 2 kN b, dS kN further
  static constexpr uint32_t kP = 384;                     // P of buffer b at kP + kN b, H kN / 2 further
};

template <int N>
__device__ __forceinline__ void tm_load(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 32) kf::tc::ld_32x32b_x32(taddr, r);
  else kf::tc::ld_32x32b_x16(taddr, r);
}
template <int N>
__device__ __forceinline__ void tm_store(uint32_t taddr, const uint32_t (&r)[N]) {
  if constexpr (N == 16) kf::tc::st_32x32b_x16(taddr, r);
  else kf::tc::st_32x32b_x8(taddr, r);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
fa_jvp_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_tq,
                    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_tk,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tv,
                    const FaArgs p) {
  using L = JvpLayout<D>;
  constexpr int BN = L::kN, KG = L::kKeysG;
  using C = Cfg<D, true, BN>;
  // With one V stage, "P / H of tile j written" cannot share the V stage's barrier (tile j+1's
  // softmax arrivals could land in tile j's phase): the output thread waits on p_full as well.
  constexpr bool kFoldP = C::kVStages >= 2;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  const Bars<D, true, BN> bars(smem);
  float* row_sums = reinterpret_cast<float*>(smem + C::kScratchOffset);  // [2][kBM]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kScratchOffset + C::kScratchBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qtile * kBM;
  const int kvh = h / (p.Hq / p.Hkv);
  const bool has_tq = p.tq != nullptr, has_tk = p.tk != nullptr, has_tv = p.tv != nullptr;
  const bool has_h = has_tq || has_tk;
  int k_end = p.Nk;
  if (p.causal) k_end = min(p.Nk, max(0, q0 + kBM + p.Nk - p.Nq));
  const int ntiles = (k_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    // Each MMA thread waits on one barrier per tile where it can (a probe costs ~200 cycles
    // while the tensor cores read shared memory): the k_full phase of tile j completes when
    // K / tK of tile j have landed AND every softmax thread has read tile j-2's scores out of
    // buffer j & 1; the v_full phase of tile j when V / tV of tile j have landed AND (kFoldP)
    // every softmax thread has written tile j's P and H.
    if (kFoldP) bars.init(1, 2 * kBM, 2 * kBM);  // p_full is not used
    else bars.init(2 * kBM, 2 * kBM, 0);
    *abort_flag = 0;
    kf::fence_mbar_init();
  }
  if (warp == kMmaWarp) kf::tc::tmem_alloc(bars.tmem_slot, kTmemCols);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *bars.tmem_slot;
  // Buffers 0 and 1 start free: the softmax threads' share of tiles 0 and 1's k_full phases.
  if (warp < 8) {
    kf::mbar_arrive(&bars.k_full[0]);
    kf::mbar_arrive(&bars.k_full[1]);
  }

  if (warp == kProducerWarp) {
    if (lane == 0)
      produce<D>(bars, smem, &tm_q, &tm_tq, &tm_k, &tm_tk, &tm_v, &tm_tv, has_tq, has_tk, has_h, has_tv, h, kvh,
                 q0, b, ntiles, abort_flag);
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // Scores of tile j into buffer j & 1 once K of tile j has landed and tile j-2's softmax has
      // read that buffer (one barrier).
      const uint32_t q_addr = kf::smem_u32(smem), tq_addr = q_addr + C::kQBytes;
      bool ok = kf::mbar_wait_or_abort<true>(bars.q_full, 0, &g_fa_error, abort_flag);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int buf = j & 1, st = j % C::kKStages;
        if (!(ok = kf::mbar_wait_or_abort<true>(&bars.k_full[st], (j / C::kKStages) & 1, &g_fa_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t k_base = kf::smem_u32(smem + C::kKOffset + st * C::kStageBytes);
        const uint32_t s_col = tmem + L::kS + 2 * BN * buf;
        issue_scores<D, C::kKPair, C::kKBox, BN>(q_addr, tq_addr, k_base, s_col, has_tq, has_tk, kBf16);
        kf::tc::commit(&bars.s_full[buf]);
        kf::tc::commit(&bars.k_empty[st]);
      }
    }
  } else if (warp == kPvWarp) {
    if (lane == 0) {
      // tO += P tV + H V for tile j once its V / tV have arrived and its P / H are written.
      constexpr uint32_t idPV = kf::tc::idesc_f16(kBf16 ? 1 : 0, kBM, D, false, true);
      uint32_t acc_started = 0;
      bool ok = true;
      for (int j = 0; ok && j < ntiles; ++j) {
        const int buf = j & 1, st = j % C::kVStages;
        if (!(ok = kf::mbar_wait_or_abort<true>(&bars.v_full[st], (j / C::kVStages) & 1, &g_fa_error, abort_flag)))
          break;
        if (!kFoldP && !(ok = kf::mbar_wait_or_abort<true>(&bars.p_full[buf], (j >> 1) & 1, &g_fa_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t v_base = kf::smem_u32(smem + C::kVOffset + st * C::kStageBytes);
        const uint32_t p_col = tmem + L::kP + BN * buf;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          if (has_tv) {
            kf::tc::mma_ts(tmem + kAccCol, p_col + kk * 8,
                           dsw(v_base + C::kTileBytes, kk * 2048, C::kKBox), idPV, acc_started);
            acc_started = 1;
          }
          if (has_h) {
            kf::tc::mma_ts(tmem + kAccCol, p_col + BN / 2 + kk * 8,
                           dsw(v_base, kk * 2048, C::kKBox), idPV, acc_started);
            acc_started = 1;
          }
        }
        kf::tc::commit(&bars.pv_done[buf]);
        kf::tc::commit(&bars.v_empty[st]);
      }
      kf::tc::commit(bars.acc_full);
    }
  } else {
    const int group = warp >> 2;   // softmax warpgroup: keys [KG group, KG group + KG) of every tile
    const int quarter = warp & 3;  // TMEM lanes [32 quarter, 32 quarter + 32)
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float lse_l2 = qrow < p.Nq ? p.lse_in[(static_cast<int64_t>(b) * p.Hq + h) * p.Nq + qrow] * kLog2e
                                     : __int_as_float(0x7f800000);
    const int limit = p.causal ? min(p.Nk, qrow + p.Nk - p.Nq + 1) : p.Nk;  // keys [0, limit) visible
    // Pairs of keys go through the f32x2 units: exponent argument, H and its row sum.
    const uint64_t c2 = kf::f2_pack(p.scale_log2, p.scale_log2), nl2 = kf::f2_pack(-lse_l2, -lse_l2);
    const uint64_t g2 = kf::f2_pack(p.scale, p.scale);
    uint64_t csum2 = kf::f2_pack(0.f, 0.f);
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int buf = j & 1;
      ok = kf::mbar_wait_or_abort(&bars.s_full[buf], (j >> 1) & 1, &g_fa_error, abort_flag);
      // The P / H columns of this buffer were last read by tile j-2's output MMAs.
      if (ok && j >= 2) ok = kf::mbar_wait_or_abort(&bars.pv_done[buf], ((j >> 1) - 1) & 1, &g_fa_error, abort_flag);
      // Warp-uniform outcome: the tcgen05 copies below are .sync.aligned.
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      kf::tc::fence_after_sync();
      const uint32_t s_col = lane_base + L::kS + 2 * BN * buf + KG * group;
      const uint32_t p_col = lane_base + L::kP + BN * buf + (KG / 2) * group;  // 16-bit: 2 keys per column
      const int kc = j * BN + KG * group;
      const bool full = kc + KG <= limit;  // no masking inside these keys for this row
      uint32_t sr[KG], tr[KG], pp[KG / 2], hh[KG / 2];
      tm_load<KG>(s_col, sr);
      if (has_h) tm_load<KG>(s_col + BN, tr);
      kf::tc::wait_ld();
      // This thread's share of buffer j & 1 is read: tile j+2's scores may go there (its share
      // of the k_full phase of tile j+2).
      kf::tc::fence_before_sync();
      kf::mbar_arrive(&bars.k_full[(j + 2) % C::kKStages]);
#pragma unroll
      for (int i = 0; i < KG / 2; ++i) {
        const float2 a = kf::f2_unpack(kf::f2_fma(kf::f2_pack(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])),
                                                  c2, nl2));
        float p0 = ex2(a.x), p1 = ex2(a.y);
        if (!full) {
          p0 = kc + 2 * i < limit ? p0 : 0.f;
          p1 = kc + 2 * i + 1 < limit ? p1 : 0.f;
        }
        pp[i] = pack2(p0, p1, kBf16);
        if (has_h) {
          const uint64_t hv = kf::f2_mul(
              kf::f2_mul(kf::f2_pack(p0, p1), kf::f2_pack(__uint_as_float(tr[2 * i]), __uint_as_float(tr[2 * i + 1]))), g2);
          csum2 = kf::f2_add(csum2, hv);
          const float2 hf = kf::f2_unpack(hv);
          hh[i] = pack2(hf.x, hf.y, kBf16);
        }
      }
      tm_store<KG / 2>(p_col, pp);
      if (has_h) tm_store<KG / 2>(p_col + BN / 2, hh);
      kf::tc::wait_st();
      kf::tc::fence_before_sync();
      kf::mbar_arrive(kFoldP ? &bars.v_full[j % C::kVStages] : &bars.p_full[buf]);
    }
    const float2 cs = kf::f2_unpack(csum2);
    row_sums[group * kBM + row] = cs.x + cs.y;
    softmax_groups_sync();
    const float csum = row_sums[row] + row_sums[kBM + row];
    // Epilogue: tO = acc - rowsum(H) * O; warpgroup g writes columns [g D/2, (g + 1) D/2).
    if (ok) ok = kf::mbar_wait_or_abort(bars.acc_full, 0, &g_fa_error, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      kf::tc::fence_after_sync();
      const int64_t roff = ((static_cast<int64_t>(b) * p.Nq + qrow) * p.Hq + h) * p.D;  // real head dim
      const T* orow = static_cast<const T*>(p.o_in) + roff;
      T* trow = static_cast<T*>(p.to_out) + roff;
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int c = group * (D / 64) + cc;  // 32-column chunk
        uint32_t ar[32];
        kf::tc::ld_32x32b_x32(lane_base + kAccCol + c * 32, ar);
        kf::tc::wait_ld();
        if (qrow < p.Nq) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (c * 32 + v * 8 >= p.D) break;  // padding columns (D < 128): zero, not stored
            const uint4 o = *reinterpret_cast<const uint4*>(orow + c * 32 + v * 8);
            const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
            uint32_t tw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 of = kf::Mma<T>::to_f2(ow[e]);
              const int i = v * 8 + e * 2;
              const float a0 = ntiles > 0 ? __uint_as_float(ar[i]) : 0.f;
              const float a1 = ntiles > 0 ? __uint_as_float(ar[i + 1]) : 0.f;
              tw[e] = pack2(a0 - csum * of.x, a1 - csum * of.y, kBf16);
            }
            *reinterpret_cast<uint4*>(trow + c * 32 + v * 8) = make_uint4(tw[0], tw[1], tw[2], tw[3]);
          }
        }
      }
    }
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================================================
// One-pass forward (+ JVP): O, LSE (and tO) with online statistics
// (flash-attention-jvp-derivation.md sections 7-8):
//   E = exp2(x - m), x = gamma log2(e) S;  l += rowsum(E);  U += E V
//   H = E * gamma (tQ K^T + Q tK^T);       r += rowsum(H);  G += H V + E tV
//   O = U / l;  tO = G / l - (r / l) O;  LSE = (m + log2 l) ln 2
// Both softmax warpgroups work on every 64-key tile, each on 32 of its keys; they exchange the
// tile row maxima through shared memory. The reference max m only moves when a tile's max
// exceeds it by more than 8 (a factor 256 in E); then the accumulators U, G of that row are
// rescaled in TMEM after the previous tile's output MMAs have completed. Tensor memory:
//   D = 128 + JVP: [0, 128) G (tO accumulator) | [128, 384) two S / dS buffers | [384, 512) U
//   D = 128 forward: [0, 128) U | [128, 512) three S buffers
//   D = 64:  [0, 64) U | [64, 128) G | [128, 512) three S / dS buffers
//   D = 256 (forward only, head dims 136..256): [0, 256) U | [256, 512) two S buffers
// P and H (16-bit) overwrite the first 16 columns of each warpgroup's 32-column S / dS half, so
// tile j's score MMAs wait for tile j-NB's output MMAs (same buffer). With two buffers that
// chain (scores, softmax, output MMAs, buffer free) set the period of the forward at D = 64;
// three let the scores of tile j+2 run while tiles j and j+1 are in the softmax and output
// stages.
// The scores are issued as in the standalone kernel ([S | Q tK^T] = Q [K ; tK]^T, then
// dS += tQ K^T). For D = 64 the output MMAs are merged the same way, since an N = 64 MMA runs at
// 2/3 of the tensor core's rate: [U | G] += E [V | tV] (V, tV adjacent: two 64-wide MN blocks)
// then G += H V. That takes U at [0, 64) and G at [64, 128), next to each other.
// ============================================================================================
template <int D, bool kJvp>
struct FusedCols {
  static constexpr bool kMerge = D == 64;
  static constexpr uint32_t kU = D == 128 && kJvp ? 384 : 0;  // U: E V
  static constexpr uint32_t kG = kMerge ? 64 : 0;             // G: H V + E tV (the tO accumulator)
  // Score buffers at kBufCol + 128 b: three where the accumulators leave 384 columns (the
  // forward at D = 64 and 128, forward + JVP at D = 64), else two.
  static constexpr int kBufs = (D == 64 || (D == 128 && !kJvp)) ? 3 : 2;
};
constexpr float kRescaleThreshold = 8.f;  // log2 units

template <typename T, int D, bool kJvp>
__global__ void __launch_bounds__(kThreads, 1)
fa_fused_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_tq,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_tk,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tv,
                      const FaArgs p) {
  using C = Cfg<D, kJvp>;
  constexpr int NB = FusedCols<D, kJvp>::kBufs;  // score buffers
  static_assert(NB <= C::kKStages, "a buffer's free arrival for tile j + NB lands in that tile's K stage");
  static_assert(NB <= C::kVStages, "the softmax threads reach tile j + NB only after tile j's output MMAs: "
                "the V phase they arrive on must be the one of their own tile");
  static_assert(D <= 128 || !kJvp, "D = 256 tensor memory holds the forward's accumulator only");
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  const Bars<D, kJvp> bars(smem);
  float* tile_max = reinterpret_cast<float*>(smem + C::kScratchOffset);  // [NB buffers][2 groups][kBM]
  float* part_sums = tile_max + 2 * NB * kBM;                              // [2 groups][kBM]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(part_sums + 2 * kBM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qtile * kBM;
  const int kvh = h / (p.Hq / p.Hkv);
  const bool has_tq = kJvp && p.tq != nullptr, has_tk = kJvp && p.tk != nullptr;
  const bool has_tv = kJvp && p.tv != nullptr;
  const bool has_h = has_tq || has_tk;
  int k_end = p.Nk;
  if (p.causal) k_end = min(p.Nk, max(0, q0 + kBM + p.Nk - p.Nq));
  const int ntiles = (k_end + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    // The k_full phase of tile j completes when K / tK of tile j have landed AND tile j-NB's
    // output MMAs (which read the P / H written over score buffer j % NB) are done: the output
    // thread commits to it. The v_full phase of tile j completes when V / tV of tile j have landed AND
    // every softmax thread has written tile j's P and H. p_full is not used here.
    bars.init(1, 1, 2 * kBM);
    *abort_flag = 0;
    kf::fence_mbar_init();
  }
  if (warp == kMmaWarp) kf::tc::tmem_alloc(bars.tmem_slot, kTmemCols);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *bars.tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0)
      produce<D>(bars, smem, &tm_q, &tm_tq, &tm_k, &tm_tk, &tm_v, &tm_tv, has_tq, has_tk, true, has_tv, h, kvh,
                 q0, b, ntiles, abort_flag);
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // Scores of tile j into buffer j % NB once K of tile j has landed and tile j-NB's output MMAs
      // have consumed the P / H that overwrote that buffer (one barrier).
      const uint32_t q_addr = kf::smem_u32(smem), tq_addr = q_addr + C::kQBytes;
      bool ok = kf::mbar_wait_or_abort<true>(bars.q_full, 0, &g_fa_error, abort_flag);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int buf = j % NB, st = j % C::kKStages;
        if (!(ok = kf::mbar_wait_or_abort<true>(&bars.k_full[st], (j / C::kKStages) & 1, &g_fa_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t k_base = kf::smem_u32(smem + C::kKOffset + st * C::kStageBytes);
        const uint32_t s_col = tmem + C::kBufCol + 128 * buf;
        issue_scores<D, C::kKPair, C::kKBox, kBN>(q_addr, tq_addr, k_base, s_col, has_tq, has_tk, kBf16);
        kf::tc::commit(&bars.s_full[buf]);
        kf::tc::commit(&bars.k_empty[st]);
      }
    }
  } else if (warp == kPvWarp) {
    if (lane == 0) {
      constexpr uint32_t idPV = kf::tc::idesc_f16(kBf16 ? 1 : 0, kBM, D, false, true);
      constexpr uint32_t idPV2 = kf::tc::idesc_f16(kBf16 ? 1 : 0, kBM, 2 * D, false, true);
      constexpr uint32_t kU = FusedCols<D, kJvp>::kU, kG = FusedCols<D, kJvp>::kG;
      uint32_t u_started = 0, g_started = 0;
      bool ok = true;
      // Score buffers start free: this thread's share of tiles 0 .. NB-1's k_full phases.
      for (int t = 0; t < NB; ++t) kf::mbar_arrive(&bars.k_full[t]);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int buf = j % NB, st = j % C::kVStages;
        if (!(ok = kf::mbar_wait_or_abort<true>(&bars.v_full[st], (j / C::kVStages) & 1, &g_fa_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t v_base = kf::smem_u32(smem + C::kVOffset + st * C::kStageBytes);
        const uint32_t p_col = tmem + C::kBufCol + 128 * buf;
        const uint32_t h_col = p_col + 64;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // keys [16 kk, 16 kk + 16): warpgroup kk / 2 wrote them at columns 32 (kk / 2) + 8 (kk % 2)
          const uint32_t acol = (kk >> 1) * 32 + (kk & 1) * 8;
          const uint64_t vdesc = dsw(v_base, kk * 2048, kBN * 128);
          if (FusedCols<D, kJvp>::kMerge && has_tv) {
            // [U | G] += E [V | tV]: V and tV are the two 64-wide MN blocks of one operand
            kf::tc::mma_ts(tmem + kU, p_col + acol, dsw(v_base, kk * 2048, C::kTileBytes),
                           idPV2, u_started);
            u_started = g_started = 1;
            if (has_h) kf::tc::mma_ts(tmem + kG, h_col + acol, vdesc, idPV, 1);
            continue;
          }
          kf::tc::mma_ts(tmem + kU, p_col + acol, vdesc, idPV, u_started);
          u_started = 1;
          if (has_h) {
            kf::tc::mma_ts(tmem + kG, h_col + acol, vdesc, idPV, g_started);
            g_started = 1;
          }
          if (has_tv) {
            kf::tc::mma_ts(tmem + kG, p_col + acol,
                           dsw(v_base + C::kTileBytes, kk * 2048, kBN * 128), idPV, g_started);
            g_started = 1;
          }
        }
        kf::tc::commit(&bars.pv_done[buf]);
        kf::tc::commit(&bars.v_empty[st]);
        kf::tc::commit(&bars.k_full[(j + NB) % C::kKStages]);  // score buffer j % NB is free for tile j+NB
      }
      kf::tc::commit(bars.acc_full);
    }
  } else {
    const int group = warp >> 2;   // which 32 keys of each tile this warpgroup handles
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int limit = qrow >= p.Nq ? 0 : (p.causal ? min(p.Nk, qrow + p.Nk - p.Nq + 1) : p.Nk);
    float m_ref = -INFINITY;
    // Row sums of E and H as f32x2 pairs; pairs of keys share the f32x2 instructions.
    uint64_t l2 = kf::f2_pack(0.f, 0.f), r2 = l2;
    const uint64_t c2 = kf::f2_pack(p.scale_log2, p.scale_log2), g2 = kf::f2_pack(p.scale, p.scale);
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int buf = j % NB;
      if (ok) ok = kf::mbar_wait_or_abort(&bars.s_full[buf], (j / NB) & 1, &g_fa_error, abort_flag);
      ok = __all_sync(0xffffffffu, ok);  // the tcgen05 copies below are .sync.aligned
      kf::tc::fence_after_sync();
      const uint32_t s_col = lane_base + C::kBufCol + 128 * buf + group * 32;
      const uint32_t ts_col = s_col + 64;
      uint32_t sr[32], tr[32];
      float mx = -INFINITY;
      const int kc = j * kBN + group * 32;
      if (ok) {
        kf::tc::ld_32x32b_x32(s_col, sr);
        if (has_h) kf::tc::ld_32x32b_x32(ts_col, tr);
        kf::tc::wait_ld();
        // Row max of the raw scores (masked keys -inf), then scaled: the scale is positive.
        if (kc + 32 <= limit) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = kc + i < limit ? __uint_as_float(sr[i]) : -INFINITY;
            sr[i] = __float_as_uint(x);
            mx = fmaxf(mx, x);
          }
        }
        mx *= p.scale_log2;
      }
      // Exchange the two halves' maxima (every softmax thread reaches this barrier).
      tile_max[(buf * 2 + group) * kBM + row] = mx;
      softmax_groups_sync();
      mx = fmaxf(tile_max[(buf * 2) * kBM + row], tile_max[(buf * 2 + 1) * kBM + row]);
      if (ok) {
        // A warp moves to new reference maxima when any of its rows grew past the threshold
        // (warp-uniform, as the tensor-memory copies are .sync.aligned); the other rows move to
        // their own max as well, with alpha = 1 where it did not change.
        if (__any_sync(0xffffffffu, mx > m_ref + kRescaleThreshold)) {
          const float m_new = fmaxf(m_ref, mx);
          if (j > 0) {
            // Rescale the accumulators once the previous tile's output MMAs are done (rows
            // with no key seen yet hold zeros: alpha = 1).
            const float alpha = m_ref == -INFINITY ? 1.f : ex2(m_ref - m_new);
            ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&bars.pv_done[(j - 1) % NB], ((j - 1) / NB) & 1,
                                                                &g_fa_error, abort_flag));
            kf::tc::fence_after_sync();
            if (ok) {
#pragma unroll
              for (int c = 0; c < D / 64; ++c) {
                const uint32_t col = (group * (D / 2)) + c * 32;
                uint32_t ar[32];
                kf::tc::ld_32x32b_x32(lane_base + FusedCols<D, kJvp>::kU + col, ar);
                kf::tc::wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) ar[i] = __float_as_uint(__uint_as_float(ar[i]) * alpha);
                kf::tc::st_32x32b_x32(lane_base + FusedCols<D, kJvp>::kU + col, ar);
                if (kJvp) {
                  kf::tc::ld_32x32b_x32(lane_base + FusedCols<D, kJvp>::kG + col, ar);
                  kf::tc::wait_ld();
#pragma unroll
                  for (int i = 0; i < 32; ++i) ar[i] = __float_as_uint(__uint_as_float(ar[i]) * alpha);
                  kf::tc::st_32x32b_x32(lane_base + FusedCols<D, kJvp>::kG + col, ar);
                }
              }
            }
            const uint64_t alpha2 = kf::f2_pack(alpha, alpha);
            l2 = kf::f2_mul(l2, alpha2);
            r2 = kf::f2_mul(r2, alpha2);
          }
          m_ref = m_new;
        }
        const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
        const uint64_t nm2 = kf::f2_pack(-m_use, -m_use);
        uint32_t pp[16], hh[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          // E = 2^(S gamma log2(e) - m): one f32x2 FMA per key pair, masked keys give 2^-inf = 0
          const float2 a = kf::f2_unpack(
              kf::f2_fma(kf::f2_pack(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), c2, nm2));
          const float e0 = ex2(a.x), e1 = ex2(a.y);
          const uint64_t e2 = kf::f2_pack(e0, e1);
          l2 = kf::f2_add(l2, e2);
          pp[i] = pack2(e0, e1, kBf16);
          if (has_h) {
            const uint64_t hv =
                kf::f2_mul(kf::f2_mul(e2, kf::f2_pack(__uint_as_float(tr[2 * i]), __uint_as_float(tr[2 * i + 1]))), g2);
            r2 = kf::f2_add(r2, hv);
            const float2 hf = kf::f2_unpack(hv);
            hh[i] = pack2(hf.x, hf.y, kBf16);
          }
        }
        kf::tc::st_32x32b_x16(s_col, pp);
        if (has_h) kf::tc::st_32x32b_x16(ts_col, hh);
        kf::tc::wait_st();
      }
      kf::tc::fence_before_sync();
      kf::mbar_arrive(&bars.v_full[j % C::kVStages]);
    }
    // Combine the two warpgroups' row sums.
    const float2 lf = kf::f2_unpack(l2), rf = kf::f2_unpack(r2);
    const float l_part = lf.x + lf.y, r_part = rf.x + rf.y;
    part_sums[group * kBM + row] = l_part;
    softmax_groups_sync();
    const float l_tot = part_sums[row] + part_sums[kBM + row];
    softmax_groups_sync();
    part_sums[group * kBM + row] = r_part;
    softmax_groups_sync();
    const float r_tot = part_sums[row] + part_sums[kBM + row];
    if (ok) ok = kf::mbar_wait_or_abort(bars.acc_full, 0, &g_fa_error, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      kf::tc::fence_after_sync();
      const float inv_l = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const float rl = r_tot * inv_l;
      const int64_t roff = ((static_cast<int64_t>(b) * p.Nq + qrow) * p.Hq + h) * p.D;  // real head dim
      T* orow = static_cast<T*>(p.o_out) + roff;
      T* trow = kJvp ? static_cast<T*>(p.to_out) + roff : nullptr;
      if (group == 0 && qrow < p.Nq) {
        const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
        p.lse_out[(static_cast<int64_t>(b) * p.Hq + h) * p.Nq + qrow] =
            l_tot > 0.f ? (m_use + log2f(l_tot)) * 0.6931471805599453f : __int_as_float(0x7f800000);
      }
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        const int col = group * (D / 2) + c * 32;
        uint32_t ur[32], gr[32];
        kf::tc::ld_32x32b_x32(lane_base + FusedCols<D, kJvp>::kU + col, ur);
        if (kJvp) kf::tc::ld_32x32b_x32(lane_base + FusedCols<D, kJvp>::kG + col, gr);
        kf::tc::wait_ld();
        if (qrow < p.Nq) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (col + v * 8 >= p.D) break;  // padding columns (D < 128): zero, not stored
            uint32_t ow[4], tw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = v * 8 + e * 2;
              const float o0 = ntiles > 0 ? __uint_as_float(ur[i]) * inv_l : 0.f;
              const float o1 = ntiles > 0 ? __uint_as_float(ur[i + 1]) * inv_l : 0.f;
              ow[e] = pack2(o0, o1, kBf16);
              if (kJvp) {
                const float g0 = ntiles > 0 ? __uint_as_float(gr[i]) * inv_l : 0.f;
                const float g1 = ntiles > 0 ? __uint_as_float(gr[i + 1]) * inv_l : 0.f;
                tw[e] = pack2(g0 - rl * o0, g1 - rl * o1, kBf16);
              }
            }
            *reinterpret_cast<uint4*>(orow + col + v * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
            if (kJvp) *reinterpret_cast<uint4*>(trow + col + v * 8) = make_uint4(tw[0], tw[1], tw[2], tw[3]);
          }
        }
      }
    }
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D>
int launch_jvp(const FaArgs& a, int dtype, cudaStream_t stream) {
  constexpr int BN = JvpLayout<D>::kN;
  using C = Cfg<D, true, BN>;
  CUtensorMap mq, mtq, mk, mtk, mv, mtv;
  // The maps carry the real head dim: boxes past it (D < 128 or < 256) read as zeros.
  if (!encode_bnhd(&mq, a.q, dtype, a.B, a.Nq, a.Hq, a.D, kBM) ||
      !encode_bnhd(&mtq, a.tq ? a.tq : a.q, dtype, a.B, a.Nq, a.Hq, a.D, kBM) ||
      !encode_bnhd(&mk, a.k, dtype, a.B, a.Nk, a.Hkv, a.D, BN) ||
      !encode_bnhd(&mtk, a.tk ? a.tk : a.k, dtype, a.B, a.Nk, a.Hkv, a.D, BN) ||
      !encode_bnhd(&mv, a.v, dtype, a.B, a.Nk, a.Hkv, a.D, BN) ||
      !encode_bnhd(&mtv, a.tv ? a.tv : a.v, dtype, a.B, a.Nk, a.Hkv, a.D, BN))
    return KF_ERR_CUDA;
  auto kernel = fa_jvp_sm100_kernel<T, D>;
  const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kThreads, C::kSmemBytes, nullptr);
  if (prep != KF_OK) return prep;
  const dim3 grid((a.Nq + kBM - 1) / kBM, a.Hq, a.B);
  kernel<<<grid, kThreads, C::kSmemBytes, stream>>>(mq, mtq, mk, mtk, mv, mtv, a);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

template <typename T, int D, bool kJvp>
int launch_fused(const FaArgs& a, int dtype, cudaStream_t stream) {
  using C = Cfg<D, kJvp>;
  CUtensorMap mq, mtq, mk, mtk, mv, mtv;
  // The maps carry the real head dim: boxes past it (D < 128) read as zeros.
  if (!encode_bnhd(&mq, a.q, dtype, a.B, a.Nq, a.Hq, a.D, kBM) ||
      !encode_bnhd(&mtq, a.tq ? a.tq : a.q, dtype, a.B, a.Nq, a.Hq, a.D, kBM) ||
      !encode_bnhd(&mk, a.k, dtype, a.B, a.Nk, a.Hkv, a.D, kBN) ||
      !encode_bnhd(&mtk, a.tk ? a.tk : a.k, dtype, a.B, a.Nk, a.Hkv, a.D, kBN) ||
      !encode_bnhd(&mv, a.v, dtype, a.B, a.Nk, a.Hkv, a.D, kBN) ||
      !encode_bnhd(&mtv, a.tv ? a.tv : a.v, dtype, a.B, a.Nk, a.Hkv, a.D, kBN))
    return KF_ERR_CUDA;
  auto kernel = fa_fused_sm100_kernel<T, D, kJvp>;
  const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kThreads, C::kSmemBytes, nullptr);
  if (prep != KF_OK) return prep;
  const dim3 grid((a.Nq + kBM - 1) / kBM, a.Hq, a.B);
  kernel<<<grid, kThreads, C::kSmemBytes, stream>>>(mq, mtq, mk, mtk, mv, mtv, a);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

}  // namespace

int kf_internal_fa_error(unsigned int* code) {
  unsigned int v = 0;
  KF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fa_error, sizeof(v)));
  if (v != 0) {
    const unsigned int zero = 0;
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_fa_error, &zero, sizeof(zero)));
  }
  *code = v;
  return KF_OK;
}

namespace kf::fa {

// Head dims (multiples of 8): 8..56 run the D = 64 kernels, 72..120 the D = 128 kernels and
// 136..248 the D = 256 kernels on zero-padded tiles (TMA fills the columns past D with zeros;
// the epilogues store only real columns). The one-pass forward + JVP kernel stops at 128.
bool sm100_head_dim(int d) { return d >= 8 && d <= 128; }

bool sm100_jvp_supported(const FaArgs& a) {
  return a.D >= 8 && a.D <= 256 && (a.tq != nullptr || a.tk != nullptr || a.tv != nullptr);
}

bool sm100_fused_supported(const FaArgs& a, int mode) {
  if (mode == kModeFwd) return a.D >= 8 && a.D <= 256;
  if (!sm100_head_dim(a.D)) return false;
  return a.tq != nullptr || a.tk != nullptr || a.tv != nullptr;
}

int launch_sm100_fused(const FaArgs& a, int mode, int dtype, cudaStream_t s) {
  const bool jvp = mode == kModeFwdJvp;
  if (a.D > 128) {
    if (jvp) return KF_ERR_UNSUPPORTED;
    return dtype == KF_DTYPE_BF16 ? launch_fused<__nv_bfloat16, 256, false>(a, dtype, s)
                                  : launch_fused<__half, 256, false>(a, dtype, s);
  }
  if (dtype == KF_DTYPE_BF16) {
    if (a.D <= 64) return jvp ? launch_fused<__nv_bfloat16, 64, true>(a, dtype, s) : launch_fused<__nv_bfloat16, 64, false>(a, dtype, s);
    return jvp ? launch_fused<__nv_bfloat16, 128, true>(a, dtype, s) : launch_fused<__nv_bfloat16, 128, false>(a, dtype, s);
  }
  if (a.D <= 64) return jvp ? launch_fused<__half, 64, true>(a, dtype, s) : launch_fused<__half, 64, false>(a, dtype, s);
  return jvp ? launch_fused<__half, 128, true>(a, dtype, s) : launch_fused<__half, 128, false>(a, dtype, s);
}

int launch_sm100_jvp(const FaArgs& a, int dtype, cudaStream_t s) {
  if (dtype == KF_DTYPE_BF16) {
    if (a.D > 128) return launch_jvp<__nv_bfloat16, 256>(a, dtype, s);
    return a.D <= 64 ? launch_jvp<__nv_bfloat16, 64>(a, dtype, s) : launch_jvp<__nv_bfloat16, 128>(a, dtype, s);
  }
  if (a.D > 128) return launch_jvp<__half, 256>(a, dtype, s);
  return a.D <= 64 ? launch_jvp<__half, 64>(a, dtype, s) : launch_jvp<__half, 128>(a, dtype, s);
}

}  // namespace kf::fa
