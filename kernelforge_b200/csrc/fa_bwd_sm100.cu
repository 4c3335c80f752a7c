// FlashAttention backward (reverse-mode VJP) on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head dims up to 256 (other than 64, 128 and 256 on zero-padded
// tiles), fp16 / bf16, causal (bottom-right), GQA.
//
// Replaces the flash_attn binary's _flash_attn_backward that FlashAttentionFunction.backward
// calls (flash_attention_jvp/custom.py:255-266). After the row-statistics pass of fa_bwd.cu
// (row_nlse = -LSE log2 e, row_ndelta = -rowsum(dO O), padded), either one kernel that computes
// dQ, dK and dV with dQ summed at L2 (fa_bwd_fused_sm100_kernel, head dims up to 128; the
// default, as flash_attn's deterministic=False) or two kernels with no atomics (deterministic):
//
//   dq kernel    query-stationary: 128 query rows of one (batch, head) per CTA, 64-key tiles
//                (32-key tiles at D = 256)
//                  S  = Q K^T,  dP = dO V^T           score MMAs into three TMEM buffers
//                  P  = 2^(S gamma log2 e - LSE log2 e),  dS = P (dP - delta)
//                  dQ += dS K                          A = dS (16-bit, TMEM), B = K (MN-major)
//   dkdv kernel  key-stationary: 128 keys of one (batch, KV head) per CTA; the 64-query tiles of
//                every query head of the group, in order (the group sum is sequential)
//                  S^T = K Q^T,  dP^T = V dO^T
//                  P^T, dS^T (16-bit) written over the first 32 columns of their fp32 tiles
//                  dV += P^T dO,  dK += dS^T Q         B = dO, Q (MN-major)
// Output scaling: dQ and dK by gamma at the end.
//
// Warp roles (352 threads), as in the forward-mode kernels of fa_sm100.cu:
//   warps 0..3, 4..7  two softmax warpgroups; both work on every tile, warpgroup g on streamed
//                     columns [32 g, 32 g + 32), one thread per stationary row (= one TMEM lane)
//   warp 8            TMA producer: the stationary pair once, then a ring of streamed pairs
//   warp 9            TMEM owner; one thread issues the score MMAs
//   warp 10           one thread issues the accumulating MMAs
// Every wait is a bounded mbarrier wait that records KF_ERR_DEVICE_TIMEOUT and gives up.
#include <climits>

#include "fa_common.cuh"
#include "kf_tcgen05.cuh"

namespace {

using kf::fa::BwdArgs;
using kf::fa::encode_bnhd;

__device__ unsigned int g_fa_bwd_error = 0;
// The first bounded wait that gave up: role << 24 | tile (roles: 1 producer, 2 score MMAs,
// 3 accumulating MMAs, 4 softmax, 5 epilogue, 6 dQ warps).
__device__ unsigned int g_fa_bwd_where = 0;
__device__ __forceinline__ void note_gave_up(unsigned int role, int t) {
  atomicCAS(&g_fa_bwd_where, 0u, (role << 24) | (static_cast<unsigned int>(t) & 0xFFFFFFu));
}

constexpr int kRows = 128;     // stationary rows per CTA
constexpr int kThreads = 352;  // 11 warps
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kOutWarp = 10;
constexpr uint32_t kTmemCols = 512;

// Shared memory: the stationary pair (Q, dO or K, V), a ring of streamed pairs (K, V or Q, dO)
// with, per stage, the tile's row statistics of each kind (dkdv only), then the barriers.
// D = 256: the stationary pair takes 128 KB, so the streamed tiles are 32 rows (3 stages of
// 2 x 16 KB), and the dK / dV accumulators (2 x 256 columns together) are split by head-dim
// halves over two CTAs per key block, each recomputing the key block's scores.
// kFused (D <= 128): after the barriers, one 16-bit dS^T tile per score buffer (the dQ MMAs'
// B operand), then the dQ warps' staging boxes.
template <int D, bool kFused = false> struct Cfg {
  static constexpr int kTile = D <= 128 ? 64 : 32;       // streamed rows per tile
  static constexpr int kKB = D / 64;                     // 128-byte boxes along the head dim
  static constexpr int kStatBytes = kKB * kRows * 128;   // one stationary operand
  static constexpr int kTileBytes = kKB * kTile * 128;   // one streamed operand tile
  static constexpr int kStages = D == 64 ? 4 : 3;
  static constexpr int kBufCols = 2 * kTile;             // S and dP (or S^T and dP^T) of a buffer
  // Score buffers may not outnumber ring stages: a buffer's "free" arrival for tile t + bufs
  // must land in that tile's phase of its stage.
  static constexpr uint32_t kDqBuf = D <= 128 ? 128 : 256;  // dQ accumulator below it
  static constexpr int kDqBufs = (512 - kDqBuf) / kBufCols < kStages ? (512 - kDqBuf) / kBufCols : kStages;
  static constexpr int kAccN = D == 256 ? 128 : D;       // dV / dK columns per CTA
  static constexpr int kHalves = D / kAccN;              // CTAs per key block
  static constexpr uint32_t kDkdvBuf = 2 * kAccN;        // dV at 0, dK at kAccN
  static constexpr int kDkdvBufs =
      (512 - kDkdvBuf) / kBufCols < kStages ? (512 - static_cast<int>(kDkdvBuf)) / kBufCols : kStages;
  static constexpr int kRingOffset = 2 * kStatBytes;
  static constexpr int kRowStatOffset = kRingOffset + kStages * 2 * kTileBytes;
  static constexpr int kBarOffset = kRowStatOffset + kStages * 2 * kTile * 4;
  static constexpr int kDsBytes = kRows * kTile * 2;
  static constexpr int kDsOffset = (kBarOffset + 256 + 1023) / 1024 * 1024;
  // kFused: after the dS^T tiles, one 64-query x 32-column fp32 dQ box per head-dim quarter, the
  // staging of its dQ warp's TMA reduction.
  static constexpr int kDqBoxBytes = 64 * 32 * 4;
  static constexpr int kDqStageOffset = kDsOffset + kDkdvBufs * kDsBytes;
  static constexpr int kSmemBytes =
      (kFused ? kDqStageOffset + (D / 32) * kDqBoxBytes : kBarOffset + 256) + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 232448, "shared memory");
};
constexpr int kMaxBufs = 3;

template <int D> struct Bars {
  uint64_t* stat_full;
  uint64_t* ring_full;   // [kStages] the tile's operands landed AND its score buffer is free
  uint64_t* ring_empty;  // [kStages] the accumulating MMAs of the stage's tile completed
  uint64_t* s_full;      // [kMaxBufs] score MMAs of tile t complete
  uint64_t* p_full;      // [kMaxBufs] softmax of tile t done (scores read, 16-bit operands written)
  uint64_t* acc_full;
  uint64_t* dq_full;     // [kMaxBufs] fused kernel: the dQ^T MMAs of tile t complete
  uint64_t* drain;       // both MMA-issuing threads' MMAs complete (before TMEM is freed)
  uint32_t* tmem_slot;
  int* abort_flag;
  __device__ explicit Bars(uint8_t* smem) {
    using C = Cfg<D>;
    stat_full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    ring_full = stat_full + 1;
    ring_empty = ring_full + C::kStages;
    s_full = ring_empty + C::kStages;
    p_full = s_full + kMaxBufs;
    acc_full = p_full + kMaxBufs;
    dq_full = acc_full + 1;
    drain = dq_full + kMaxBufs;
    tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  }
  // buffer_arrivals: how many arrivals free a score buffer (the accumulating thread's commit,
  // or the fused kernel's four dQ warps), besides the producer's, so the score thread waits on
  // one barrier per tile.
  __device__ void init(uint32_t buffer_arrivals) const {
    using C = Cfg<D>;
    kf::mbar_init(stat_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      kf::mbar_init(&ring_full[s], 1 + buffer_arrivals);
      kf::mbar_init(&ring_empty[s], 1);
    }
    for (int i = 0; i < kMaxBufs; ++i) {
      kf::mbar_init(&s_full[i], 1);
      kf::mbar_init(&p_full[i], 2 * kRows);  // both softmax warpgroups
      kf::mbar_init(&dq_full[i], 1);
    }
    kf::mbar_init(acc_full, 1);
    kf::mbar_init(drain, 2);
    *abort_flag = 0;
  }
};

// Streamed tile t of a CTA: head h_base + t / count, rows (first + t % count) * tile.
struct TileWalk {
  int h_base, first, count, tile;
  __device__ int head(int t) const { return h_base + t / count; }
  __device__ int row0(int t) const { return (first + t % count) * tile; }
};

// TMA producer (one thread). kRowStats: each stage also carries the tile's 64 row statistics.
template <int D, bool kRowStats>
__device__ void produce(const Bars<D>& bars, uint8_t* smem, const CUtensorMap* tm_s0, const CUtensorMap* tm_s1,
                        const CUtensorMap* tm_t0, const CUtensorMap* tm_t1, int stat_head, int stat_row0, int b,
                        const TileWalk& walk, int ntiles, const BwdArgs& p) {
  using C = Cfg<D>;
  volatile int* abort = bars.abort_flag;
  kf::prefetch_tensormap(tm_s0);
  kf::prefetch_tensormap(tm_t0);
  kf::mbar_arrive_expect_tx(bars.stat_full, 2 * C::kStatBytes);
  for (int kb = 0; kb < C::kKB; ++kb) {
    kf::tma_load_4d(smem + kb * kRows * 128, tm_s0, bars.stat_full, kb * 64, stat_head, stat_row0, b);
    kf::tma_load_4d(smem + C::kStatBytes + kb * kRows * 128, tm_s1, bars.stat_full, kb * 64, stat_head, stat_row0, b);
  }
  constexpr uint32_t kStageTx = 2 * C::kTileBytes + (kRowStats ? 2 * C::kTile * 4 : 0);
  for (int t = 0; t < ntiles; ++t) {
    const int st = t % C::kStages;
    if (t >= C::kStages &&
        !kf::mbar_wait_or_abort<true>(&bars.ring_empty[st], ((t / C::kStages) - 1) & 1, &g_fa_bwd_error, abort)) {
      note_gave_up(1, t);
      return;
    }
    uint8_t* base = smem + C::kRingOffset + st * 2 * C::kTileBytes;
    const int h = walk.head(t), r0 = walk.row0(t);
    kf::mbar_arrive_expect_tx(&bars.ring_full[st], kStageTx);
    for (int kb = 0; kb < C::kKB; ++kb) {
      kf::tma_load_4d(base + kb * C::kTile * 128, tm_t0, &bars.ring_full[st], kb * 64, h, r0, b);
      kf::tma_load_4d(base + C::kTileBytes + kb * C::kTile * 128, tm_t1, &bars.ring_full[st], kb * 64, h, r0, b);
    }
    if (kRowStats) {
      // r0 + kTile <= NqP and NqP is a multiple of 128: 16-byte aligned, in bounds.
      const int64_t off = (static_cast<int64_t>(b) * p.Hq + h) * p.NqP + r0;
      float* rs = reinterpret_cast<float*>(smem + C::kRowStatOffset + st * 2 * C::kTile * 4);
      kf::bulk_load(rs, p.row_nlse + off, C::kTile * 4, &bars.ring_full[st]);
      kf::bulk_load(rs + C::kTile, p.row_ndelta + off, C::kTile * 4, &bars.ring_full[st]);
    }
  }
}

// D[128 x TILE] = A[128 x D] B[TILE x D]^T; A, B K-major 128-byte-swizzled tiles.
// The descriptors are built once; each K step only adds a constant offset, which keeps the
// issuing thread's instruction count per MMA small.
template <int D, int TILE>
__device__ __forceinline__ void issue_scores(uint32_t a_addr, uint32_t b_addr, uint32_t d_col, uint32_t idesc) {
  const uint64_t a_desc = kf::tc::desc_sw128(a_addr, 16, 1024), b_desc = kf::tc::desc_sw128(b_addr, 16, 1024);
#pragma unroll
  for (int k = 0; k < D / 16; ++k) {
    const uint32_t aoff = (k >> 2) * kRows * 128 + (k & 3) * 32;
    const uint32_t boff = (k >> 2) * TILE * 128 + (k & 3) * 32;
    kf::tc::mma_ss(d_col, kf::tc::desc_advance(a_desc, aoff), kf::tc::desc_advance(b_desc, boff), idesc, k > 0);
  }
}

// D[128 x N] += A[128 x TILE] B[TILE x N]; A 16-bit in TMEM (8 columns per 16 of K), B an
// MN-major 128-byte-swizzled tile (64-element blocks TILE * 128 bytes apart). kSplitA: K rows
// [G g, G g + G) of A (G = TILE / 2) start at column G g (each softmax warpgroup packed its G
// values into the first G / 2 of its own G columns); otherwise A is packed contiguously.
template <int TILE, bool kSplitA>
__device__ __forceinline__ void issue_accumulate(uint32_t d_col, uint32_t a_col, uint32_t b_addr, uint32_t idesc,
                                                 uint32_t& started) {
  constexpr int kG = TILE / 2, kSteps = kG / 16;  // K16 steps per warpgroup's keys
  const uint64_t b_desc = kf::tc::desc_sw128(b_addr, TILE * 128, 1024);
#pragma unroll
  for (int kk = 0; kk < TILE / 16; ++kk) {
    const uint32_t acol = kSplitA ? (kk / kSteps) * kG + (kk % kSteps) * 8 : kk * 8;
    kf::tc::mma_ts(d_col, a_col + acol, kf::tc::desc_advance(b_desc, kk * 2048), idesc, started);
    started = 1;
  }
}

// Tensor-memory copies of one softmax warpgroup's G scores (G = 32 or 16) and G / 2 packed
// 16-bit results per row.
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

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  return bf16 ? kf::Mma<__nv_bfloat16>::from_f2(a, b) : kf::Mma<__half>::from_f2(a, b);
}

// 2^x with the MUFU instruction (flushes subnormal results to zero; exp2(-inf) = 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, const int* abort) {
  return kf::mbar_wait_or_abort(bar, parity, &g_fa_bwd_error, const_cast<volatile int*>(abort));
}
// Bounded wait that does not give up early on the CTA's abort flag (draining in-flight MMAs).
__device__ __forceinline__ bool wait_drain_again(uint64_t* bar) {
  return kf::mbar_wait_bounded(bar, 0, &g_fa_bwd_error);
}
__device__ __forceinline__ bool wait_relaxed(uint64_t* bar, uint32_t parity, const int* abort) {
  return kf::mbar_wait_or_abort<true>(bar, parity, &g_fa_bwd_error, const_cast<volatile int*>(abort));
}

// Epilogue store of 32 accumulator columns of one row: out = acc * mul (zeros when nothing was
// accumulated); only the first `valid` columns exist (head dims below the kernel's padded one).
template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const uint32_t (&acc)[32], float mul, bool any, int valid) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    if (v * 8 >= valid) break;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = v * 8 + e * 2;
      w[e] = any ? pack2(__uint_as_float(acc[i]) * mul, __uint_as_float(acc[i + 1]) * mul, kBf16) : 0u;
    }
    *reinterpret_cast<uint4*>(dst + v * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ============================================================================================
// dQ. Tensor memory: [0, D) dQ accumulator | kDqBufs score buffers, S_b at kDqBuf + kBufCols b
// and dP_b kTile further. Warpgroup g reads keys [G g, G g + G) of S_b and dP_b (G = kTile / 2)
// and writes dS (16-bit) over the first G / 2 of its G S_b columns, so tile t+kDqBufs's score
// MMAs wait for tile t's accumulating MMAs.
// ============================================================================================
template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
fa_bwd_dq_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const BwdArgs p) {
  using C = Cfg<D>;
  constexpr int TILE = C::kTile, G = TILE / 2;
  constexpr uint32_t kDqAcc = 0;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  const Bars<D> bars(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * kRows;
  const int kvh = h / (p.Hq / p.Hkv);
  int k_end = p.Nk;
  if (p.causal) k_end = min(p.Nk, max(0, q0 + kRows + p.Nk - p.Nq));
  const int ntiles = (k_end + TILE - 1) / TILE;

  if (threadIdx.x == 0) {
    bars.init(1);
    kf::fence_mbar_init();
  }
  if (warp == kMmaWarp) kf::tc::tmem_alloc(bars.tmem_slot, kTmemCols);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *bars.tmem_slot;
  const int* abort = bars.abort_flag;

  if (warp == kProducerWarp) {
    if (lane == 0)
      produce<D, false>(bars, smem, &tm_q, &tm_do, &tm_k, &tm_v, h, q0, b, TileWalk{kvh, 0, max(ntiles, 1), TILE},
                        ntiles, p);
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, TILE, false, false);
      const uint32_t q_addr = kf::smem_u32(smem), do_addr = q_addr + C::kStatBytes;
      bool ok = wait_relaxed(bars.stat_full, 0, abort);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int buf = t % C::kDqBufs, st = t % C::kStages;
        if (!(ok = wait_relaxed(&bars.ring_full[st], (t / C::kStages) & 1, abort))) break;
        kf::tc::fence_after_sync();
        const uint32_t k_addr = kf::smem_u32(smem + C::kRingOffset + st * 2 * C::kTileBytes);
        const uint32_t s_col = tmem + C::kDqBuf + C::kBufCols * buf;
        issue_scores<D, TILE>(q_addr, k_addr, s_col, idS);                          // S  = Q K^T
        issue_scores<D, TILE>(do_addr, k_addr + C::kTileBytes, s_col + TILE, idS);  // dP = dO V^T
        kf::tc::commit(&bars.s_full[buf]);
      }
    }
  } else if (warp == kOutWarp) {
    if (lane == 0) {
      constexpr uint32_t idA = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, D, false, true);
      uint32_t started = 0;
      bool ok = true;
      // Score buffers start free: the first kDqBufs tiles' buffer arrivals.
      for (int t = 0; t < C::kDqBufs; ++t) kf::mbar_arrive(&bars.ring_full[t % C::kStages]);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int buf = t % C::kDqBufs, st = t % C::kStages;
        if (!(ok = wait_relaxed(&bars.p_full[buf], (t / C::kDqBufs) & 1, abort))) break;
        kf::tc::fence_after_sync();
        const uint32_t k_addr = kf::smem_u32(smem + C::kRingOffset + st * 2 * C::kTileBytes);
        issue_accumulate<TILE, true>(tmem + kDqAcc, tmem + C::kDqBuf + C::kBufCols * buf, k_addr, idA,
                                     started);  // dQ += dS K
        kf::tc::commit(&bars.ring_empty[st]);
        // Buffer `buf` is free for tile t + kDqBufs (that tile's ring stage: its phase is the
        // next one to complete there, as the score thread already waited for tile t).
        kf::tc::commit(&bars.ring_full[(t + C::kDqBufs) % C::kStages]);
      }
      kf::tc::commit(bars.acc_full);
    }
  } else {
    const int group = warp >> 2, quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int64_t stat = (static_cast<int64_t>(b) * p.Hq + h) * p.NqP + qrow;  // qrow < NqP
    const float nlse = p.row_nlse[stat], ndelta = p.row_ndelta[stat];
    const int limit = p.causal ? min(p.Nk, qrow + p.Nk - p.Nq + 1) : p.Nk;  // keys [0, limit) visible
    const uint64_t c2 = kf::f2_pack(p.scale_log2, p.scale_log2), nl2 = kf::f2_pack(nlse, nlse);
    const uint64_t nd2 = kf::f2_pack(ndelta, ndelta);
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t % C::kDqBufs;
      ok = __all_sync(0xffffffffu, wait(&bars.s_full[buf], (t / C::kDqBufs) & 1, abort));  // .sync.aligned copies follow
      if (!ok) break;
      kf::tc::fence_after_sync();
      const uint32_t s_col = lane_base + C::kDqBuf + C::kBufCols * buf + G * group;  // this warpgroup's G keys
      const int kc = t * TILE + G * group;
      const bool full = kc + G <= limit;
      uint32_t sv[G], dv[G], dd[G / 2];
      tm_load<G>(s_col, sv);
      tm_load<G>(s_col + TILE, dv);
      kf::tc::wait_ld();
#pragma unroll
      for (int i = 0; i < G / 2; ++i) {
        const float2 a = kf::f2_unpack(
            kf::f2_fma(kf::f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), c2, nl2));
        float p0 = ex2(a.x), p1 = ex2(a.y);
        if (!full) {
          p0 = kc + 2 * i < limit ? p0 : 0.f;
          p1 = kc + 2 * i + 1 < limit ? p1 : 0.f;
        }
        const uint64_t ds = kf::f2_mul(
            kf::f2_pack(p0, p1), kf::f2_add(kf::f2_pack(__uint_as_float(dv[2 * i]), __uint_as_float(dv[2 * i + 1])), nd2));
        const float2 df = kf::f2_unpack(ds);
        dd[i] = pack2(df.x, df.y, kBf16);
      }
      tm_store<G / 2>(s_col, dd);
      kf::tc::wait_st();
      kf::tc::fence_before_sync();
      kf::mbar_arrive(&bars.p_full[buf]);
    }
    // Epilogue: dQ = gamma acc; warpgroup g writes columns [g D/2, (g + 1) D/2).
    if (ok) ok = wait(bars.acc_full, 0, abort);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      kf::tc::fence_after_sync();
      T* dst = static_cast<T*>(p.dq) + ((static_cast<int64_t>(b) * p.Nq + qrow) * p.Hq + h) * p.D;  // real head dim
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int c = group * (D / 64) + cc;  // 32-column chunk
        uint32_t ar[32];
        kf::tc::ld_32x32b_x32(lane_base + kDqAcc + c * 32, ar);
        kf::tc::wait_ld();
        if (qrow < p.Nq) store_row32<T>(dst + c * 32, ar, p.scale, ntiles > 0, p.D - c * 32);
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
// dK, dV. Tensor memory: [0, kAccN) dV | [kAccN, 2 kAccN) dK | kDkdvBufs score buffers: S^T_b at
// 2 kAccN + kBufCols b, dP^T_b kTile further (3 buffers for D = 64 and 256, 2 for D = 128).
// Warpgroup g reads queries [G g, G g + G) of S^T_b and dP^T_b (G = kTile / 2) and writes P^T
// and dS^T (16-bit) over the first G / 2 of those G columns, so tile t+kBufs's score MMAs wait
// for tile t's accumulating MMAs. D = 256: CTA 2 k + c of the grid's x axis is key block k and
// head-dim half c (dV, dK columns [128 c, 128 c + 128)).
// ============================================================================================
template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
fa_bwd_dkdv_sm100_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                         const BwdArgs p) {
  using C = Cfg<D>;
  constexpr int TILE = C::kTile, G = TILE / 2;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kDv = 0, kDk = C::kAccN, kBuf = C::kDkdvBuf;
  constexpr int kBufs = C::kDkdvBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  const Bars<D> bars(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int half = C::kHalves > 1 ? static_cast<int>(blockIdx.x) % C::kHalves : 0;
  const int k0 = static_cast<int>(blockIdx.x) / C::kHalves * kRows;
  const int group = p.Hq / p.Hkv;
  // Key k is visible to query q iff q >= k + Nq - Nk (causal): queries below k0 + Nq - Nk see
  // none of these keys.
  const int q_first = p.causal ? max(0, k0 + p.Nq - p.Nk) : 0;
  const int qt_first = q_first / TILE;
  const int qt_count = max(0, (p.Nq + TILE - 1) / TILE - qt_first);
  const int ntiles = group * qt_count;
  const TileWalk walk{kvh * group, qt_first, max(qt_count, 1), TILE};

  if (threadIdx.x == 0) {
    bars.init(1);
    kf::fence_mbar_init();
  }
  if (warp == kMmaWarp) kf::tc::tmem_alloc(bars.tmem_slot, kTmemCols);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *bars.tmem_slot;
  const int* abort = bars.abort_flag;

  if (warp == kProducerWarp) {
    if (lane == 0) produce<D, true>(bars, smem, &tm_k, &tm_v, &tm_q, &tm_do, kvh, k0, b, walk, ntiles, p);
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, TILE, false, false);
      const uint32_t k_addr = kf::smem_u32(smem), v_addr = k_addr + C::kStatBytes;
      bool ok = wait_relaxed(bars.stat_full, 0, abort);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int buf = t % kBufs, st = t % C::kStages;
        if (!(ok = wait_relaxed(&bars.ring_full[st], (t / C::kStages) & 1, abort))) break;
        kf::tc::fence_after_sync();
        const uint32_t q_addr = kf::smem_u32(smem + C::kRingOffset + st * 2 * C::kTileBytes);
        const uint32_t s_col = tmem + kBuf + C::kBufCols * buf;
        issue_scores<D, TILE>(k_addr, q_addr, s_col, idS);                          // S^T  = K Q^T
        issue_scores<D, TILE>(v_addr, q_addr + C::kTileBytes, s_col + TILE, idS);   // dP^T = V dO^T
        kf::tc::commit(&bars.s_full[buf]);
      }
    }
  } else if (warp == kOutWarp) {
    if (lane == 0) {
      constexpr uint32_t idA = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, C::kAccN, false, true);
      // This CTA's head-dim columns of dO and Q: 64-column blocks TILE x 128 bytes apart.
      const uint32_t bcol = static_cast<uint32_t>(half) * (C::kAccN / 64) * TILE * 128;
      uint32_t v_started = 0, k_started = 0;
      bool ok = true;
      // Score buffers start free: the first kBufs tiles' buffer arrivals.
      for (int t = 0; t < kBufs; ++t) kf::mbar_arrive(&bars.ring_full[t % C::kStages]);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int buf = t % kBufs, st = t % C::kStages;
        if (!(ok = wait_relaxed(&bars.p_full[buf], (t / kBufs) & 1, abort))) break;
        kf::tc::fence_after_sync();
        const uint32_t q_addr = kf::smem_u32(smem + C::kRingOffset + st * 2 * C::kTileBytes) + bcol;
        const uint32_t s_col = tmem + kBuf + C::kBufCols * buf;
        issue_accumulate<TILE, true>(tmem + kDv, s_col, q_addr + C::kTileBytes, idA, v_started);  // dV += P^T dO
        issue_accumulate<TILE, true>(tmem + kDk, s_col + TILE, q_addr, idA, k_started);           // dK += dS^T Q
        kf::tc::commit(&bars.ring_empty[st]);
        kf::tc::commit(&bars.ring_full[(t + kBufs) % C::kStages]);  // buffer free for tile t + kBufs
      }
      kf::tc::commit(bars.acc_full);
    }
  } else {
    const int wg = warp >> 2, quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int key = k0 + row;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int q_min = p.causal ? key + p.Nq - p.Nk : INT_MIN;  // queries [q_min, Nq) see this key
    const uint64_t c2 = kf::f2_pack(p.scale_log2, p.scale_log2);
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t % kBufs;
      ok = __all_sync(0xffffffffu, wait(&bars.s_full[buf], (t / kBufs) & 1, abort));
      if (!ok) break;
      kf::tc::fence_after_sync();
      const uint32_t s_col = lane_base + kBuf + C::kBufCols * buf + G * wg;  // this warpgroup's G queries
      const int r0 = walk.row0(t) + G * wg;
      const bool full = r0 >= q_min;
      const float* rs =
          reinterpret_cast<const float*>(smem + C::kRowStatOffset + (t % C::kStages) * 2 * TILE * 4) + G * wg;
      uint32_t sv[G], dv[G], pp[G / 2], dd[G / 2];
      tm_load<G>(s_col, sv);
      tm_load<G>(s_col + TILE, dv);
      kf::tc::wait_ld();
#pragma unroll
      for (int i = 0; i < G / 2; ++i) {
        const float2 nl = *reinterpret_cast<const float2*>(rs + 2 * i);
        const float2 nd = *reinterpret_cast<const float2*>(rs + TILE + 2 * i);
        const float2 a = kf::f2_unpack(
            kf::f2_fma(kf::f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), c2, kf::f2_pack(nl.x, nl.y)));
        float p0 = ex2(a.x), p1 = ex2(a.y);
        if (!full) {
          p0 = r0 + 2 * i >= q_min ? p0 : 0.f;
          p1 = r0 + 2 * i + 1 >= q_min ? p1 : 0.f;
        }
        const uint64_t ds = kf::f2_mul(
            kf::f2_pack(p0, p1),
            kf::f2_add(kf::f2_pack(__uint_as_float(dv[2 * i]), __uint_as_float(dv[2 * i + 1])), kf::f2_pack(nd.x, nd.y)));
        const float2 df = kf::f2_unpack(ds);
        pp[i] = pack2(p0, p1, kBf16);
        dd[i] = pack2(df.x, df.y, kBf16);
      }
      tm_store<G / 2>(s_col, pp);
      tm_store<G / 2>(s_col + TILE, dd);
      kf::tc::wait_st();
      kf::tc::fence_before_sync();
      kf::mbar_arrive(&bars.p_full[buf]);
    }
    // Epilogue: dV = acc, dK = gamma acc; warpgroup g writes accumulator columns
    // [g kAccN / 2, (g + 1) kAccN / 2), head-dim columns half * kAccN further.
    if (ok) ok = wait(bars.acc_full, 0, abort);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      kf::tc::fence_after_sync();
      const int64_t off = ((static_cast<int64_t>(b) * p.Nk + key) * p.Hkv + kvh) * p.D;  // real head dim
      const int col0 = half * C::kAccN;
      T* dk = static_cast<T*>(p.dk) + off + col0;
      T* dv = static_cast<T*>(p.dv) + off + col0;
#pragma unroll
      for (int cc = 0; cc < C::kAccN / 64; ++cc) {
        const int c = wg * (C::kAccN / 64) + cc;
        uint32_t ar[32], br[32];
        kf::tc::ld_32x32b_x32(lane_base + kDv + c * 32, ar);
        kf::tc::ld_32x32b_x32(lane_base + kDk + c * 32, br);
        kf::tc::wait_ld();
        if (key < p.Nk && col0 + c * 32 < p.D) {
          store_row32<T>(dv + c * 32, ar, 1.f, ntiles > 0, p.D - col0 - c * 32);
          store_row32<T>(dk + c * 32, br, p.scale, ntiles > 0, p.D - col0 - c * 32);
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
// dQ, dK, dV in one key-stationary kernel (head dims up to 128; dQ summed at L2, so its
// summation order varies from run to run). The dK / dV kernel's schedule, plus per tile
//   dQ^T = K^T dS^T     M = head dim, N = 64 queries, K = 128 keys; A = K (MN-major, as loaded),
//                       B = dS^T (MN-major, written to shared memory by the softmax warps)
// into the tile's dP^T columns, which the softmax warps have read by then. P^T and dS^T (16-bit)
// share the S^T columns: warpgroup g's P^T at 32 g, its dS^T at 32 g + 16. Warps 11..14 read
// dQ^T (one head-dim row per lane; their reads free the score buffer), write it transposed into
// their own 64-query x 32-column fp32 box in shared memory, and add the box to dq_acc with one
// TMA tensor reduction, performed at L2 (at D = 128 about 4% faster per call than a per-lane
// red.global.add of the same values). At D = 64 the dQ^T MMA is M = 128 over K's block and V's
// (lanes 64..127, V^T dS^T, are not read).
// ============================================================================================
constexpr int kFusedThreads = 480;
constexpr int kDqWarp0 = 11;

template <typename T, int D>
__global__ void __launch_bounds__(kFusedThreads, 1)
fa_bwd_fused_sm100_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_dq, const BwdArgs p) {
  using C = Cfg<D, true>;
  constexpr int TILE = C::kTile, G = TILE / 2;
  static_assert(TILE == 64 && C::kAccN == D, "64-query tiles, one CTA per key block");
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kDv = 0, kDk = D, kBuf = C::kDkdvBuf;
  constexpr int kBufs = C::kDkdvBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  const Bars<D> bars(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int k0 = static_cast<int>(blockIdx.x) * kRows;
  const int group = p.Hq / p.Hkv;
  const int q_first = p.causal ? max(0, k0 + p.Nq - p.Nk) : 0;
  const int qt_first = q_first / TILE;
  const int qt_count = max(0, (p.Nq + TILE - 1) / TILE - qt_first);
  const int ntiles = group * qt_count;
  const TileWalk walk{kvh * group, qt_first, max(qt_count, 1), TILE};

  if (threadIdx.x == 0) {
    // A score buffer is free once each dQ warp has read its dQ^T rows and the dV / dK MMAs that
    // read its P^T and dS^T have completed (the accumulating thread's commit).
    bars.init(5);
    kf::fence_mbar_init();
  }
  if (warp == kMmaWarp) kf::tc::tmem_alloc(bars.tmem_slot, kTmemCols);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *bars.tmem_slot;
  const int* abort = bars.abort_flag;

  if (warp == kProducerWarp) {
    if (lane == 0) produce<D, true>(bars, smem, &tm_k, &tm_v, &tm_q, &tm_do, kvh, k0, b, walk, ntiles, p);
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, TILE, false, false);
      const uint32_t k_addr = kf::smem_u32(smem), v_addr = k_addr + C::kStatBytes;
      bool ok = wait_relaxed(bars.stat_full, 0, abort);
      if (!ok) note_gave_up(2, -1);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int buf = t % kBufs, st = t % C::kStages;
        if (!(ok = wait_relaxed(&bars.ring_full[st], (t / C::kStages) & 1, abort))) {
          note_gave_up(2, t);
          break;
        }
        kf::tc::fence_after_sync();
        const uint32_t q_addr = kf::smem_u32(smem + C::kRingOffset + st * 2 * C::kTileBytes);
        const uint32_t s_col = tmem + kBuf + C::kBufCols * buf;
        issue_scores<D, TILE>(k_addr, q_addr, s_col, idS);                          // S^T  = K Q^T
        issue_scores<D, TILE>(v_addr, q_addr + C::kTileBytes, s_col + TILE, idS);   // dP^T = V dO^T
        kf::tc::commit(&bars.s_full[buf]);
      }
      kf::tc::commit(bars.drain);  // completes once every MMA issued above has
    }
  } else if (warp == kOutWarp) {
    if (lane == 0) {
      constexpr uint32_t idA = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, D, false, true);
      constexpr uint32_t idQ = kf::tc::idesc_f16(kBf16 ? 1 : 0, kRows, TILE, true, true);
      // K^T: 64-element head-dim blocks one K box (kRows x 128 bytes) apart; at D = 64 the
      // second block is V's.
      const uint64_t kt_desc = kf::tc::desc_sw128(kf::smem_u32(smem), kRows * 128, 1024);
      uint32_t v_started = 0, k_started = 0;
      // Score buffers start free: this thread's share of the first kBufs tiles' buffer arrivals.
      for (int t = 0; t < kBufs; ++t) kf::mbar_arrive(&bars.ring_full[t % C::kStages]);
      bool ok = wait_relaxed(bars.stat_full, 0, abort);
      if (!ok) note_gave_up(3, -1);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int buf = t % kBufs, st = t % C::kStages;
        if (!(ok = wait_relaxed(&bars.p_full[buf], (t / kBufs) & 1, abort))) {
          note_gave_up(3, t);
          break;
        }
        kf::tc::fence_after_sync();
        const uint32_t q_addr = kf::smem_u32(smem + C::kRingOffset + st * 2 * C::kTileBytes);
        const uint32_t s_col = tmem + kBuf + C::kBufCols * buf;
        // dQ^T = K^T dS^T first, over the block's 128 keys (16 keys, 2048 bytes of both operands, a
        // step): the dQ warps read it out while the dV / dK MMAs run.
        const uint64_t ds_desc =
            kf::tc::desc_sw128(kf::smem_u32(smem + C::kDsOffset + buf * C::kDsBytes), kRows * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < kRows / 16; ++kk)
          kf::tc::mma_ss(s_col + TILE, kf::tc::desc_advance(kt_desc, kk * 2048),
                         kf::tc::desc_advance(ds_desc, kk * 2048), idQ, kk > 0);
        kf::tc::commit(&bars.dq_full[buf]);
        issue_accumulate<TILE, true>(tmem + kDv, s_col, q_addr + C::kTileBytes, idA, v_started);  // dV += P^T dO
        issue_accumulate<TILE, true>(tmem + kDk, s_col + G / 2, q_addr, idA, k_started);          // dK += dS^T Q
        kf::tc::commit(&bars.ring_empty[st]);
        kf::tc::commit(&bars.ring_full[(t + kBufs) % C::kStages]);  // P^T, dS^T read: buffer free for t + kBufs
      }
      kf::tc::commit(bars.acc_full);
      kf::tc::commit(bars.drain);
    }
  } else if (warp >= kDqWarp0) {
    const int quarter = warp & 3;        // this lane's head-dim row of dQ^T: quarter * 32 + lane
    const bool live = quarter * 32 < D;  // warp-uniform
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float* box = reinterpret_cast<float*>(smem + C::kDqStageOffset + quarter * C::kDqBoxBytes);
    if (live && lane == 0) kf::prefetch_tensormap(&tm_dq);
    // Score buffers start free: the first kBufs tiles' buffer arrivals.
    if (lane == 0)
      for (int t = 0; t < kBufs; ++t) kf::mbar_arrive(&bars.ring_full[t % C::kStages]);
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t % kBufs;
      if (!__all_sync(0xffffffffu, wait(&bars.dq_full[buf], (t / kBufs) & 1, abort))) {
        if (lane == 0) note_gave_up(6, t);
        break;
      }
      kf::tc::fence_after_sync();
      uint32_t va[32], vb[32];  // queries 0..31, 32..63 of the tile
      if (live) {
        const uint32_t col = lane_base + kBuf + C::kBufCols * buf + TILE;
        kf::tc::ld_32x32b_x32(col, va);
        kf::tc::ld_32x32b_x32(col + 32, vb);
        kf::tc::wait_ld();
      }
      kf::tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) kf::mbar_arrive(&bars.ring_full[(t + kBufs) % C::kStages]);  // free for tile t + kBufs
      if (live) {
        // The box holds query j's 32 head-dim values of this quarter in row j (128 bytes): lanes
        // write consecutive floats. Its previous reduction must have read it first.
        if (lane == 0) kf::tma_store_wait_read0();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          box[j * 32 + lane] = __uint_as_float(va[j]);
          box[(j + 32) * 32 + lane] = __uint_as_float(vb[j]);
        }
        kf::fence_proxy_async_smem();  // the TMA reads the box through the async proxy
        __syncwarp();
        if (lane == 0) {
          // Rows r0..r0+63 of dq_acc viewed as [B Hq NqP, Dp] (r0 + 64 <= NqP), columns
          // quarter * 32 .. + 31.
          kf::tma_reduce_add_2d(&tm_dq, box, quarter * 32, (b * p.Hq + walk.head(t)) * p.NqP + walk.row0(t));
          kf::tma_store_commit();
        }
      }
    }
    if (live && lane == 0) kf::tma_store_wait_all0();  // every reduction complete before exit
  } else {
    const int wg = warp >> 2, quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int key = k0 + row;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int q_min = p.causal ? key + p.Nq - p.Nk : INT_MIN;  // queries [q_min, Nq) see this key
    const uint64_t c2 = kf::f2_pack(p.scale_log2, p.scale_log2);
    bool ok = true;
    for (int t = 0; ok && t < ntiles; ++t) {
      const int buf = t % kBufs;
      ok = __all_sync(0xffffffffu, wait(&bars.s_full[buf], (t / kBufs) & 1, abort));
      if (!ok) {
        if (lane == 0) note_gave_up(4, t);
        break;
      }
      kf::tc::fence_after_sync();
      const uint32_t s_col = lane_base + kBuf + C::kBufCols * buf + G * wg;  // this warpgroup's G queries
      const int r0 = walk.row0(t) + G * wg;
      const bool full = r0 >= q_min;
      const float* rs =
          reinterpret_cast<const float*>(smem + C::kRowStatOffset + (t % C::kStages) * 2 * TILE * 4) + G * wg;
      uint32_t sv[G], dv[G], pp[G / 2], dd[G / 2];
      tm_load<G>(s_col, sv);
      tm_load<G>(s_col + TILE, dv);
      kf::tc::wait_ld();
#pragma unroll
      for (int i = 0; i < G / 2; ++i) {
        const float2 nl = *reinterpret_cast<const float2*>(rs + 2 * i);
        const float2 nd = *reinterpret_cast<const float2*>(rs + TILE + 2 * i);
        const float2 a = kf::f2_unpack(
            kf::f2_fma(kf::f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), c2, kf::f2_pack(nl.x, nl.y)));
        float p0 = ex2(a.x), p1 = ex2(a.y);
        if (!full) {
          p0 = r0 + 2 * i >= q_min ? p0 : 0.f;
          p1 = r0 + 2 * i + 1 >= q_min ? p1 : 0.f;
        }
        const uint64_t ds = kf::f2_mul(
            kf::f2_pack(p0, p1),
            kf::f2_add(kf::f2_pack(__uint_as_float(dv[2 * i]), __uint_as_float(dv[2 * i + 1])), kf::f2_pack(nd.x, nd.y)));
        const float2 df = kf::f2_unpack(ds);
        pp[i] = pack2(p0, p1, kBf16);
        dd[i] = pack2(df.x, df.y, kBf16);
      }
      tm_store<G / 2>(s_col, pp);
      tm_store<G / 2>(s_col + G / 2, dd);
      // dS^T row `row` (128 bytes: 64 queries), this warpgroup's 64-byte half, 128-byte swizzle.
      uint8_t* ds_row = smem + C::kDsOffset + buf * C::kDsBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(ds_row + (((4 * wg + c) ^ (row & 7)) << 4)) =
            make_uint4(dd[4 * c], dd[4 * c + 1], dd[4 * c + 2], dd[4 * c + 3]);
      kf::fence_proxy_async_smem();  // the dQ MMAs read dS^T through the async proxy
      kf::tc::wait_st();
      kf::tc::fence_before_sync();
      kf::mbar_arrive(&bars.p_full[buf]);
    }
    // Epilogue: dV = acc, dK = gamma acc; warpgroup g writes columns [g D / 2, (g + 1) D / 2).
    if (ok && !wait(bars.acc_full, 0, abort)) {
      ok = false;
      note_gave_up(5, 0);
    }
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      kf::tc::fence_after_sync();
      const int64_t off = ((static_cast<int64_t>(b) * p.Nk + key) * p.Hkv + kvh) * p.D;  // real head dim
      T* dk = static_cast<T*>(p.dk) + off;
      T* dv = static_cast<T*>(p.dv) + off;
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int c = wg * (D / 64) + cc;
        uint32_t ar[32], br[32];
        kf::tc::ld_32x32b_x32(lane_base + kDv + c * 32, ar);
        kf::tc::ld_32x32b_x32(lane_base + kDk + c * 32, br);
        kf::tc::wait_ld();
        if (key < p.Nk && c * 32 < p.D) {
          store_row32<T>(dv + c * 32, ar, 1.f, ntiles > 0, p.D - c * 32);
          store_row32<T>(dk + c * 32, br, p.scale, ntiles > 0, p.D - c * 32);
        }
      }
    }
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    // Tensor memory is freed only once both issuing threads' MMAs have completed, also when a
    // wait above gave up with MMAs in flight.
    if (lane == 0 && !wait(bars.drain, 0, abort) && !wait_drain_again(bars.drain)) note_gave_up(7, 0);
    __syncwarp();
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D>
int launch_fused(const BwdArgs& a, int dtype, cudaStream_t stream) {
  using C = Cfg<D, true>;
  if (a.dq_acc == nullptr || a.Dp != D) return KF_ERR_INVALID_ARGUMENT;
  CUtensorMap mk, mv, mq, mdo, mdq;
  // dq_acc [B, Hq, NqP, Dp] fp32 as a 2-D map of B Hq NqP rows, boxes of 64 rows x 32 columns.
  const uint64_t dq_dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(a.B) * a.Hq * a.NqP};
  const uint64_t dq_strides[1] = {static_cast<uint64_t>(D) * 4};
  const uint32_t dq_box[2] = {32, 64};
  if (dq_dims[1] > (uint64_t(1) << 31)) return KF_ERR_UNSUPPORTED;  // TMA row coordinates are 32-bit
  if (!encode_bnhd(&mk, a.k, dtype, a.B, a.Nk, a.Hkv, a.D, kRows) ||
      !encode_bnhd(&mv, a.v, dtype, a.B, a.Nk, a.Hkv, a.D, kRows) ||
      !encode_bnhd(&mq, a.q, dtype, a.B, a.Nq, a.Hq, a.D, C::kTile) ||
      !encode_bnhd(&mdo, a.dout, dtype, a.B, a.Nq, a.Hq, a.D, C::kTile) ||
      !kf_host::encode_tiled(&mdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.dq_acc, dq_dims, dq_strides, dq_box,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
    return KF_ERR_CUDA;
  auto kernel = fa_bwd_fused_sm100_kernel<T, D>;
  const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kFusedThreads, C::kSmemBytes, nullptr);
  if (prep != KF_OK) return prep;
  kernel<<<dim3((a.Nk + kRows - 1) / kRows, a.Hkv, a.B), kFusedThreads, C::kSmemBytes, stream>>>(mk, mv, mq, mdo,
                                                                                                 mdq, a);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

template <typename T, int D>
int launch(const BwdArgs& a, int dtype, cudaStream_t stream) {
  using C = Cfg<D>;
  {
    CUtensorMap mq, mdo, mk, mv;
    // The maps carry the real head dim: boxes past it (D < 128 or < 256) read as zeros.
    if (!encode_bnhd(&mq, a.q, dtype, a.B, a.Nq, a.Hq, a.D, kRows) ||
        !encode_bnhd(&mdo, a.dout, dtype, a.B, a.Nq, a.Hq, a.D, kRows) ||
        !encode_bnhd(&mk, a.k, dtype, a.B, a.Nk, a.Hkv, a.D, C::kTile) ||
        !encode_bnhd(&mv, a.v, dtype, a.B, a.Nk, a.Hkv, a.D, C::kTile))
      return KF_ERR_CUDA;
    auto kernel = fa_bwd_dq_sm100_kernel<T, D>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kThreads, C::kSmemBytes, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3((a.Nq + kRows - 1) / kRows, a.Hq, a.B), kThreads, C::kSmemBytes, stream>>>(mq, mdo, mk, mv, a);
    KF_LAUNCH_CHECK();
  }
  {
    CUtensorMap mk, mv, mq, mdo;
    if (!encode_bnhd(&mk, a.k, dtype, a.B, a.Nk, a.Hkv, a.D, kRows) ||
        !encode_bnhd(&mv, a.v, dtype, a.B, a.Nk, a.Hkv, a.D, kRows) ||
        !encode_bnhd(&mq, a.q, dtype, a.B, a.Nq, a.Hq, a.D, C::kTile) ||
        !encode_bnhd(&mdo, a.dout, dtype, a.B, a.Nq, a.Hq, a.D, C::kTile))
      return KF_ERR_CUDA;
    auto kernel = fa_bwd_dkdv_sm100_kernel<T, D>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kThreads, C::kSmemBytes, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3((a.Nk + kRows - 1) / kRows * C::kHalves, a.Hkv, a.B), kThreads, C::kSmemBytes, stream>>>(
        mk, mv, mq, mdo, a);
    KF_LAUNCH_CHECK();
  }
  return KF_OK;
}

}  // namespace

int kf_internal_fa_bwd_error(unsigned int* code) {
  unsigned int v = 0;
  KF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fa_bwd_error, sizeof(v)));
  if (v != 0) {
    const unsigned int zero = 0;
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_fa_bwd_error, &zero, sizeof(zero)));
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_fa_bwd_where, &zero, sizeof(zero)));
  }
  *code = v;
  return KF_OK;
}

// Where the first bounded wait of the backward kernels gave up (role << 24 | tile), 0 if none;
// read before kf_internal_fa_bwd_error clears it.
int kf_internal_fa_bwd_where(unsigned int* where) {
  KF_CUDA_TRY(cudaMemcpyFromSymbol(where, g_fa_bwd_where, sizeof(*where)));
  return KF_OK;
}

namespace kf::fa {

// Head dims up to 256: 8..56 run the D = 64 kernels, 72..120 the D = 128 kernels and 136..248
// the D = 256 kernels on zero-padded tiles.
bool sm100_bwd_supported(const BwdArgs& a) { return a.D >= 8 && a.D <= 256; }

int launch_sm100_bwd(const BwdArgs& a, int dtype, cudaStream_t s) {
  if (a.dq_acc != nullptr) {  // one kernel, dQ summed at L2 (head dims up to 128)
    if (a.D > 128) return KF_ERR_INVALID_ARGUMENT;
    if (dtype == KF_DTYPE_BF16)
      return a.D <= 64 ? launch_fused<__nv_bfloat16, 64>(a, dtype, s) : launch_fused<__nv_bfloat16, 128>(a, dtype, s);
    return a.D <= 64 ? launch_fused<__half, 64>(a, dtype, s) : launch_fused<__half, 128>(a, dtype, s);
  }
  if (dtype == KF_DTYPE_BF16) {
    if (a.D > 128) return launch<__nv_bfloat16, 256>(a, dtype, s);
    return a.D <= 64 ? launch<__nv_bfloat16, 64>(a, dtype, s) : launch<__nv_bfloat16, 128>(a, dtype, s);
  }
  if (a.D > 128) return launch<__half, 256>(a, dtype, s);
  return a.D <= 64 ? launch<__half, 64>(a, dtype, s) : launch<__half, 128>(a, dtype, s);
}

}  // namespace kf::fa
