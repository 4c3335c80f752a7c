// SANA ReLU linear attention over packed QKV for sm_100a.
//
// Computes LiteLA.attn_matmul (SANA_LinearAttention/original.py:99-117) as the reference's
// split-sequence kernels do (SANA_LinearAttention/custom.py:98-388), in two launches:
//
//  1. sana_vk_producer   grid (splits, head pairs, batch)
//     Each CTA streams its token range of K and V for a head pair through a TMA/mbarrier ring
//     (SWIZZLE_128B boxes of 64 tokens x 2 heads) and accumulates, per head (one warp),
//         VK[r][c] += v[t][r] * relu(k[t][c])      (mma.sync m16n8k16, fp32 accumulators)
//         ksum[c]  += relu(k[t][c])                (fp32, from the same B fragments)
//     and writes this split's fp32 partial [VK ; ksum] (33 x 32 per head) to the workspace.
//     The per-head product is 32 x 32: below tcgen05's smallest M, so the warp-level MMA does
//     it; it hides under the K/V stream.
//  2. sana_out_tc        persistent, one CTA per (SM, slot), programmatic dependent launch
//     out[t][r] = (VK relu(q_t))_r / (ksum . relu(q_t) + eps) on the tcgen05 tensor cores,
//     128 tokens x one head pair per item: relu(Q) in tensor memory as operand A, the
//     split-summed [VK ; ksum] as hi + lo 16-bit halves in shared memory as operand B (so the
//     fp32 sums keep ~16 mantissa bits), fp32 accumulators in tensor memory; ksum is the 33rd
//     row of B, like the reference's ones-row padding. The output tile is staged in shared
//     memory and written with a TMA store.
//
// Intensity is ~16 flop/byte: the path is HBM-bound. K/V are read once by (1), Q read once
// and out written once by (2); the partials (S x 4 KB per head) stay in L2.
// Shapes outside the fast path (fp32 input, head dims other than 32, tiny tensors) run the
// generic kernels below (CUDA-core fp32 arithmetic, partials reduced by the last CTA).
#include "kf_sm100.cuh"
#include "kf_tcgen05.cuh"

#include <algorithm>
#include <type_traits>

namespace {

__device__ unsigned int g_sana_error = 0;

constexpr int kD = 32;                 // fast-path head dim
constexpr int kTok = 64;               // tokens per tile / TMA box
constexpr int kBoxBytes = kTok * 128;  // 64 tokens x 128 bytes
constexpr int kRows = kD + 1;          // 32 VK rows + the ksum row

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Split count of the generic path: ~2 CTAs per SM over (batch, head) units.
int generic_splits(int64_t B, int64_t H, int64_t N, int64_t requested) {
  const int64_t tiles = std::max<int64_t>(1, ceil_div(N, kTok));
  int64_t s = requested;
  if (s <= 0) {
    const int64_t units = std::max<int64_t>(1, B * H);
    const int64_t target = static_cast<int64_t>(kf_host::current_device_sms()) * 2;
    s = std::max<int64_t>(1, (target + units / 2) / units);
  }
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({s, tiles, 1024})));
}

// Fast path: the producer's CTAs are (split, batch, head pair); default about two per SM.
constexpr int kFastHeads = 2;
constexpr int kMaxFastSplits = 8;  // the epilogue stages all splits of a head pair at once
int fast_splits(int64_t B, int64_t H, int64_t N, int64_t requested) {
  const int64_t tiles = std::max<int64_t>(1, ceil_div(N, kTok));
  int64_t s = requested;
  if (s <= 0) {
    const int64_t units = B * ceil_div(H, kFastHeads);
    const int64_t target = static_cast<int64_t>(kf_host::current_device_sms()) * 2;
    s = (target + units / 2) / std::max<int64_t>(units, 1);
  }
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({s, tiles, kMaxFastSplits})));
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Both paths start the workspace with the same arrival counters (B*H u32, zero between calls:
// the last CTA of each unit resets its counter), so a caller may alternate paths on one
// workspace.
//   generic: [counters | partials: B*H*S*(d+1)*d fp32 | final: B*H*(d+1)*d fp32]
//   fast:    [counters (unused) | partials: B*H*S*33*32 fp32]
struct WorkspaceLayout {
  size_t counter_off, partial_off, final_off, total;
};
WorkspaceLayout layout_for(int64_t B, int64_t H, int64_t d, int64_t S) {
  WorkspaceLayout l;
  const size_t per_head = static_cast<size_t>(d + 1) * d;
  l.counter_off = 0;
  l.partial_off = align256(static_cast<size_t>(B * H) * sizeof(unsigned int));
  l.final_off = l.partial_off + align256(static_cast<size_t>(B * H * S) * per_head * sizeof(float));
  l.total = l.final_off + align256(static_cast<size_t>(B * H) * per_head * sizeof(float));
  return l;
}

constexpr int kBHalfRows = 48;                     // B rows of one head: 32 VK rows, ksum, 15 zero
constexpr int kBImageBytes = kBHalfRows * 128;     // one head's B: 48 rows x (32 hi + 32 lo) 16-bit
struct FastLayout {
  size_t partial_off, total;
};
FastLayout fast_layout(int64_t B, int64_t H, int64_t S) {
  FastLayout l;
  l.partial_off = align256(static_cast<size_t>(B * H) * sizeof(unsigned int));
  l.total = l.partial_off + align256(static_cast<size_t>(B * H * S) * kRows * kD * sizeof(float));
  return l;
}

// Power-of-two scale that brings max|value| below 2^14 (fp16 operand range); 1 for bf16.
__device__ __forceinline__ float operand_scale(float max_abs, bool fp16) {
  if (!fp16 || !(max_abs > 0.f)) return 1.f;
  const int e = static_cast<int>((__float_as_uint(max_abs) >> 23) & 0xffu) - 126;  // max < 2^e
  const int biased = min(max(127 + 14 - e, 1), 254);
  return __uint_as_float(static_cast<uint32_t>(biased) << 23);
}

// ------------------------------------------------------------------------------------------
// qk_norm of LiteLA.forward (SANA_LinearAttention/original.py:92-96, 127-128): q and k each go
// through an RMSNorm over the C channels of their token (rmsnorm/original.py:40-52) before the
// attention, y = cast(cast(x r) w) with r = 1 / sqrt(mean(x^2) + eps). The kernels below apply
// it where they read q and k (fragment registers, or the Q rows bound for tensor memory), so the
// normalised q and k never exist in memory; r of every token comes from one stats pass
// (sana_qk_stats) into the workspace, padded to kStatsPad tokens per batch so that every tile's
// lookups stay in bounds (padded tokens carry r = 0).
// ------------------------------------------------------------------------------------------
constexpr int kStatsPad = 128;
struct QkNorm {
  const float* stats;  // [B][npad][2]: r of q, r of k per token
  const void* wq;      // [C] q_norm weight, input dtype
  const void* wk;      // [C] k_norm weight, input dtype
  int npad;            // tokens per batch in `stats` (N rounded up to kStatsPad)
};

// Two packed 16-bit values through the reference's two roundings: cast(cast(x r) w). The
// second is the product of two 16-bit values, exact in fp32 and rounded once to the dtype:
// exactly what a packed 16-bit multiply returns, so w2 (the two weights, packed) multiplies
// the packed normalised values directly.
template <typename T>
__device__ __forceinline__ uint32_t qk_apply2(uint32_t v, float r0, float r1, uint32_t w2) {
  const float2 x = kf::Mma<T>::to_f2(v);
  const float2 n = kf::f2_unpack(kf::f2_mul(kf::f2_pack(x.x, x.y), kf::f2_pack(r0, r1)));
  return kf::Mma<T>::mul2(kf::Mma<T>::from_f2(n.x, n.y), w2);
}
// A 16-bit weight in both halves of a packed pair.
template <typename T>
__device__ __forceinline__ uint32_t weight_pair(const void* w, int c) {
  const uint32_t h = static_cast<const unsigned short*>(w)[c];
  return h | (h << 16);
}
template <typename T>
__device__ __forceinline__ float qk_apply1(float x, float r, float w) {
  return kf::Elem<T>::round_f(kf::Elem<T>::round_f(x * r) * w);
}
template <typename T>
__device__ __forceinline__ float weight_at(const void* w, int c) {
  return kf::Elem<T>::to_f(static_cast<const T*>(w)[c]);
}
// r of q (which = 0) or k (which = 1) of token `tok` of batch b.
__device__ __forceinline__ float stats_at(const QkNorm& n, int b, int tok, int which) {
  return __ldg(n.stats + (static_cast<int64_t>(b) * n.npad + tok) * 2 + which);
}

// r of q (which = 0) or k (which = 1) of the even token t0 and of t0 + 1: one 16-byte load.
__device__ __forceinline__ float2 stats_pair(const QkNorm& n, int b, int t0, int which) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(n.stats + (static_cast<int64_t>(b) * n.npad + t0) * 2));
  return which ? make_float2(v.y, v.w) : make_float2(v.x, v.z);
}

// The K fragments of one 16-token step (mma.sync B operand: register 0 holds tokens t0 + 2 tig
// and + 1, register 1 tokens + 8 and + 9, of channel 8 nt + gid) through the k norm of head h.
// The weights are read where they are used (L1-resident), so nothing stays live across loops.
template <typename T>
__device__ __forceinline__ void qk_norm_k(uint32_t (&bf)[4][2], const QkNorm& n, int b, int t0, int lane, int h) {
  const int tig = lane & 3, gid = lane >> 2;
  const float2 ra = stats_pair(n, b, t0 + 2 * tig, 1), rb = stats_pair(n, b, t0 + 8 + 2 * tig, 1);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const uint32_t w = weight_pair<T>(n.wk, h * kD + nt * 8 + gid);
    bf[nt][0] = qk_apply2<T>(bf[nt][0], ra.x, ra.y, w);
    bf[nt][1] = qk_apply2<T>(bf[nt][1], rb.x, rb.y, w);
  }
}

// The Q fragments of one 16-token step (mma.sync A operand, k step ks: registers 0 / 1 hold
// tokens t0 + gid / + 8 at channels 16 ks + 2 tig, + 1; registers 2 / 3 the same at + 8)
// through the q norm of head h.
template <typename T>
__device__ __forceinline__ void qk_norm_q(uint32_t (&a)[2][4], const QkNorm& n, int b, int t0, int lane, int h) {
  const int tig = lane & 3, gid = lane >> 2;
  const float r0 = stats_at(n, b, t0 + gid, 0), r8 = stats_at(n, b, t0 + gid + 8, 0);
  const T* w = static_cast<const T*>(n.wq) + h * kD + 2 * tig;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const uint32_t lo = __ldg(reinterpret_cast<const unsigned int*>(w + ks * 16));
    const uint32_t hi = __ldg(reinterpret_cast<const unsigned int*>(w + ks * 16 + 8));
    a[ks][0] = qk_apply2<T>(a[ks][0], r0, r0, lo);
    a[ks][1] = qk_apply2<T>(a[ks][1], r8, r8, lo);
    a[ks][2] = qk_apply2<T>(a[ks][2], r0, r0, hi);
    a[ks][3] = qk_apply2<T>(a[ks][3], r8, r8, hi);
  }
}

// One warp per token: r of its q and k rows, 1 / sqrt(sum(x^2) / C + eps) in fp32 (the
// reference's rsqrt of the mean), 0 for the padding tokens N .. npad - 1.
template <typename T>
__global__ void __launch_bounds__(256)
sana_qk_stats(const T* __restrict__ qkv, float* __restrict__ stats, int N, int C, int npad, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok = blockIdx.x * 8 + warp, b = blockIdx.y;
  if (tok >= npad) return;
  float rq = 0.f, rk = 0.f;
  if (tok < N) {
    const T* q = qkv + (static_cast<int64_t>(b) * N + tok) * 3 * C;
    const T* k = q + C;
    float sq = 0.f, sk = 0.f;
    if constexpr (sizeof(T) == 2) {
      if ((C & 7) == 0) {
        for (int c = lane * 8; c < C; c += 256) {
          const uint4 a = *reinterpret_cast<const uint4*>(q + c), e = *reinterpret_cast<const uint4*>(k + c);
          const uint32_t av[4] = {a.x, a.y, a.z, a.w}, ev[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 x = kf::Mma<T>::to_f2(av[i]), y = kf::Mma<T>::to_f2(ev[i]);
            sq = fmaf(x.x, x.x, fmaf(x.y, x.y, sq));
            sk = fmaf(y.x, y.x, fmaf(y.y, y.y, sk));
          }
        }
      } else {
        for (int c = lane; c < C; c += 32) {
          const float x = kf::Elem<T>::to_f(q[c]), y = kf::Elem<T>::to_f(k[c]);
          sq = fmaf(x, x, sq);
          sk = fmaf(y, y, sk);
        }
      }
    } else {
      for (int c = lane; c < C; c += 32) {
        sq = fmaf(q[c], q[c], sq);
        sk = fmaf(k[c], k[c], sk);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    rq = 1.f / sqrtf(sq / static_cast<float>(C) + eps);
    rk = 1.f / sqrtf(sk / static_cast<float>(C) + eps);
  }
  if (lane == 0)
    *reinterpret_cast<float2*>(stats + (static_cast<int64_t>(b) * npad + tok) * 2) = make_float2(rq, rk);
}

// ------------------------------------------------------------------------------------------
// Fast path, kernel 1: K^T V and ksum per split; each split writes its fp32 partial.
// ------------------------------------------------------------------------------------------
template <typename T, int G, int STAGES, bool kNorm>
__global__ void __launch_bounds__(G * 32)
sana_vk_producer(const __grid_constant__ CUtensorMap qkv_map, float* __restrict__ partial, int H,
                 int tiles, int tiles_per_split, const QkNorm nrm) {
  constexpr int kPairs = G / 2;
  constexpr int kStageBytes = 2 * kPairs * kBoxBytes;  // K boxes, then V boxes
  constexpr int kHeadElems = kRows * kD;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);

  const int split = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int h0 = hg * G;
  const int t_begin = split * tiles_per_split;
  const int n_local = max(0, min(tiles, t_begin + tiles_per_split) - t_begin);

  if (threadIdx.x == 0) {
    kf::prefetch_tensormap(&qkv_map);
    for (int s = 0; s < STAGES; ++s) kf::mbar_init(&full[s], 1);
    kf::fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int local_tile, int stage) {
    uint8_t* base = smem + stage * kStageBytes;
    kf::mbar_arrive_expect_tx(&full[stage], kStageBytes);
    const int tok = (t_begin + local_tile) * kTok;
#pragma unroll
    for (int p = 0; p < kPairs; ++p) {
      const int c0 = (h0 + 2 * p) * kD;
      kf::tma_load_4d(base + p * kBoxBytes, &qkv_map, &full[stage], c0, 1, tok, b);
      kf::tma_load_4d(base + (kPairs + p) * kBoxBytes, &qkv_map, &full[stage], c0, 2, tok, b);
    }
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES && i < n_local; ++i) issue(i, i);
  }

  float acc[2][4][4];
  float ksum[4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    ksum[nt] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.f;
  }
  const int pair = warp >> 1, g = warp & 1;
  const int sub = lane >> 3;
  bool aborted = false;
  for (int i = 0; i < n_local; ++i) {
    const int stage = i % STAGES;
    const bool ok = kf::mbar_wait_bounded(&full[stage], (i / STAGES) & 1, &g_sana_error);
    if (ok) {
      const uint32_t kbase = kf::smem_u32(smem + stage * kStageBytes + pair * kBoxBytes);
      const uint32_t vbase = kf::smem_u32(smem + stage * kStageBytes + (kPairs + pair) * kBoxBytes);
#pragma unroll
      for (int ks = 0; ks < kTok / 16; ++ks) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          // A = V^T (M = v channel, K = token): transposed 8x8 loads of token-major rows.
          const int row = ks * 16 + (lane & 7) + (sub >> 1) * 8;
          const int chunk = g * 4 + mt * 2 + (sub & 1);
          kf::ldsm_x4_t(vbase + kf::swz128(row, chunk), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
        }
        uint32_t bf[4][2];
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          // B = relu(K) (K = token, N = k channel), two n-tiles per x4 load.
          const int row = ks * 16 + (lane & 7) + (sub & 1) * 8;
          const int chunk = g * 4 + np * 2 + (sub >> 1);
          kf::ldsm_x4_t(kbase + kf::swz128(row, chunk), bf[2 * np][0], bf[2 * np][1],
                        bf[2 * np + 1][0], bf[2 * np + 1][1]);
        }
        // A head past H (odd H) reads zeros: its weights are not read.
        if constexpr (kNorm) {
          if (h0 + warp < H) qk_norm_k<T>(bf, nrm, b, (t_begin + i) * kTok + ks * 16, lane, h0 + warp);
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          bf[nt][0] = kf::Mma<T>::relu2(bf[nt][0]);
          bf[nt][1] = kf::Mma<T>::relu2(bf[nt][1]);
          const float2 x = kf::Mma<T>::to_f2(bf[nt][0]);
          const float2 y = kf::Mma<T>::to_f2(bf[nt][1]);
          ksum[nt] += (x.x + x.y) + (y.x + y.y);
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) kf::Mma<T>::run(acc[mt][nt], a[mt], bf[nt]);
      }
    }
    // Everyone is done with this stage (or everyone gives up together).
    if (!__syncthreads_and(ok)) {
      aborted = true;
      break;
    }
    if (threadIdx.x == 0 && i + STAGES < n_local) issue(i + STAGES, stage);
  }

  // The epilogue grid may start its prologue (its Q loads do not depend on this kernel).
  kf::pdl_launch_dependents();
  // This split's partial [VK ; ksum] of each head -> partial[b][h][split] (33 x 32 fp32). After a
  // timeout nothing is written (the error word is set and the results are not used).
  const int h = h0 + warp;
  if (!aborted && h < H) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 1);
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 2);
    }
    float* dst = partial + ((static_cast<size_t>(b) * H + h) * S + split) * kHeadElems;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int r = mt * 16 + gid, c = nt * 8 + tig * 2;
        *reinterpret_cast<float2*>(dst + r * kD + c) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
        *reinterpret_cast<float2*>(dst + (r + 8) * kD + c) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
      }
    if (tig == 0) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) dst[kD * kD + nt * 8 + gid] = ksum[nt];
    }
  }
}

// ------------------------------------------------------------------------------------------
// Fast path, kernel 2: normalised output on the 5th-generation tensor cores.
//
// One persistent CTA per SM walks a contiguous range of items (batch, head pair, 128-token
// tile), with warp-specialised roles:
//   * workers, warps 0-15, in two groups taking alternate items. Worker warp (group g, head hd,
//     quarter q) handles tokens 32 q .. 32 q + 31 of the tile -- its tensor-memory lanes -- for
//     head hd: it writes A = relu(Q) (M = 128 tokens, K = 32 q channels, packed 16-bit pairs)
//     into tensor memory, and after the MMAs reads D = A.B (128 x 48 fp32) and writes
//     out[r][c] = D[r][c] / (D[r][32] + eps) with its own TMA store (32 tokens x 32 channels);
//   * two MMA warps (16, 17), one per group: for each of the group's items and each head, once
//     the head's four workers have prepared A, four K = 16 MMAs D = A.B_hi + A.B_lo; each also
//     keeps its group's Q stages full with TMA;
//   * B = [VK ; ksum ; 0] of a head pair, as hi + lo 16-bit halves side by side along K (so the
//     fp32 split sums keep ~16 mantissa bits), swizzled like a 128-byte TMA tile: built from the
//     producer's split partials, summed in split order (deterministic). The first two head pairs
//     of the CTA are built at the start by every non-MMA thread; later ones by the B warp (18)
//     while the workers run. fp16 inputs scale B by a power of two that keeps max|VK| below
//     2^14 (eps is scaled with it); bf16 needs no scaling.
// A and D are double-buffered per group in tensor memory (2 groups x 2 buffers x 2 heads x 64
// columns), B per head pair in shared memory. Every wait is on an mbarrier; inside the loop the
// CTA never synchronises as a whole.
// ------------------------------------------------------------------------------------------
constexpr int kOutTok = 128;                    // tokens per item
constexpr int kWorkerWarps = 16;
constexpr int kMmaWarp0 = 16;                   // MMA warps 16 (group 0) and 17 (group 1)
constexpr int kBWarp = 18;
constexpr int kEpiThreads = 32 * 19;
constexpr int kBuildThreads = 32 * (kWorkerWarps + 1);  // workers + B warp build the first B tiles
constexpr int kQTileBytes = kOutTok * 128;      // 128 tokens x one head pair (64 channels)
constexpr uint32_t kEpiTmemCols = 512;
constexpr uint32_t kBuildBar = 1;               // named barrier of the first B build
// Tensor memory of (group g, buffer j, head hd): D at 64 (4 g + 2 j + hd) + [0, 48), A at + 48 + [0, 16).
__device__ __forceinline__ uint32_t tm_slot(int g, int j, int hd) { return 64u * (4 * g + 2 * j + hd); }

template <typename O>
struct EpiCfg {
  static constexpr int kStages = sizeof(O) == 4 ? 8 : 10;                 // Q ring depth (even)
  static constexpr int kWarpOutBytes = 32 * kD * int(sizeof(O));          // 32 tokens x 32 channels
  static constexpr int kQOff = 0;
  static constexpr int kOutOff = kStages * kQTileBytes;
  static constexpr int kBOff = kOutOff + kWorkerWarps * kWarpOutBytes;    // [buffer][head] x kBImageBytes
  static constexpr int kSmemBytes = kBOff + 4 * kBImageBytes + 1024;
};
static_assert(EpiCfg<__nv_bfloat16>::kStages % 2 == 0 && EpiCfg<float>::kStages % 2 == 0,
              "each MMA warp refills its own group's stages");

// Sum of the S split partials of (head h of the pair, row n, k values 8 kg .. 8 kg + 7), in split
// order, straight from the workspace (L2).
__device__ __forceinline__ void sum_splits(const float* __restrict__ partial, int b, int h, int H, int S, int n,
                                           int kg, float (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = 0.f;
  if (h >= H) return;
  const float* src = partial + (static_cast<size_t>(b) * H + h) * S * (kRows * kD) + n * kD + kg * 8;
  constexpr int kBatch = 4;  // splits whose loads are in flight together
  for (int sp0 = 0; sp0 < S; sp0 += kBatch) {
    float4 x[kBatch][2];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (sp0 + u < S) {
        x[u][0] = __ldcg(reinterpret_cast<const float4*>(src + (sp0 + u) * (kRows * kD)));
        x[u][1] = __ldcg(reinterpret_cast<const float4*>(src + (sp0 + u) * (kRows * kD) + 4));
      }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (sp0 + u < S) {
        v[0] += x[u][0].x; v[1] += x[u][0].y; v[2] += x[u][0].z; v[3] += x[u][0].w;
        v[4] += x[u][1].x; v[5] += x[u][1].y; v[6] += x[u][1].z; v[7] += x[u][1].w;
      }
  }
}

__device__ __forceinline__ float max_abs8(const float (&v)[8]) {
  float m = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
  return m;
}

// One B row chunk: 8 k values of row n as hi and lo halves, into tile `tile` (one head).
template <typename T>
__device__ __forceinline__ void store_b_chunk(uint8_t* tile, int n, int kg, const float (&v)[8], float scale) {
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float x0 = v[2 * e] * scale, x1 = v[2 * e + 1] * scale;
    hi[e] = kf::Mma<T>::from_f2(x0, x1);
    const float2 hf = kf::Mma<T>::to_f2(hi[e]);
    lo[e] = kf::Mma<T>::from_f2(x0 - hf.x, x1 - hf.y);
  }
  uint8_t* row = tile + n * 128;
  *reinterpret_cast<uint4*>(row + ((kg ^ (n & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(row + (((4 + kg) ^ (n & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

template <typename T, typename O, bool kNorm>
__global__ void __maxnreg__(96)
sana_out_tc(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap out_map,
            const float* __restrict__ partial, int H, int S, int head_pairs, int tiles_out, int total_items,
            int items_per_cta, float eps, const QkNorm nrm) {
  using Cfg = EpiCfg<O>;
  constexpr int kStages = Cfg::kStages;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr bool kFp16 = std::is_same<T, __half>::value;
  constexpr int kTasks = 2 * kRows * 4;  // B chunks of a head pair: (head, row, group of 8 k values)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t q_full[kStages];
  __shared__ uint64_t ready[2][2][2];   // [group][head][buffer]: the head's 4 workers prepared A
  __shared__ uint64_t d_full[2][2][2];  // [group][head][buffer]: D computed
  __shared__ uint64_t b_ready[2];       // [B buffer]: B of a head pair built
  __shared__ uint64_t unit_done[2];     // [B buffer]: all 16 workers are past a head pair
  __shared__ float eps_s[2][2];         // [B buffer][head]
  __shared__ uint32_t max_bits[2][2];   // [B buffer][head]: max |VK| of the first two head pairs (fp16)
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int first = blockIdx.x * items_per_cta;
  const int n_items = min(total_items, first + items_per_cta) - first;
  if (n_items <= 0) return;  // uniform for the whole CTA
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int first_unit = first / tiles_out;
  const int n_units = (first + n_items - 1) / tiles_out - first_unit + 1;
  uint8_t* const btiles = smem + Cfg::kBOff;

  if (t == 0) {
    kf::prefetch_tensormap(&q_map);
    kf::prefetch_tensormap(&out_map);
    for (int st = 0; st < kStages; ++st) kf::mbar_init(&q_full[st], 1);
    for (int g = 0; g < 2; ++g)
      for (int h = 0; h < 2; ++h)
        for (int j = 0; j < 2; ++j) {
          kf::mbar_init(&ready[g][h][j], 4);
          kf::mbar_init(&d_full[g][h][j], 1);
        }
    for (int j = 0; j < 2; ++j) {
      kf::mbar_init(&b_ready[j], 1);
      kf::mbar_init(&unit_done[j], kWorkerWarps);
      max_bits[j][0] = max_bits[j][1] = 0u;
    }
    abort_flag = 0;
    kf::fence_mbar_init();
  }
  if (warp == kMmaWarp0) kf::tc::tmem_alloc(&tmem_slot, kEpiTmemCols);
  for (int e = t; e < 4 * (kBHalfRows - kRows) * 8; e += kEpiThreads) {  // B rows 33..47 stay zero
    const int tile = e / ((kBHalfRows - kRows) * 8), row = kRows + (e / 8) % (kBHalfRows - kRows);
    *reinterpret_cast<uint4*>(btiles + tile * kBImageBytes + row * 128 + (e % 8) * 16) = make_uint4(0, 0, 0, 0);
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  auto unit_of = [&](int k) { return (first + k) / tiles_out; };

  if (warp == kMmaWarp0 || warp == kMmaWarp0 + 1) {
    // ---- MMA issue and Q loads of group g (one thread) ----
    const int g = warp - kMmaWarp0;
    if (lane == 0) {
      uint32_t commits[2][2] = {};  // [head][buffer]
      int loaded = -1, next_load = g;
      auto load = [&](int k) {
        const int it = first + k;
        const int unit = it / tiles_out, tt = it % tiles_out;
        const int b = unit / head_pairs, hp = unit % head_pairs;
        const int st = k % kStages;
        kf::mbar_arrive_expect_tx(&q_full[st], kQTileBytes);
        kf::tma_load_4d(smem + Cfg::kQOff + st * kQTileBytes, &q_map, &q_full[st], hp * 2 * kD, 0, tt * kOutTok, b);
        loaded = k;
      };
      // Q loads: at most kStages items ahead, and only two per group before the first B is ready,
      // so that B's reads of the split partials do not queue behind the whole ring's loads.
      auto top_up = [&](int limit) {
        for (; next_load < n_items && next_load < limit; next_load += 2) load(next_load);
      };
      top_up(g + 4);
      constexpr uint32_t idesc = kf::tc::idesc_f16(kBf16 ? 1 : 0, kOutTok, kBHalfRows, false, false);
      int b_unit = -1;
      for (int k = g, i = 0; k < n_items; k += 2, ++i) {
        const int j = i & 1;
        const int u = unit_of(k) - first_unit;
        // A new head pair's B was written by ordinary stores: observe it with acquire.
        if (u != b_unit) {
          if (!kf::mbar_wait_or_abort(&b_ready[u & 1], (u >> 1) & 1, &g_sana_error, &abort_flag)) break;
          b_unit = u;
        }
        bool ok = true;
        for (int h = 0; h < 2 && ok; ++h) {
          // A arrives through tensor memory (ordered by the workers' tcgen05 fences).
          ok = kf::mbar_wait_or_abort<true>(&ready[g][h][j], (i >> 1) & 1, &g_sana_error, &abort_flag);
          if (!ok) break;
          kf::tc::fence_after_sync();
          const uint32_t slot = tm_slot(g, j, h);
          const uint32_t b_addr = kf::smem_u32(btiles + ((u & 1) * 2 + h) * kBImageBytes);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)  // hi k 0-15, hi k 16-31, lo k 0-15, lo k 16-31
            kf::tc::mma_ts(tmem + slot, tmem + slot + 48 + (ks & 1) * 8, kf::tc::desc_sw128(b_addr + ks * 32, 16, 1024),
                           idesc, ks > 0 ? 1u : 0u);
          kf::tc::commit(&d_full[g][h][j]);
          ++commits[h][j];
        }
        if (!ok) break;
        // Both heads' workers have read Q(k): the stages of this group's items up to k can take
        // items up to k + kStages (a TMA issue may block: after the MMAs). The ring fills at
        // two loads per item, not in one burst.
        top_up(min(k + kStages + 1, next_load + 4));
      }
      // Leave nothing in flight on exit (after a timeout): MMA groups and Q loads.
      for (int h = 0; h < 2; ++h)
        for (int j = 0; j < 2; ++j)
          if (commits[h][j] > 0) kf::mbar_wait_bounded(&d_full[g][h][j], (commits[h][j] - 1) & 1, &g_sana_error);
      for (int k = loaded; k >= 0 && k > loaded - kStages; k -= 2)
        kf::mbar_wait_bounded(&q_full[k % kStages], (k / kStages) & 1, &g_sana_error);
    }
  } else {
    // ---- B tiles of the first two head pairs: every worker and the B warp, one chunk each ----
    kf::pdl_wait_primary();  // the partials come from the producer grid
    const int n_first = min(n_units, 2);
    const int task = warp == kBWarp ? 32 * kWorkerWarps + lane : t;  // < kBuildThreads
    const int bu = task / kTasks, bt = task % kTasks;
    const int bh = bt / (kRows * 4), bn = (bt / 4) % kRows, bkg = bt % 4;
    const bool has_task = bu < n_first;
    float v[8];
    int bb = 0, bhp = 0;
    if (has_task) {
      const int unit = first_unit + bu;
      bb = unit / head_pairs;
      bhp = unit % head_pairs;
      sum_splits(partial, bb, 2 * bhp + bh, H, S, bn, bkg, v);
      if (kFp16) atomicMax(&max_bits[bu][bh], __float_as_uint(max_abs8(v)));
    }
    if (kFp16) kf::named_bar_sync(kBuildBar, kBuildThreads);
    auto scale_of = [&](int bu_, int h) {
      return kFp16 ? operand_scale(__uint_as_float(max_bits[bu_][h]), true) : 1.f;
    };
    if (has_task) store_b_chunk<T>(btiles + (bu * 2 + bh) * kBImageBytes, bn, bkg, v, scale_of(bu, bh));
    kf::fence_proxy_async_smem();  // the tensor cores read B through the async proxy
    kf::named_bar_sync(kBuildBar, kBuildThreads);
    if (warp == kBWarp && lane == 0)
      for (int u = 0; u < n_first; ++u) {
        eps_s[u][0] = eps * scale_of(u, 0);
        eps_s[u][1] = eps * scale_of(u, 1);
        kf::mbar_arrive(&b_ready[u]);
      }

    if (warp == kBWarp) {
      // ---- B tiles of later head pairs (only ranges crossing more than two head pairs) ----
      for (int u = 2; u < n_units; ++u) {
        // Buffer u & 1 was last used by head pair u - 2: every worker must be past it.
        if (!__all_sync(0xffffffffu, kf::mbar_wait_or_abort(&unit_done[u & 1], ((u >> 1) - 1) & 1,
                                                            &g_sana_error, &abort_flag)))
          break;
        const int unit = first_unit + u;
        const int b = unit / head_pairs, hp = unit % head_pairs;
        float mx0 = 0.f, mx1 = 0.f;
        if (kFp16) {  // first pass: the scale
          for (int tk = lane; tk < kTasks; tk += 32) {
            float w[8];
            sum_splits(partial, b, 2 * hp + tk / (kRows * 4), H, S, (tk / 4) % kRows, tk % 4, w);
            if (tk < kRows * 4) mx0 = fmaxf(mx0, max_abs8(w)); else mx1 = fmaxf(mx1, max_abs8(w));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
          }
        }
        const float sc0 = kFp16 ? operand_scale(mx0, true) : 1.f, sc1 = kFp16 ? operand_scale(mx1, true) : 1.f;
        for (int tk = lane; tk < kTasks; tk += 32) {
          const int h = tk / (kRows * 4);
          float w[8];
          sum_splits(partial, b, 2 * hp + h, H, S, (tk / 4) % kRows, tk % 4, w);
          store_b_chunk<T>(btiles + ((u & 1) * 2 + h) * kBImageBytes, (tk / 4) % kRows, tk % 4, w, h ? sc1 : sc0);
        }
        kf::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          eps_s[u & 1][0] = eps * sc0;
          eps_s[u & 1][1] = eps * sc1;
          kf::mbar_arrive(&b_ready[u & 1]);
        }
        __syncwarp();
      }
    } else {
      // ---- workers ----
      const int g = warp >> 3, hd = (warp >> 2) & 1, quarter = warp & 3;
      const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
      const int r = quarter * 32 + lane;  // token within the tile
      const int n_g = (n_items - g + 1) / 2;
      uint8_t* stage_out = smem + Cfg::kOutOff + warp * Cfg::kWarpOutBytes;
      // relu(Q) of local item i (item 2 i + g), this warp's tokens and head, into A buffer i & 1;
      // then tell the MMA warp (this warp has also finished reading D of local item i - 2).
      auto prep = [&](int i) -> bool {
        const int k = 2 * i + g;
        const int st = k % kStages;
        const bool got = kf::mbar_wait_or_abort(&q_full[st], (k / kStages) & 1, &g_sana_error, &abort_flag);
        if (!__all_sync(0xffffffffu, got)) return false;  // warp-uniform: the tcgen05 copy is .sync.aligned
        const uint8_t* row = smem + Cfg::kQOff + st * kQTileBytes + r * 128;
        float rq = 0.f;
        int head = 0;
        if constexpr (kNorm) {  // this thread's token: r of its q row; the head's q_norm weights
          const int it = first + k;
          const int unit = it / tiles_out;
          head = 2 * (unit % head_pairs) + hd;
          rq = stats_at(nrm, unit / head_pairs, (it % tiles_out) * kOutTok + r, 0);
        }
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 x = *reinterpret_cast<const uint4*>(row + (((hd * 4 + j) ^ (r & 7)) << 4));
          if constexpr (kNorm) {
            // channels 8 j .. 8 j + 7 of the head (a head past H is all zero: weights unread)
            const uint4 wv = head < H ? __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(nrm.wq) + head * kD) + j)
                                      : make_uint4(0, 0, 0, 0);
            x.x = qk_apply2<T>(x.x, rq, rq, wv.x);
            x.y = qk_apply2<T>(x.y, rq, rq, wv.y);
            x.z = qk_apply2<T>(x.z, rq, rq, wv.z);
            x.w = qk_apply2<T>(x.w, rq, rq, wv.w);
          }
          w[4 * j + 0] = kf::Mma<T>::relu2(x.x);
          w[4 * j + 1] = kf::Mma<T>::relu2(x.y);
          w[4 * j + 2] = kf::Mma<T>::relu2(x.z);
          w[4 * j + 3] = kf::Mma<T>::relu2(x.w);
        }
        kf::tc::st_32x32b_x16(tmem + lanes + tm_slot(g, i & 1, hd) + 48, w);
        kf::tc::wait_st();
        kf::tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) kf::mbar_arrive(&ready[g][hd][i & 1]);
        return true;
      };
      int units_done = 0;  // head pairs this warp has announced as finished
      auto finish_units = [&](int upto) {
        for (; units_done < upto; ++units_done)
          if (lane == 0) kf::mbar_arrive(&unit_done[units_done & 1]);
      };
      bool ok = n_g > 0 && prep(0);
      if (ok && n_g > 1) ok = prep(1);
      int eps_unit = -1;
      float eps_h = 0.f;
      for (int i = 0; ok && i < n_g; ++i) {
        const int k = 2 * i + g;
        const int unit = unit_of(k), tt = (first + k) % tiles_out;
        const int b = unit / head_pairs, hp = unit % head_pairs;
        const int u = unit - first_unit;
        finish_units(u);  // every earlier head pair is done for this warp
        if (u != eps_unit) {
          // Head pairs 0 and 1 were built before the loop (named barrier); later ones by the B warp.
          if (u >= 2 && !__all_sync(0xffffffffu, kf::mbar_wait_or_abort(&b_ready[u & 1], (u >> 1) & 1,
                                                                        &g_sana_error, &abort_flag)))
            break;
          eps_unit = u;
          eps_h = u < 2 ? eps * scale_of(u, hd) : eps_s[u & 1][hd];
        }
        if (!__all_sync(0xffffffffu, kf::mbar_wait_or_abort<false, true>(&d_full[g][hd][i & 1], (i >> 1) & 1,
                                                                          &g_sana_error, &abort_flag)))
          break;
        kf::tc::fence_after_sync();
        uint32_t num[32], den[2];
        kf::tc::ld_32x32b_x32(tmem + lanes + tm_slot(g, i & 1, hd), num);
        kf::tc::ld_32x32b_x2(tmem + lanes + tm_slot(g, i & 1, hd) + kD, den);
        kf::tc::wait_ld();
        const float inv = __frcp_rn(__uint_as_float(den[0]) + eps_h);
        // Stage this warp's 32 tokens x 32 channels (rows of 64 bytes, 64-byte swizzle, for 16-bit
        // out; rows of 128 bytes, 128-byte swizzle, for fp32) once its previous store has read it.
        if (lane == 0) kf::tma_store_wait_read0();
        __syncwarp();
        if constexpr (sizeof(O) == 4) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(stage_out + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_float4(__uint_as_float(num[4 * j]) * inv, __uint_as_float(num[4 * j + 1]) * inv,
                            __uint_as_float(num[4 * j + 2]) * inv, __uint_as_float(num[4 * j + 3]) * inv);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              pk[e] = kf::Mma<O>::from_f2(__uint_as_float(num[8 * j + 2 * e]) * inv,
                                          __uint_as_float(num[8 * j + 2 * e + 1]) * inv);
            *reinterpret_cast<uint4*>(stage_out + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
        kf::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && 2 * hp + hd < H) {
          kf::tma_store_3d(&out_map, stage_out, hp * 2 * kD + hd * kD, tt * kOutTok + quarter * 32, b);
          kf::tma_store_commit();
        }
        if (i + 2 < n_g) ok = prep(i + 2);
      }
      finish_units(n_units);
      if (lane == 0) kf::tma_store_wait_read0();  // shared memory outlives the stores' reads
    }
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp0) {
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, kEpiTmemCols);
  }
}

// ------------------------------------------------------------------------------------------
// Generic path (fp32 input, any head dim dividing 128, small tensors): CUDA-core fp32.
// Split partials go to the workspace; the last CTA of a (batch, head) to arrive -- an atomic
// counter, no waiting -- sums them in split order and resets the counter for the next call.
// ------------------------------------------------------------------------------------------
constexpr int kGenThreads = 256;
constexpr int kGenTok = 32;

template <typename T, bool kNorm>
__global__ void __launch_bounds__(kGenThreads)
sana_vk_generic(const T* __restrict__ qkv, float* __restrict__ partial, float* __restrict__ final_vk,
                unsigned int* __restrict__ counters, int H, int d, int N, int tiles_per_split, const QkNorm nrm) {
  extern __shared__ float gsm[];
  const int nelem = (d + 1) * d;
  float* acc = gsm;
  float* kt = acc + nelem;
  float* vt = kt + kGenTok * d;
  __shared__ int s_last;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x;
  const int64_t C = static_cast<int64_t>(H) * d;
  for (int e = threadIdx.x; e < nelem; e += kGenThreads) acc[e] = 0.f;
  const int tok0 = split * tiles_per_split * kTok;
  const int tok1 = min(N, tok0 + tiles_per_split * kTok);
  for (int t0 = tok0; t0 < tok1; t0 += kGenTok) {
    __syncthreads();
    for (int e = threadIdx.x; e < kGenTok * d; e += kGenThreads) {
      const int tt = e / d, c = e % d, tok = t0 + tt;
      float kv = 0.f, vv = 0.f;
      if (tok < tok1) {
        const T* row = qkv + (static_cast<int64_t>(b) * N + tok) * 3 * C + static_cast<int64_t>(h) * d + c;
        kv = kf::Elem<T>::to_f(row[C]);
        if constexpr (kNorm) kv = qk_apply1<T>(kv, stats_at(nrm, b, tok, 1), weight_at<T>(nrm.wk, h * d + c));
        kv = fmaxf(kv, 0.f);
        vv = kf::Elem<T>::to_f(row[2 * C]);
      }
      kt[e] = kv;
      vt[e] = vv;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nelem; e += kGenThreads) {
      const int r = e / d, c = e % d;
      float a = acc[e];
      for (int tt = 0; tt < kGenTok; ++tt) a = fmaf(r < d ? vt[tt * d + r] : 1.f, kt[tt * d + c], a);
      acc[e] = a;
    }
  }
  __syncthreads();
  float* dst = partial + ((static_cast<size_t>(b) * H + h) * S + split) * nelem;
  for (int e = threadIdx.x; e < nelem; e += kGenThreads) __stcg(dst + e, acc[e]);
  __threadfence();
  __syncthreads();
  unsigned int* counter = counters + static_cast<size_t>(b) * H + h;
  if (threadIdx.x == 0) s_last = (atomicAdd(counter, 1u) == static_cast<unsigned int>(S - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* src = partial + (static_cast<size_t>(b) * H + h) * S * nelem;
  float* out = final_vk + (static_cast<size_t>(b) * H + h) * nelem;
  for (int e = threadIdx.x; e < nelem; e += kGenThreads) {
    float sum = 0.f;
    for (int s = 0; s < S; ++s) sum += __ldcg(src + static_cast<size_t>(s) * nelem + e);
    out[e] = sum;
  }
  if (threadIdx.x == 0) *counter = 0u;
}

template <typename T, typename O, bool kNorm>
__global__ void __launch_bounds__(kGenThreads)
sana_out_generic(const T* __restrict__ qkv, const float* __restrict__ final_vk, O* __restrict__ out,
                 int H, int d, int N, float eps, const QkNorm nrm) {
  extern __shared__ float gsm[];
  const int nelem = (d + 1) * d;
  float* vk = gsm;
  float* qt = vk + nelem;
  float* inv_den = qt + kGenTok * d;
  const int t0 = blockIdx.x * kGenTok, h = blockIdx.y, b = blockIdx.z;
  const int64_t C = static_cast<int64_t>(H) * d;
  const float* src = final_vk + (static_cast<size_t>(b) * H + h) * nelem;
  for (int e = threadIdx.x; e < nelem; e += kGenThreads) vk[e] = __ldcg(src + e);
  for (int e = threadIdx.x; e < kGenTok * d; e += kGenThreads) {
    const int tt = e / d, c = e % d, tok = t0 + tt;
    float qv = 0.f;
    if (tok < N) {
      qv = kf::Elem<T>::to_f(qkv[(static_cast<int64_t>(b) * N + tok) * 3 * C + static_cast<int64_t>(h) * d + c]);
      if constexpr (kNorm) qv = qk_apply1<T>(qv, stats_at(nrm, b, tok, 0), weight_at<T>(nrm.wq, h * d + c));
      qv = fmaxf(qv, 0.f);
    }
    qt[e] = qv;
  }
  __syncthreads();
  if (threadIdx.x < kGenTok) {
    float s = 0.f;
    for (int c = 0; c < d; ++c) s = fmaf(vk[d * d + c], qt[threadIdx.x * d + c], s);
    inv_den[threadIdx.x] = __frcp_rn(s + eps);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kGenTok * d; e += kGenThreads) {
    const int tt = e / d, r = e % d, tok = t0 + tt;
    if (tok >= N) continue;
    float num = 0.f;
    for (int c = 0; c < d; ++c) num = fmaf(vk[r * d + c], qt[tt * d + c], num);
    out[(static_cast<int64_t>(b) * N + tok) * C + static_cast<int64_t>(h) * d + r] =
        kf::Elem<O>::from_f(num * inv_den[tt]);
  }
}

// ------------------------------------------------------------------------------------------
// Fused path: one launch, one (batch, head) unit per CTA (or per cluster) at a time, no workspace.
//
// When the batch x head units fill the SMs (or when the caller asks for it with splits = -1),
// every CTA owns whole heads, so the K^T V reduction never leaves the CTA and no second launch
// waits for it. Per unit, one TMA producer warp streams through a 16-stage ring of 8 KB stages
//   phase 1: K and V boxes of 64 tokens x 32 channels (64-byte rows, 64-byte swizzle);
//   phase 2: Q boxes of 128 tokens x 32 channels;
// and 16 compute warps consume them in turn: stage number x of the CTA's whole sequence goes to
// warp x mod 16, so the warp that waits for a ring slot's next fill is the one that released its
// previous fill (that keeps every parity wait within one phase of the barrier):
//   phase 1: VK += V^T relu(K) and ksum += relu(K) per warp (mma.sync m16n8k16, fp32), then the
//            16 warp partials are summed in warp order in shared memory (deterministic);
//   phase 2: every warp holds B = [VK ; ksum] as hi + lo 16-bit halves in registers (so the
//            fp32 sums keep ~16 mantissa bits, as on the tcgen05 path) and, per 16 tokens,
//            D = relu(Q) B_hi + relu(Q) B_lo, out = D[:, :32] / (D[:, 32] + eps), staged in
//            shared memory and written with a TMA store.
// The producer runs ahead into the next unit, so the next K/V tiles and the first Q tiles are
// in flight while the warps reduce. fp16 inputs scale B by a power of two that keeps max|B|
// below 2^14, with eps scaled alike.
//
// Cluster form (sana_head_cluster): when there are fewer units than SMs, a cluster of CS CTAs
// shares one unit. CTA rank r takes the r-th of CS equal ranges of K/V tiles and of Q tiles and
// sums its warp partials, and the CTAs combine them by pushing over distributed shared memory
// (st.async, whose bytes complete on the receiving CTA's own mbarrier, so no cluster-scope
// fence or remote read is on the path): rank r owns the r-th of CS chunks of [VK ; ksum].
//   round 1 (reduce-scatter): every CTA pushes each chunk into its owner's receive slot;
//   round 2 (all-gather): the owner sums its chunk over the ranks in rank order into `tot` and
//            pushes the sums into every peer's `tot`.
// Every CTA thus holds the same bits, whatever the timing. For a later unit a CTA pushes only
// after every peer has signalled `xdone` (re-armed its rounds and finished with its `tot` and
// receive slots); the last unit sends no signal, so nothing reaches a CTA that has exited.
// All of these waits are bounded like the ring's. It is its own kernel: one template for both
// forms measured 2% slower on the one-CTA form (B=2, H=70, N=16384), with identical source for
// that form.
// ------------------------------------------------------------------------------------------
constexpr int kFusedWarps = 16;                          // compute warps
constexpr int kFusedThreads = 32 * (kFusedWarps + 1);    // + the TMA producer warp
constexpr int kFusedStages = 16;
constexpr int kFusedStageBytes = 8192;                   // K + V boxes (64 tokens), or a Q box (128 tokens)
constexpr int kFusedKTok = 64;
constexpr int kFusedQTok = 128;
constexpr int kFusedSub = 16;                            // tokens per output store
constexpr int kFusedPartBytes = kRows * kD * 4;          // one warp's [VK ; ksum] partial, fp32
constexpr int kFusedSlotBytes = 5 * 1024;                // per-warp slot, 1024-byte aligned
constexpr uint32_t kFusedBar = 2;                        // named barrier of the compute warps
struct FusedSmem {
  static constexpr int kRingOff = 0;
  // Warp w's slot: its phase-1 partial, then (reused) its phase-2 output staging, two 16-token
  // buffers at 1024-byte aligned offsets (the swizzled TMA store tiles need that alignment).
  static constexpr int kPartOff = kFusedStages * kFusedStageBytes;
  static constexpr int kRedOff = kPartOff + kFusedWarps * kFusedSlotBytes;  // reduced [VK ; ksum]
  static constexpr int kBarOff = kRedOff + kFusedPartBytes + 16;            // + two max|B| words
  static constexpr int kBytes = kBarOff + 2 * kFusedStages * 8 + 16 + 1024;
};
// Cluster form: the same up to `red` (this CTA's [VK ; ksum]), then the cluster sum `tot`, the
// receive area of the reduce-scatter (per sending rank, its slice of this CTA's chunk), and three
// more mbarriers (xready1, xready2, xdone) after the abort word.
constexpr int kXVec = kFusedPartBytes / 16;  // 16-byte vectors of one [VK ; ksum]
struct ClusterSmem {
  static constexpr int kRingOff = FusedSmem::kRingOff;
  static constexpr int kPartOff = FusedSmem::kPartOff;
  static constexpr int kRedOff = FusedSmem::kRedOff;
  static constexpr int kTotOff = kRedOff + kFusedPartBytes;
  static constexpr int kRecvOff = kTotOff + kFusedPartBytes;
  static constexpr int kRecvBytes = 4352;                     // >= cs * ceil(kXVec / cs) * 16, cs <= 8
  static constexpr int kMaxOff = kRecvOff + kRecvBytes;       // two max|B| words
  static constexpr int kBarOff = kMaxOff + 16;
  static constexpr int kBytes = kBarOff + 2 * kFusedStages * 8 + 16 + 24 + 1024;
};
static_assert(ClusterSmem::kRedOff % 16 == 0 && ClusterSmem::kTotOff % 16 == 0 && ClusterSmem::kRecvOff % 16 == 0 &&
                  kFusedPartBytes % 16 == 0,
              "the cluster exchange moves 16-byte vectors");
constexpr int recv_bytes_needed(int cs) { return cs * ((kXVec + cs - 1) / cs) * 16; }
static_assert(recv_bytes_needed(2) <= ClusterSmem::kRecvBytes && recv_bytes_needed(3) <= ClusterSmem::kRecvBytes &&
                  recv_bytes_needed(4) <= ClusterSmem::kRecvBytes && recv_bytes_needed(5) <= ClusterSmem::kRecvBytes &&
                  recv_bytes_needed(6) <= ClusterSmem::kRecvBytes && recv_bytes_needed(7) <= ClusterSmem::kRecvBytes &&
                  recv_bytes_needed(8) <= ClusterSmem::kRecvBytes && kXVec <= 32 * kFusedWarps,
              "receive slots of the reduce-scatter; one vector per compute thread");
constexpr int kFusedMaxCluster = 8;  // portable cluster size limit
static_assert(kFusedPartBytes <= kFusedSlotBytes && 2 * 2048 <= kFusedSlotBytes, "slot sizes");
// Ring slot x % kFusedStages is consumed by warp x % kFusedWarps: with equal counts the warp that
// waits for a slot's next fill is the one that released the previous fill, so no parity wait on
// `full` can see a phase two fills old and no extra arrival can reach `empty`.
static_assert(kFusedStages == kFusedWarps, "ring depth must equal the number of compute warps");

// Index of element (r, c) of a [VK ; ksum] partial or sum in shared memory (33 rows of 32 fp32).
// The warp partials are written, and the B fragments read, as float2 pairs by 8 rows x 4
// column pairs per instruction; with plain 128-byte rows those 8 rows share banks (8-way
// conflicts). XOR-ing column bits 3-4 with row bits 0-1 spreads them over all banks (two
// wavefronts per instruction). The sums over partials and across a cluster are elementwise, so
// they do not depend on the layout.
__device__ __forceinline__ int part_idx(int r, int c) { return r * kD + (c ^ ((r & 3) << 3)); }

// Byte offset of 16-byte chunk c of row r in a tile of 64-byte rows written with 64-byte swizzle.
__device__ __forceinline__ uint32_t swz64(uint32_t row, uint32_t chunk) {
  return row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4);
}

template <typename T, typename O, bool kNorm>
__global__ void __launch_bounds__(kFusedThreads, 1)
sana_head_fused(const __grid_constant__ CUtensorMap kv_map, const __grid_constant__ CUtensorMap q_map,
                const __grid_constant__ CUtensorMap out_map, int B, int H, int N, float eps,
                const QkNorm nrm) {
  constexpr bool kFp16 = std::is_same<T, __half>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + FusedSmem::kBarOff);
  uint64_t* empty = full + kFusedStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kFusedStages);
  float* red = reinterpret_cast<float*>(smem + FusedSmem::kRedOff);
  unsigned int* max_bits = reinterpret_cast<unsigned int*>(red + kRows * kD);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3, sub = lane >> 3;
  const int units = B * H;
  const int kv_tiles = (N + kFusedKTok - 1) / kFusedKTok;
  const int q_tiles = (N + kFusedQTok - 1) / kFusedQTok;
  const int per_unit = kv_tiles + q_tiles;  // ring stages per unit

  if (threadIdx.x == 0) {
    kf::prefetch_tensormap(&kv_map);
    kf::prefetch_tensormap(&q_map);
    kf::prefetch_tensormap(&out_map);
    for (int s = 0; s < kFusedStages; ++s) {
      kf::mbar_init(&full[s], 1);
      kf::mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    max_bits[0] = max_bits[1] = 0u;
    kf::fence_mbar_init();
  }
  __syncthreads();

  if (warp == kFusedWarps) {
    // ---- TMA producer (one thread): every unit's K/V tiles, then its Q tiles ----
    if (lane == 0) {
      int seq = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int b = u / H, h = u % H;
        for (int i = 0; i < per_unit; ++i, ++seq) {
          const int st = seq % kFusedStages;
          if (seq >= kFusedStages &&
              !kf::mbar_wait_or_abort<true>(&empty[st], ((seq / kFusedStages) - 1) & 1, &g_sana_error, abort_flag))
            return;
          uint8_t* base = smem + FusedSmem::kRingOff + st * kFusedStageBytes;
          kf::mbar_arrive_expect_tx(&full[st], kFusedStageBytes);
          if (i < kv_tiles) {
            kf::tma_load_4d(base, &kv_map, &full[st], h * kD, 1, i * kFusedKTok, b);
            kf::tma_load_4d(base + kFusedStageBytes / 2, &kv_map, &full[st], h * kD, 2, i * kFusedKTok, b);
          } else {
            kf::tma_load_4d(base, &q_map, &full[st], h * kD, 0, (i - kv_tiles) * kFusedQTok, b);
          }
        }
      }
    }
    return;
  }

  // ---- compute warps ----
  uint8_t* part = smem + FusedSmem::kPartOff + warp * kFusedSlotBytes;  // this warp's slot
  int seq0 = 0;  // ring sequence number of the unit's first stage
  bool ok = true;
  int parity = 0;  // max|B| word of this unit (two words: one is reset while the other is in use)
  for (int u = blockIdx.x; u < units; u += gridDim.x, seq0 += per_unit, parity ^= 1) {
    const int b = u / H, h = u % H;
    // Phase 1: this warp's K/V tiles.
    float acc[2][4][4];
    float ksum[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.f;
    }
    for (int i = (warp - seq0 % kFusedWarps + kFusedWarps) % kFusedWarps; i < kv_tiles; i += kFusedWarps) {
      const int seq = seq0 + i, st = seq % kFusedStages;
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&full[st], (seq / kFusedStages) & 1,
                                                                  &g_sana_error, abort_flag));
      if (!ok) break;
      const uint32_t kbase = kf::smem_u32(smem + FusedSmem::kRingOff + st * kFusedStageBytes);
      const uint32_t vbase = kbase + kFusedStageBytes / 2;
#pragma unroll
      for (int ks = 0; ks < kFusedKTok / 16; ++ks) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          // A = V^T (M = v channel, K = token): transposed 8x8 loads of token-major rows.
          const int row = ks * 16 + (lane & 7) + (sub >> 1) * 8;
          kf::ldsm_x4_t(vbase + swz64(row, mt * 2 + (sub & 1)), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
        }
        uint32_t bf[4][2];
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          // B = relu(K) (K = token, N = k channel), two n-tiles per x4 load.
          const int row = ks * 16 + (lane & 7) + (sub & 1) * 8;
          kf::ldsm_x4_t(kbase + swz64(row, np * 2 + (sub >> 1)), bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0],
                        bf[2 * np + 1][1]);
        }
        if constexpr (kNorm) qk_norm_k<T>(bf, nrm, b, i * kFusedKTok + ks * 16, lane, h);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          bf[nt][0] = kf::Mma<T>::relu2(bf[nt][0]);
          bf[nt][1] = kf::Mma<T>::relu2(bf[nt][1]);
          const float2 x = kf::Mma<T>::to_f2(bf[nt][0]);
          const float2 y = kf::Mma<T>::to_f2(bf[nt][1]);
          ksum[nt] += (x.x + x.y) + (y.x + y.y);
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) kf::Mma<T>::run(acc[mt][nt], a[mt], bf[nt]);
      }
      __syncwarp();
      if (lane == 0) kf::mbar_arrive(&empty[st]);
    }
    // This warp's partial [VK ; ksum] into its slot (its previous output stores must have read it).
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 1);
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 2);
    }
    if (lane == 0) kf::tma_store_wait_read0();
    __syncwarp();
    float* pw = reinterpret_cast<float*>(part);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int r = mt * 16 + gid, c = nt * 8 + tig * 2;
        *reinterpret_cast<float2*>(pw + part_idx(r, c)) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
        *reinterpret_cast<float2*>(pw + part_idx(r + 8, c)) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
      }
    if (tig == 0) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) pw[part_idx(kD, nt * 8 + gid)] = ksum[nt];
    }
    kf::named_bar_sync(kFusedBar, 32 * kFusedWarps);
    // Every compute thread is past the previous unit's read of the other word.
    if (threadIdx.x == 0) max_bits[parity ^ 1] = 0u;
    // Sum of the 16 partials in warp order, and max|B| for the fp16 scale.
    float m = 0.f;
    for (int e = threadIdx.x; e < kRows * kD; e += 32 * kFusedWarps) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kFusedWarps; ++w)
        s += reinterpret_cast<const float*>(smem + FusedSmem::kPartOff + w * kFusedSlotBytes)[e];
      red[e] = s;
      m = fmaxf(m, fabsf(s));
    }
    if (kFp16) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) atomicMax(&max_bits[parity], __float_as_uint(m));  // non-negative floats order as integers
    }
    kf::named_bar_sync(kFusedBar, 32 * kFusedWarps);
    const float scale = operand_scale(__uint_as_float(max_bits[parity]), kFp16);
    const float eps_s = eps * scale;
    // B fragments (K = q channel c, N = output row r: VK[r][c], r = 32 is ksum[c], rows 33..39 zero)
    // as hi and lo halves.
    uint32_t bhi[2][5][2], blo[2][5][2];
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
      for (int nt = 0; nt < 5; ++nt) {
        const int r = nt * 8 + gid;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int c = ks * 16 + tig * 2 + half * 8;
          float x0 = 0.f, x1 = 0.f;
          if (r <= kD) {
            const float2 x = *reinterpret_cast<const float2*>(red + part_idx(r, c));  // c even
            x0 = x.x * scale;
            x1 = x.y * scale;
          }
          bhi[ks][nt][half] = kf::Mma<T>::from_f2(x0, x1);
          const float2 hf = kf::Mma<T>::to_f2(bhi[ks][nt][half]);
          blo[ks][nt][half] = kf::Mma<T>::from_f2(x0 - hf.x, x1 - hf.y);
        }
      }
    // Phase 2: this warp's Q tiles, 16 tokens at a time.
    int nstore = 0;
    for (int j = (warp - (seq0 + kv_tiles) % kFusedWarps + kFusedWarps) % kFusedWarps; j < q_tiles;
         j += kFusedWarps) {
      const int seq = seq0 + kv_tiles + j, st = seq % kFusedStages;
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&full[st], (seq / kFusedStages) & 1,
                                                                  &g_sana_error, abort_flag));
      if (!ok) break;
      const uint32_t qbase = kf::smem_u32(smem + FusedSmem::kRingOff + st * kFusedStageBytes);
#pragma unroll 1
      for (int m16 = 0; m16 < kFusedQTok / kFusedSub; ++m16) {
        uint32_t a[2][4];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const int row = m16 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          kf::ldsm_x4(qbase + swz64(row, ks * 2 + (lane >> 4)), a[ks][0], a[ks][1], a[ks][2], a[ks][3]);
          if constexpr (!kNorm) {
#pragma unroll
            for (int e = 0; e < 4; ++e) a[ks][e] = kf::Mma<T>::relu2(a[ks][e]);
          }
        }
        if constexpr (kNorm) {
          qk_norm_q<T>(a, nrm, b, j * kFusedQTok + m16 * kFusedSub, lane, h);
#pragma unroll
          for (int ks = 0; ks < 2; ++ks)
#pragma unroll
            for (int e = 0; e < 4; ++e) a[ks][e] = kf::Mma<T>::relu2(a[ks][e]);
        }
        if (m16 == kFusedQTok / kFusedSub - 1) {  // the stage is no longer read
          __syncwarp();
          if (lane == 0) kf::mbar_arrive(&empty[st]);
        }
        float d[5][4];
#pragma unroll
        for (int nt = 0; nt < 5; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) d[nt][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
#pragma unroll
          for (int nt = 0; nt < 5; ++nt) {
            kf::Mma<T>::run(d[nt], a[ks], bhi[ks][nt]);
            kf::Mma<T>::run(d[nt], a[ks], blo[ks][nt]);
          }
        // Denominator D[row][32]: column 0 of n-tile 4, held by the quad's first thread.
        const float den0 = __shfl_sync(0xffffffffu, d[4][0], lane & ~3);
        const float den1 = __shfl_sync(0xffffffffu, d[4][2], lane & ~3);
        const float inv0 = __frcp_rn(den0 + eps_s), inv1 = __frcp_rn(den1 + eps_s);
        // Stage 16 tokens x 32 channels in buffer (nstore & 1) once its previous store has read it.
        uint8_t* stage = part + (nstore & 1) * (kFusedSub * kD * int(sizeof(O)));
        if (lane == 0) kf::tma_store_wait_read1();
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int c = nt * 8 + tig * 2;
          if constexpr (sizeof(O) == 4) {
            // rows of 128 bytes, 128-byte swizzle
            const uint32_t off = (c & 3) * 4;
            *reinterpret_cast<float2*>(stage + gid * 128 + (((c >> 2) ^ (gid & 7)) << 4) + off) =
                make_float2(d[nt][0] * inv0, d[nt][1] * inv0);
            *reinterpret_cast<float2*>(stage + (gid + 8) * 128 + (((c >> 2) ^ ((gid + 8) & 7)) << 4) + off) =
                make_float2(d[nt][2] * inv1, d[nt][3] * inv1);
          } else {
            // rows of 64 bytes, 64-byte swizzle
            const uint32_t off = (c & 7) * 2;
            *reinterpret_cast<uint32_t*>(stage + swz64(gid, c >> 3) + off) =
                kf::Mma<O>::from_f2(d[nt][0] * inv0, d[nt][1] * inv0);
            *reinterpret_cast<uint32_t*>(stage + swz64(gid + 8, c >> 3) + off) =
                kf::Mma<O>::from_f2(d[nt][2] * inv1, d[nt][3] * inv1);
          }
        }
        kf::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          kf::tma_store_3d(&out_map, stage, h * kD, j * kFusedQTok + m16 * kFusedSub, b);
          kf::tma_store_commit();
        }
        ++nstore;
      }
    }
  }
  if (lane == 0) kf::tma_store_wait_read0();  // shared memory outlives the stores' reads
}

template <typename T, typename O, bool kNorm>
__global__ void __launch_bounds__(kFusedThreads, 1)
sana_head_cluster(const __grid_constant__ CUtensorMap kv_map, const __grid_constant__ CUtensorMap q_map,
                const __grid_constant__ CUtensorMap out_map, int B, int H, int N, float eps,
                const QkNorm nrm) {
  constexpr bool kFp16 = std::is_same<T, __half>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ClusterSmem::kBarOff);
  uint64_t* empty = full + kFusedStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kFusedStages);
  uint64_t* xready1 = empty + kFusedStages + 2;  // past the 16-byte abort word
  uint64_t* xready2 = xready1 + 1;
  uint64_t* xdone = xready2 + 1;
  float* red = reinterpret_cast<float*>(smem + ClusterSmem::kRedOff);
  float* tot = reinterpret_cast<float*>(smem + ClusterSmem::kTotOff);
  const float4* recv = reinterpret_cast<const float4*>(smem + ClusterSmem::kRecvOff);
  unsigned int* max_bits = reinterpret_cast<unsigned int*>(smem + ClusterSmem::kMaxOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3, sub = lane >> 3;
  const int units = B * H;
  // CS CTAs per unit (one cluster); this CTA is rank `rank`.
  const int cs = static_cast<int>(kf::cluster_nctarank());
  const int rank = static_cast<int>(kf::cluster_ctarank());
  // Exchange chunks: rank r owns vectors [r c4, min(kXVec, (r + 1) c4)) of [VK ; ksum].
  const int c4 = (kXVec + cs - 1) / cs;
  const int own0 = min(kXVec, rank * c4), own1 = min(kXVec, own0 + c4);
  const uint32_t bytes1 = static_cast<uint32_t>((cs - 1) * (own1 - own0) * 16);  // reduce-scatter in
  const uint32_t bytes2 = static_cast<uint32_t>((kXVec - (own1 - own0)) * 16);    // all-gather in
  const int first_unit = static_cast<int>(kf::cluster_id_x());
  const int unit_step = static_cast<int>(kf::cluster_count_x());
  // This CTA's share of every unit: K/V tiles [kv0, kv0 + kv_tiles), Q tiles [q0, q0 + q_tiles).
  const int kv_all = (N + kFusedKTok - 1) / kFusedKTok;
  const int q_all = (N + kFusedQTok - 1) / kFusedQTok;
  const int kv_per = (kv_all + cs - 1) / cs, q_per = (q_all + cs - 1) / cs;
  const int kv0 = min(kv_all, rank * kv_per), q0 = min(q_all, rank * q_per);
  const int kv_tiles = min(kv_all, kv0 + kv_per) - kv0;
  const int q_tiles = min(q_all, q0 + q_per) - q0;
  const int per_unit = kv_tiles + q_tiles;  // ring stages per unit

  if (threadIdx.x == 0) {
    kf::prefetch_tensormap(&kv_map);
    kf::prefetch_tensormap(&q_map);
    kf::prefetch_tensormap(&out_map);
    for (int s = 0; s < kFusedStages; ++s) {
      kf::mbar_init(&full[s], 1);
      kf::mbar_init(&empty[s], 1);
    }
    // xready1 / xready2: this CTA's own arrival with the bytes its peers push in that round
    // (armed here for the first unit, re-armed before each later unit's exchange can start).
    kf::mbar_init(xready1, 1);
    kf::mbar_init(xready2, 1);
    kf::mbar_init(xdone, cs > 1 ? cs - 1 : 1);  // one arrival per peer
    *abort_flag = 0;
    max_bits[0] = max_bits[1] = 0u;
    kf::fence_mbar_init();
    if (cs > 1) {
      kf::mbar_arrive_expect_tx(xready1, bytes1);
      kf::mbar_arrive_expect_tx(xready2, bytes2);
    }
  }
  // Peers arrive on this CTA's xready / xdone, so they must be initialised cluster-wide first.
  kf::cluster_sync_all();

  if (warp == kFusedWarps) {
    // ---- TMA producer (one thread): every unit's K/V tiles, then its Q tiles ----
    if (lane == 0) {
      int seq = 0;
      for (int u = first_unit; u < units; u += unit_step) {
        const int b = u / H, h = u % H;
        for (int i = 0; i < per_unit; ++i, ++seq) {
          const int st = seq % kFusedStages;
          if (seq >= kFusedStages &&
              !kf::mbar_wait_or_abort<true>(&empty[st], ((seq / kFusedStages) - 1) & 1, &g_sana_error, abort_flag))
            return;
          uint8_t* base = smem + ClusterSmem::kRingOff + st * kFusedStageBytes;
          kf::mbar_arrive_expect_tx(&full[st], kFusedStageBytes);
          if (i < kv_tiles) {
            const int tok = (kv0 + i) * kFusedKTok;
            kf::tma_load_4d(base, &kv_map, &full[st], h * kD, 1, tok, b);
            kf::tma_load_4d(base + kFusedStageBytes / 2, &kv_map, &full[st], h * kD, 2, tok, b);
          } else {
            kf::tma_load_4d(base, &q_map, &full[st], h * kD, 0, (q0 + i - kv_tiles) * kFusedQTok, b);
          }
        }
      }
    }
    return;
  }

  // ---- compute warps ----
  uint8_t* part = smem + ClusterSmem::kPartOff + warp * kFusedSlotBytes;  // this warp's slot
  int seq0 = 0;  // ring sequence number of the unit's first stage
  bool ok = true;
  int parity = 0;  // max|B| word of this unit (two words: one is reset while the other is in use)
  int k = 0;       // units this CTA has finished (the phase of xready / xdone)
  for (int u = first_unit; u < units; u += unit_step, seq0 += per_unit, parity ^= 1, ++k) {
    const int b = u / H, h = u % H;
    // Phase 1: this warp's K/V tiles.
    float acc[2][4][4];
    float ksum[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.f;
    }
    for (int i = (warp - seq0 % kFusedWarps + kFusedWarps) % kFusedWarps; i < kv_tiles; i += kFusedWarps) {
      const int seq = seq0 + i, st = seq % kFusedStages;
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&full[st], (seq / kFusedStages) & 1,
                                                                  &g_sana_error, abort_flag));
      if (!ok) break;
      const uint32_t kbase = kf::smem_u32(smem + ClusterSmem::kRingOff + st * kFusedStageBytes);
      const uint32_t vbase = kbase + kFusedStageBytes / 2;
#pragma unroll
      for (int ks = 0; ks < kFusedKTok / 16; ++ks) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          // A = V^T (M = v channel, K = token): transposed 8x8 loads of token-major rows.
          const int row = ks * 16 + (lane & 7) + (sub >> 1) * 8;
          kf::ldsm_x4_t(vbase + swz64(row, mt * 2 + (sub & 1)), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
        }
        uint32_t bf[4][2];
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          // B = relu(K) (K = token, N = k channel), two n-tiles per x4 load.
          const int row = ks * 16 + (lane & 7) + (sub & 1) * 8;
          kf::ldsm_x4_t(kbase + swz64(row, np * 2 + (sub >> 1)), bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0],
                        bf[2 * np + 1][1]);
        }
        if constexpr (kNorm) qk_norm_k<T>(bf, nrm, b, (kv0 + i) * kFusedKTok + ks * 16, lane, h);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          bf[nt][0] = kf::Mma<T>::relu2(bf[nt][0]);
          bf[nt][1] = kf::Mma<T>::relu2(bf[nt][1]);
          const float2 x = kf::Mma<T>::to_f2(bf[nt][0]);
          const float2 y = kf::Mma<T>::to_f2(bf[nt][1]);
          ksum[nt] += (x.x + x.y) + (y.x + y.y);
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) kf::Mma<T>::run(acc[mt][nt], a[mt], bf[nt]);
      }
      __syncwarp();
      if (lane == 0) kf::mbar_arrive(&empty[st]);
    }
    // This warp's partial [VK ; ksum] into its slot (its previous output stores must have read it).
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 1);
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 2);
    }
    if (lane == 0) kf::tma_store_wait_read0();
    __syncwarp();
    float* pw = reinterpret_cast<float*>(part);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int r = mt * 16 + gid, c = nt * 8 + tig * 2;
        *reinterpret_cast<float2*>(pw + part_idx(r, c)) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
        *reinterpret_cast<float2*>(pw + part_idx(r + 8, c)) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
      }
    if (tig == 0) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) pw[part_idx(kD, nt * 8 + gid)] = ksum[nt];
    }
    kf::named_bar_sync(kFusedBar, 32 * kFusedWarps);
    // Every compute thread is past the previous unit's read of the other word.
    if (threadIdx.x == 0) max_bits[parity ^ 1] = 0u;
    const bool exchange = cs > 1;
    if (exchange && k > 0) {
      // Every thread has also finished the previous unit's `tot` and receive area: re-arm both
      // rounds for this unit, then tell the peers that they may push into them.
      if (threadIdx.x == 0) {
        kf::mbar_arrive_expect_tx(xready1, bytes1);
        kf::mbar_arrive_expect_tx(xready2, bytes2);
        for (int r = 0; r < cs; ++r)
          if (r != rank) kf::mbar_arrive_cluster_relaxed(kf::cluster_map(kf::smem_u32(xdone), r));
      }
      // ... and wait until every peer is done with its own (this CTA pushes into them below).
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(xdone, (k - 1) & 1, &g_sana_error, abort_flag));
    }
    // Sum of the 16 partials in warp order, one 16-byte vector per thread, and max|B| for the
    // fp16 scale.
    float m = 0.f;
    const int e4 = threadIdx.x;
    float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e4 < kXVec) {
#pragma unroll
      for (int w = 0; w < kFusedWarps; ++w) {
        const float4 v = reinterpret_cast<const float4*>(smem + ClusterSmem::kPartOff + w * kFusedSlotBytes)[e4];
        s4.x += v.x;
        s4.y += v.y;
        s4.z += v.z;
        s4.w += v.w;
      }
    }
    if (!exchange) {
      if (e4 < kXVec) {
        reinterpret_cast<float4*>(red)[e4] = s4;
        m = fmaxf(fmaxf(fabsf(s4.x), fabsf(s4.y)), fmaxf(fabsf(s4.z), fabsf(s4.w)));
      }
    } else {
      // Round 1 (reduce-scatter): each vector goes to the rank that owns it, into the slot of this
      // rank. No fence: the bytes complete on the owner's own mbarrier, which its threads wait on.
      const int owner = e4 / c4;
      if (e4 < kXVec && owner != rank)
        kf::st_async_f4(kf::cluster_map(kf::smem_u32(smem + ClusterSmem::kRecvOff) + (rank * c4 + e4 - owner * c4) * 16,
                                        owner),
                        s4, kf::cluster_map(kf::smem_u32(xready1), owner));
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(xready1, k & 1, &g_sana_error, abort_flag));
      // This rank's chunk summed over the ranks in rank order (the same additions in every CTA of
      // the cluster), then round 2 (all-gather): the sums go into every peer's `tot`.
      if (ok && e4 >= own0 && e4 < own1) {
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < cs; ++r) {
          const float4 v = r == rank ? s4 : recv[r * c4 + e4 - own0];
          if (r == 0) {
            t = v;
          } else {
            t.x += v.x;
            t.y += v.y;
            t.z += v.z;
            t.w += v.w;
          }
        }
        reinterpret_cast<float4*>(tot)[e4] = t;
        for (int r = 0; r < cs; ++r)
          if (r != rank)
            kf::st_async_f4(kf::cluster_map(kf::smem_u32(tot) + e4 * 16, r), t, kf::cluster_map(kf::smem_u32(xready2), r));
      }
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(xready2, k & 1, &g_sana_error, abort_flag));
      kf::named_bar_sync(kFusedBar, 32 * kFusedWarps);  // this CTA's own chunk of `tot` is written
      if (e4 < kXVec) {
        const float4 t = reinterpret_cast<const float4*>(tot)[e4];
        m = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
      }
    }
    if (kFp16) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) atomicMax(&max_bits[parity], __float_as_uint(m));  // non-negative floats order as integers
    }
    kf::named_bar_sync(kFusedBar, 32 * kFusedWarps);
    const float* vk = exchange ? tot : red;
    const float scale = operand_scale(__uint_as_float(max_bits[parity]), kFp16);
    const float eps_s = eps * scale;
    // B fragments (K = q channel c, N = output row r: VK[r][c], r = 32 is ksum[c], rows 33..39 zero)
    // as hi and lo halves.
    uint32_t bhi[2][5][2], blo[2][5][2];
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
      for (int nt = 0; nt < 5; ++nt) {
        const int r = nt * 8 + gid;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int c = ks * 16 + tig * 2 + half * 8;
          float x0 = 0.f, x1 = 0.f;
          if (r <= kD) {
            const float2 x = *reinterpret_cast<const float2*>(vk + part_idx(r, c));  // c even
            x0 = x.x * scale;
            x1 = x.y * scale;
          }
          bhi[ks][nt][half] = kf::Mma<T>::from_f2(x0, x1);
          const float2 hf = kf::Mma<T>::to_f2(bhi[ks][nt][half]);
          blo[ks][nt][half] = kf::Mma<T>::from_f2(x0 - hf.x, x1 - hf.y);
        }
      }
    // Phase 2: this warp's Q tiles, 16 tokens at a time.
    int nstore = 0;
    for (int j = (warp - (seq0 + kv_tiles) % kFusedWarps + kFusedWarps) % kFusedWarps; j < q_tiles;
         j += kFusedWarps) {
      const int seq = seq0 + kv_tiles + j, st = seq % kFusedStages;
      if (ok) ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&full[st], (seq / kFusedStages) & 1,
                                                                  &g_sana_error, abort_flag));
      if (!ok) break;
      const uint32_t qbase = kf::smem_u32(smem + ClusterSmem::kRingOff + st * kFusedStageBytes);
      // Tokens tok0 .. tok0 + 127, of which n_sub blocks of 16 reach into the sequence (>= 1).
      const int tok0 = (q0 + j) * kFusedQTok;
      const int n_sub = min(kFusedQTok / kFusedSub, (N - tok0 + kFusedSub - 1) / kFusedSub);
#pragma unroll 1
      for (int m16 = 0; m16 < n_sub; ++m16) {
        uint32_t a[2][4];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const int row = m16 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          kf::ldsm_x4(qbase + swz64(row, ks * 2 + (lane >> 4)), a[ks][0], a[ks][1], a[ks][2], a[ks][3]);
          if constexpr (!kNorm) {
#pragma unroll
            for (int e = 0; e < 4; ++e) a[ks][e] = kf::Mma<T>::relu2(a[ks][e]);
          }
        }
        if constexpr (kNorm) {
          qk_norm_q<T>(a, nrm, b, tok0 + m16 * kFusedSub, lane, h);
#pragma unroll
          for (int ks = 0; ks < 2; ++ks)
#pragma unroll
            for (int e = 0; e < 4; ++e) a[ks][e] = kf::Mma<T>::relu2(a[ks][e]);
        }
        if (m16 == n_sub - 1) {  // the stage is no longer read
          __syncwarp();
          if (lane == 0) kf::mbar_arrive(&empty[st]);
        }
        float d[5][4];
#pragma unroll
        for (int nt = 0; nt < 5; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) d[nt][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
#pragma unroll
          for (int nt = 0; nt < 5; ++nt) {
            kf::Mma<T>::run(d[nt], a[ks], bhi[ks][nt]);
            kf::Mma<T>::run(d[nt], a[ks], blo[ks][nt]);
          }
        // Denominator D[row][32]: column 0 of n-tile 4, held by the quad's first thread.
        const float den0 = __shfl_sync(0xffffffffu, d[4][0], lane & ~3);
        const float den1 = __shfl_sync(0xffffffffu, d[4][2], lane & ~3);
        const float inv0 = __frcp_rn(den0 + eps_s), inv1 = __frcp_rn(den1 + eps_s);
        // Stage 16 tokens x 32 channels in buffer (nstore & 1) once its previous store has read it.
        uint8_t* stage = part + (nstore & 1) * (kFusedSub * kD * int(sizeof(O)));
        if (lane == 0) kf::tma_store_wait_read1();
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int c = nt * 8 + tig * 2;
          if constexpr (sizeof(O) == 4) {
            // rows of 128 bytes, 128-byte swizzle
            const uint32_t off = (c & 3) * 4;
            *reinterpret_cast<float2*>(stage + gid * 128 + (((c >> 2) ^ (gid & 7)) << 4) + off) =
                make_float2(d[nt][0] * inv0, d[nt][1] * inv0);
            *reinterpret_cast<float2*>(stage + (gid + 8) * 128 + (((c >> 2) ^ ((gid + 8) & 7)) << 4) + off) =
                make_float2(d[nt][2] * inv1, d[nt][3] * inv1);
          } else {
            // rows of 64 bytes, 64-byte swizzle
            const uint32_t off = (c & 7) * 2;
            *reinterpret_cast<uint32_t*>(stage + swz64(gid, c >> 3) + off) =
                kf::Mma<O>::from_f2(d[nt][0] * inv0, d[nt][1] * inv0);
            *reinterpret_cast<uint32_t*>(stage + swz64(gid + 8, c >> 3) + off) =
                kf::Mma<O>::from_f2(d[nt][2] * inv1, d[nt][3] * inv1);
          }
        }
        kf::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          kf::tma_store_3d(&out_map, stage, h * kD, tok0 + m16 * kFusedSub, b);
          kf::tma_store_commit();
        }
        ++nstore;
      }
    }
  }
  if (lane == 0) kf::tma_store_wait_read0();  // shared memory outlives the stores' reads
  // Cluster form: no peer reads this CTA's shared memory, and every peer push into it has
  // completed (this CTA waited for all bytes of each unit); the last unit sends no `xdone`.
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
constexpr int kFastStages = 3;

// Most clusters of `cs` fused CTAs resident at once on the current device (0: that size does
// not launch). Cached per device; every instantiation has the same shape (threads, shared
// memory, one CTA per SM), so one of them answers for all.
int fused_max_clusters(int cs) {
  static int cache[64][kFusedMaxCluster + 1] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  if (dev < 0 || dev >= 64 || cs < 1 || cs > kFusedMaxCluster) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev][cs] != 0) return cache[dev][cs] > 0 ? cache[dev][cs] : 0;
  auto kernel = sana_head_cluster<__nv_bfloat16, __nv_bfloat16, false>;
  int n = 0;
  if (kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kFusedThreads, ClusterSmem::kBytes, nullptr) ==
      KF_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = ClusterSmem::kBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
  }
  cache[dev][cs] = n > 0 ? n : -1;
  return n > 0 ? n : 0;
}

// CTAs per (batch, head) unit on the fused path: 1 when the units alone give every SM work;
// otherwise the largest cluster size (at most 8, and at most one CTA per 64-token K/V stage) whose
// clusters, one per unit, are all resident at once.
int fused_cluster_size(int64_t B, int64_t H, int64_t N) {
  const int64_t units = B * H, sms = kf_host::current_device_sms();
  if (units >= sms) return 1;
  const int64_t kv_all = (N + kFusedKTok - 1) / kFusedKTok;
  int best = 1;
  for (int cs = 2; cs <= kFusedMaxCluster && cs <= kv_all && units * cs <= sms; ++cs)
    if (units <= fused_max_clusters(cs)) best = cs;
  return best;
}

// The fused path (no workspace) is the automatic choice when its CTAs give the SMs work, or
// when they outnumber the split path's producer CTAs (few heads: the split path caps its
// splits per head pair). One CTA per unit: at least 90% of the CTA slots of the last wave busy.
// Clusters: each CTA's share of the tokens between 1024 and 4096 (shorter shares carry too much
// fixed cost, and on longer ones the split path's pipeline streams faster), and at least 85% of
// the SMs busy. The rules follow same-box timings of the two paths over batch 1-4, 2-100 heads,
// 1K-16K tokens.
bool fused_preferred(int64_t B, int64_t H, int64_t N) {
  const int64_t sms = kf_host::current_device_sms();
  const int cs = fused_cluster_size(B, H, N);
  const int64_t ctas = B * H * cs;
  if (cs == 1) {
    const int64_t waves = (ctas + sms - 1) / sms;
    if (ctas * 10 >= waves * sms * 9) return true;
  } else {
    const int64_t share = N / cs;
    if (share < 1024 || share > 4096) return false;
    if (ctas * 100 >= sms * 85) return true;
  }
  return B * ceil_div(H, kFastHeads) * fast_splits(B, H, N, 0) < ctas;
}

template <typename T>
int launch_fused(const void* qkv, void* out, int B, int H, int N, float eps, int out_dtype, cudaStream_t stream,
                 const QkNorm* nrm) {
  const QkNorm nv = nrm ? *nrm : QkNorm{};
  const int C = H * kD;
  const int in_dtype = std::is_same<T, __half>::value ? KF_DTYPE_F16 : KF_DTYPE_BF16;
  const size_t es = 2;
  // qkv [B, N, 3, C] as (channel, q/k/v, token, batch); boxes of one head (32 channels,
  // 64 bytes) x 64 tokens (K, V) or x 128 tokens (Q).
  CUtensorMap kv_map, q_map, out_map;
  const uint64_t dims[4] = {static_cast<uint64_t>(C), 3, static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {C * es, 3 * C * es, static_cast<uint64_t>(N) * 3 * C * es};
  const uint32_t kv_box[4] = {static_cast<uint32_t>(kD), 1, kFusedKTok, 1};
  const uint32_t q_box[4] = {static_cast<uint32_t>(kD), 1, kFusedQTok, 1};
  if (!kf_host::encode_tiled(&kv_map, kf_host::map_type(in_dtype), 4, qkv, dims, strides, kv_box,
                             CU_TENSOR_MAP_SWIZZLE_64B) ||
      !kf_host::encode_tiled(&q_map, kf_host::map_type(in_dtype), 4, qkv, dims, strides, q_box,
                             CU_TENSOR_MAP_SWIZZLE_64B))
    return KF_ERR_CUDA;
  // out [B, N, C]: boxes of one head x 16 tokens, one per compute warp and 16 tokens.
  const size_t os = kf::dtype_size(out_dtype);
  const uint64_t odims[3] = {static_cast<uint64_t>(C), static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
  const uint64_t ostrides[2] = {C * os, static_cast<uint64_t>(N) * C * os};
  const uint32_t obox[3] = {static_cast<uint32_t>(kD), kFusedSub, 1};
  if (!kf_host::encode_tiled(&out_map, kf_host::map_type(out_dtype), 3, out, odims, ostrides, obox,
                             os == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
    return KF_ERR_CUDA;
  const int64_t units = static_cast<int64_t>(B) * H;
  const int cs = fused_cluster_size(B, H, N);
  auto run = [&](auto one_cta, auto clustered) -> int {
    if (cs == 1) {
      const int grid = static_cast<int>(std::min<int64_t>(units, kf_host::current_device_sms()));
      const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(one_cta), kFusedThreads,
                                               FusedSmem::kBytes, nullptr);
      if (prep != KF_OK) return prep;
      one_cta<<<grid, kFusedThreads, FusedSmem::kBytes, stream>>>(kv_map, q_map, out_map, B, H, N, eps, nv);
      KF_LAUNCH_CHECK();
      return KF_OK;
    }
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(clustered), kFusedThreads,
                                             ClusterSmem::kBytes, nullptr);
    if (prep != KF_OK) return prep;
    // One cluster per unit (fused_cluster_size checked that they are all resident at once).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(units * cs));
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = ClusterSmem::kBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KF_CUDA_TRY(cudaLaunchKernelEx(&cfg, clustered, kv_map, q_map, out_map, B, H, N, eps, nv));
    return KF_OK;
  };
  if (nrm) {
    switch (out_dtype) {
      case KF_DTYPE_F32: return run(sana_head_fused<T, float, true>, sana_head_cluster<T, float, true>);
      case KF_DTYPE_F16: return run(sana_head_fused<T, __half, true>, sana_head_cluster<T, __half, true>);
      default: return run(sana_head_fused<T, __nv_bfloat16, true>, sana_head_cluster<T, __nv_bfloat16, true>);
    }
  }
  switch (out_dtype) {
    case KF_DTYPE_F32: return run(sana_head_fused<T, float, false>, sana_head_cluster<T, float, false>);
    case KF_DTYPE_F16: return run(sana_head_fused<T, __half, false>, sana_head_cluster<T, __half, false>);
    default: return run(sana_head_fused<T, __nv_bfloat16, false>, sana_head_cluster<T, __nv_bfloat16, false>);
  }
}

// ws: the workspace laid out by fast_layout(B, H, S); its counters are zero between calls.
template <typename T, int G>
int launch_fast(const void* qkv, void* out, uint8_t* ws, int B, int H, int N, int S, float eps, int out_dtype,
                cudaStream_t stream, const QkNorm* nrm) {
  const QkNorm nv = nrm ? *nrm : QkNorm{};
  static_assert(G == 2, "the epilogue works on head pairs");
  const int C = H * kD;
  const int in_dtype = std::is_same<T, __half>::value ? KF_DTYPE_F16 : KF_DTYPE_BF16;
  const size_t es = 2;
  float* partial = reinterpret_cast<float*>(ws + fast_layout(B, H, S).partial_off);
  // qkv [B, N, 3, C] seen as 4-D (channel, q/k/v, token, batch); boxes of 64 channels (one
  // head pair, 128 bytes) x 64 tokens for the producer and x 128 tokens for the epilogue.
  CUtensorMap kv_map, q_map, out_map;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(C), 3, static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
    const uint64_t strides[3] = {C * es, 3 * C * es, static_cast<uint64_t>(N) * 3 * C * es};
    const uint32_t box[4] = {64, 1, kTok, 1};
    if (!kf_host::encode_tiled(&kv_map, kf_host::map_type(in_dtype), 4, qkv, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B))
      return KF_ERR_CUDA;
    const uint32_t qbox[4] = {64, 1, kOutTok, 1};
    if (!kf_host::encode_tiled(&q_map, kf_host::map_type(in_dtype), 4, qkv, dims, strides, qbox,
                               CU_TENSOR_MAP_SWIZZLE_128B))
      return KF_ERR_CUDA;
  }
  {
    // out [B, N, C]: boxes of one head (32 channels) x 32 tokens, one per epilogue worker warp.
    const size_t os = kf::dtype_size(out_dtype);
    const uint64_t dims[3] = {static_cast<uint64_t>(C), static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
    const uint64_t strides[2] = {C * os, static_cast<uint64_t>(N) * C * os};
    const uint32_t box[3] = {static_cast<uint32_t>(kD), 32, 1};
    if (!kf_host::encode_tiled(&out_map, kf_host::map_type(out_dtype), 3, out, dims, strides, box,
                               os == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      return KF_ERR_CUDA;
  }
  const int HG = (H + G - 1) / G;
  const int tiles = (N + kTok - 1) / kTok;
  const int tps = (tiles + S - 1) / S;
  {
    auto kernel = nrm ? sana_vk_producer<T, G, kFastStages, true> : sana_vk_producer<T, G, kFastStages, false>;
    const int smem = kFastStages * 2 * (G / 2) * kBoxBytes + kFastStages * 8 + 1024;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), G * 32, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3(S, HG, B), G * 32, smem, stream>>>(kv_map, partial, H, tiles, tps, nv);
    KF_LAUNCH_CHECK();
  }
  auto run = [&](auto kernel, int smem) -> int {
    int occ = 1;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kEpiThreads, smem, &occ,
                                             static_cast<int>(kEpiTmemCols));
    if (prep != KF_OK) return prep;
    const int tiles_out = (N + kOutTok - 1) / kOutTok;
    const int total = B * HG * tiles_out;
    const int grid_cap = kf_host::current_device_sms() * occ;
    const int per = (total + grid_cap - 1) / grid_cap;
    const int grid = (total + per - 1) / per;
    // Programmatic dependent launch: overlaps this grid's prologue (its Q loads) with the
    // producer's tail; the partials are read after griddepcontrol.wait.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kEpiThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, q_map, out_map, static_cast<const float*>(partial), H, S, HG,
                                   tiles_out, total, per, eps, nv));
    return KF_OK;
  };
  if (nrm) {
    switch (out_dtype) {
      case KF_DTYPE_F32: return run(sana_out_tc<T, float, true>, EpiCfg<float>::kSmemBytes);
      case KF_DTYPE_F16: return run(sana_out_tc<T, __half, true>, EpiCfg<__half>::kSmemBytes);
      default: return run(sana_out_tc<T, __nv_bfloat16, true>, EpiCfg<__nv_bfloat16>::kSmemBytes);
    }
  }
  switch (out_dtype) {
    case KF_DTYPE_F32: return run(sana_out_tc<T, float, false>, EpiCfg<float>::kSmemBytes);
    case KF_DTYPE_F16: return run(sana_out_tc<T, __half, false>, EpiCfg<__half>::kSmemBytes);
    default: return run(sana_out_tc<T, __nv_bfloat16, false>, EpiCfg<__nv_bfloat16>::kSmemBytes);
  }
}

template <typename T>
int launch_generic(const void* qkv, void* out, float* partial, float* final_vk,
                   unsigned int* counters, int B, int H, int d, int N, int S, float eps,
                   int out_dtype, cudaStream_t stream, const QkNorm* nrm) {
  const QkNorm nv = nrm ? *nrm : QkNorm{};
  const T* q = static_cast<const T*>(qkv);
  const int nelem = (d + 1) * d;
  const int tiles = (N + kTok - 1) / kTok;
  const int tps = (tiles + S - 1) / S;
  {
    const int smem = (nelem + 2 * kGenTok * d) * static_cast<int>(sizeof(float));
    auto kernel = nrm ? sana_vk_generic<T, true> : sana_vk_generic<T, false>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kGenThreads, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3(S, H, B), kGenThreads, smem, stream>>>(q, partial, final_vk, counters, H, d, N, tps, nv);
    KF_LAUNCH_CHECK();
  }
  const int smem = (nelem + kGenTok * d + kGenTok) * static_cast<int>(sizeof(float));
  const dim3 grid((N + kGenTok - 1) / kGenTok, H, B);
  auto run = [&](auto kernel, auto* optr) -> int {
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kGenThreads, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<grid, kGenThreads, smem, stream>>>(q, final_vk, optr, H, d, N, eps, nv);
    KF_LAUNCH_CHECK();
    return KF_OK;
  };
  if (nrm) {
    switch (out_dtype) {
      case KF_DTYPE_F32: return run(sana_out_generic<T, float, true>, static_cast<float*>(out));
      case KF_DTYPE_F16: return run(sana_out_generic<T, __half, true>, static_cast<__half*>(out));
      default: return run(sana_out_generic<T, __nv_bfloat16, true>, static_cast<__nv_bfloat16*>(out));
    }
  }
  switch (out_dtype) {
    case KF_DTYPE_F32: return run(sana_out_generic<T, float, false>, static_cast<float*>(out));
    case KF_DTYPE_F16: return run(sana_out_generic<T, __half, false>, static_cast<__half*>(out));
    default: return run(sana_out_generic<T, __nv_bfloat16, false>, static_cast<__nv_bfloat16*>(out));
  }
}

bool valid_head_dim(int64_t d) { return d > 0 && d <= 128 && 128 % d == 0; }

// Workspace bytes: either path may run for head dim 32 (the input dtype decides).
size_t workspace_bytes_for(int64_t B, int64_t H, int64_t d, int64_t N, int64_t requested) {
  const size_t g = layout_for(B, H, d, generic_splits(B, H, N, requested)).total;
  return d == kD ? std::max(g, fast_layout(B, H, fast_splits(B, H, N, requested)).total) : g;
}

}  // namespace

int kf_internal_sana_error(unsigned int* code) {
  unsigned int v = 0;
  KF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_sana_error, sizeof(v)));
  if (v != 0) {
    const unsigned int zero = 0;
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_sana_error, &zero, sizeof(zero)));
  }
  *code = v;
  return KF_OK;
}

KF_API size_t kf_sana_linattn_workspace_size(int64_t batch, int64_t heads, int64_t dim,
                                             int64_t seq_len, int64_t splits) {
  if (batch <= 0 || heads <= 0 || seq_len <= 0 || !valid_head_dim(dim)) return 0;
  return workspace_bytes_for(batch, heads, dim, seq_len, splits);
}

namespace {

// Validation shared by the workspace entry points.
int check_args(const void* qkv, const void* out, int64_t batch, int64_t heads, int64_t dim, int64_t seq_len,
               float eps, int in_dtype, int out_dtype) {
  if (!kf::dtype_valid(in_dtype) || !kf::dtype_valid(out_dtype)) return KF_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || seq_len <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (!valid_head_dim(dim)) return KF_ERR_UNSUPPORTED;
  if (qkv == nullptr || out == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  // TMA coordinates and kernel indices are 32-bit.
  if (batch > 65535 || seq_len > (int64_t(1) << 30) || heads * dim > (int64_t(1) << 24) ||
      batch * seq_len * 3 * heads * dim > (int64_t(1) << 40))
    return KF_ERR_UNSUPPORTED;
  if (!kf::aligned(qkv, kf::dtype_size(in_dtype)) || !kf::aligned(out, kf::dtype_size(out_dtype)))
    return KF_ERR_MISALIGNED;
  return KF_OK;
}

// The attention proper, after validation; nrm != nullptr applies qk_norm from nrm->stats.
int sana_forward(const void* qkv, void* out, uint8_t* ws, int64_t batch, int64_t heads, int64_t dim,
                 int64_t seq_len, int64_t splits, float eps, int in_dtype, int out_dtype, cudaStream_t s,
                 const QkNorm* nrm) {
  const int S_gen = generic_splits(batch, heads, seq_len, splits);
  const WorkspaceLayout lay = layout_for(batch, heads, dim, S_gen);
  float* partial = reinterpret_cast<float*>(ws + lay.partial_off);
  float* final_vk = reinterpret_cast<float*>(ws + lay.final_off);
  unsigned int* counters = reinterpret_cast<unsigned int*>(ws + lay.counter_off);
  const int B = static_cast<int>(batch), H = static_cast<int>(heads), d = static_cast<int>(dim);
  const int N = static_cast<int>(seq_len);
  const bool fast = d == kD && (in_dtype == KF_DTYPE_BF16 || in_dtype == KF_DTYPE_F16) &&
                    H * kD >= 64 && N >= kTok && kf::aligned(qkv, 16) && kf::aligned(out, 16);
  if (fast && (splits == -1 || (splits == 0 && fused_preferred(B, H, N)))) {
    // Whole heads per CTA (or per cluster of CTAs), one launch, no workspace traffic.
    if (in_dtype == KF_DTYPE_BF16) return launch_fused<__nv_bfloat16>(qkv, out, B, H, N, eps, out_dtype, s, nrm);
    return launch_fused<__half>(qkv, out, B, H, N, eps, out_dtype, s, nrm);
  }
  if (fast) {
    // Two heads (one 128-byte TMA box) per CTA measured at or above four heads on every
    // benchmark shape.
    const int S = fast_splits(B, H, N, splits);
    if (in_dtype == KF_DTYPE_BF16)
      return launch_fast<__nv_bfloat16, kFastHeads>(qkv, out, ws, B, H, N, S, eps, out_dtype, s, nrm);
    return launch_fast<__half, kFastHeads>(qkv, out, ws, B, H, N, S, eps, out_dtype, s, nrm);
  }
  switch (in_dtype) {
    case KF_DTYPE_F32:
      return launch_generic<float>(qkv, out, partial, final_vk, counters, B, H, d, N, S_gen, eps, out_dtype, s, nrm);
    case KF_DTYPE_F16:
      return launch_generic<__half>(qkv, out, partial, final_vk, counters, B, H, d, N, S_gen, eps, out_dtype, s, nrm);
    default:
      return launch_generic<__nv_bfloat16>(qkv, out, partial, final_vk, counters, B, H, d, N, S_gen, eps, out_dtype,
                                           s, nrm);
  }
}

int64_t stats_tokens(int64_t N) { return (N + kStatsPad - 1) / kStatsPad * kStatsPad; }

}  // namespace

KF_API int kf_sana_linattn_fwd(const void* qkv, void* out, void* workspace, size_t workspace_bytes,
                               int64_t batch, int64_t heads, int64_t dim, int64_t seq_len,
                               int64_t splits, float eps, int in_dtype, int out_dtype,
                               void* stream) {
  const int st = check_args(qkv, out, batch, heads, dim, seq_len, eps, in_dtype, out_dtype);
  if (st != KF_OK) return st;
  if (workspace == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < workspace_bytes_for(batch, heads, dim, seq_len, splits)) return KF_ERR_WORKSPACE;
  if (!kf::aligned(workspace, 256)) return KF_ERR_MISALIGNED;
  return sana_forward(qkv, out, static_cast<uint8_t*>(workspace), batch, heads, dim, seq_len, splits, eps,
                      in_dtype, out_dtype, static_cast<cudaStream_t>(stream), nullptr);
}

KF_API size_t kf_sana_linattn_qknorm_workspace_size(int64_t batch, int64_t heads, int64_t dim, int64_t seq_len,
                                                    int64_t splits) {
  if (batch <= 0 || heads <= 0 || seq_len <= 0 || !valid_head_dim(dim)) return 0;
  return align256(workspace_bytes_for(batch, heads, dim, seq_len, splits)) +
         align256(static_cast<size_t>(batch) * stats_tokens(seq_len) * 2 * sizeof(float));
}

KF_API int kf_sana_linattn_qknorm_fwd(const void* qkv, void* out, void* workspace, size_t workspace_bytes,
                                      int64_t batch, int64_t heads, int64_t dim, int64_t seq_len, int64_t splits,
                                      float eps, const void* q_weight, const void* k_weight, float norm_eps,
                                      int in_dtype, int out_dtype, void* stream) {
  const int st = check_args(qkv, out, batch, heads, dim, seq_len, eps, in_dtype, out_dtype);
  if (st != KF_OK) return st;
  if (workspace == nullptr || q_weight == nullptr || k_weight == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!(norm_eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < kf_sana_linattn_qknorm_workspace_size(batch, heads, dim, seq_len, splits))
    return KF_ERR_WORKSPACE;
  if (!kf::aligned(workspace, 256)) return KF_ERR_MISALIGNED;
  // The tensor-core epilogue reads each head's 32 q weights as 16-byte vectors.
  if (!kf::aligned(q_weight, 16) || !kf::aligned(k_weight, 16)) return KF_ERR_MISALIGNED;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t npad = stats_tokens(seq_len);
  float* stats = reinterpret_cast<float*>(ws + align256(workspace_bytes_for(batch, heads, dim, seq_len, splits)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int C = static_cast<int>(heads * dim), N = static_cast<int>(seq_len);
  const dim3 grid(static_cast<unsigned>((npad + 7) / 8), static_cast<unsigned>(batch));
  switch (in_dtype) {
    case KF_DTYPE_F32:
      sana_qk_stats<float><<<grid, 256, 0, s>>>(static_cast<const float*>(qkv), stats, N, C, static_cast<int>(npad),
                                                norm_eps);
      break;
    case KF_DTYPE_F16:
      sana_qk_stats<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(qkv), stats, N, C,
                                                 static_cast<int>(npad), norm_eps);
      break;
    default:
      sana_qk_stats<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(qkv), stats, N, C,
                                                        static_cast<int>(npad), norm_eps);
  }
  KF_LAUNCH_CHECK();
  const QkNorm nrm{stats, q_weight, k_weight, static_cast<int>(npad)};
  return sana_forward(qkv, out, ws, batch, heads, dim, seq_len, splits, eps, in_dtype, out_dtype, s, &nrm);
}

KF_API int kf_sana_linattn_plan(int64_t batch, int64_t heads, int64_t dim, int64_t seq_len, int64_t splits,
                                int in_dtype, int64_t* launches, int64_t* ctas_per_unit) {
  if (launches == nullptr || ctas_per_unit == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!kf::dtype_valid(in_dtype)) return KF_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || seq_len <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (!valid_head_dim(dim)) return KF_ERR_UNSUPPORTED;
  if (batch > 65535 || seq_len > (int64_t(1) << 30) || heads * dim > (int64_t(1) << 24)) return KF_ERR_UNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return KF_ERR_CUDA;
  }
  // The same tests as kf_sana_linattn_fwd, for 16-byte aligned qkv and out.
  const bool fast = dim == kD && (in_dtype == KF_DTYPE_BF16 || in_dtype == KF_DTYPE_F16) && heads * kD >= 64 &&
                    seq_len >= kTok;
  if (fast && (splits == -1 || (splits == 0 && fused_preferred(batch, heads, seq_len)))) {
    *launches = 1;
    *ctas_per_unit = fused_cluster_size(batch, heads, seq_len);
  } else {
    *launches = 2;
    *ctas_per_unit = 0;
  }
  return KF_OK;
}

// ------------------------------------------------------------------------------------------
// No-allocation variant of kf_sana_linattn_fwd.
//
// Some callers cannot allocate device memory at call time: code that runs inside another
// runtime's memory manager or a custom allocator hook, or that owns a fixed memory budget
// and may not grow it. For them the scratch (the reduced K^T V / ksum, and for the generic
// path the split partials and arrival counters) lives in this file-scope device array instead
// of a caller-provided workspace. Every GPU that loads the library holds it until exit.
// ------------------------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) uint8_t g_sana_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Device address of the scratch array in the current context. In host code the array's name is
// only a host-side stand-in, so the address comes from cudaGetSymbolAddress. A __device__
// array's address belongs to a context, not to a device: it is looked up once per device and
// again whenever that device's current context is a different one (a cudaDeviceReset, or a
// driver-API caller's own context), never reused across contexts.
int noalloc_scratch(uint8_t** out) {
  struct Entry {
    unsigned long long ctx;
    uint8_t* addr;
  };
  static Entry cache[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return KF_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return KF_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long ctx = kf_host::context_id();
  if (ctx != 0 && cache[dev].ctx == ctx && cache[dev].addr != nullptr) {
    *out = cache[dev].addr;
    return KF_OK;
  }
  // Loads the library's module into the current context if needed (creating the runtime's
  // primary context first when none is current).
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_sana_noalloc_scratch) != cudaSuccess || p == nullptr) {
    (void)cudaGetLastError();
    return KF_ERR_CUDA;
  }
  const unsigned long long now = kf_host::context_id();
  cache[dev] = Entry{now, now != 0 ? static_cast<uint8_t*>(p) : nullptr};
  *out = static_cast<uint8_t*>(p);
  return KF_OK;
}

}  // namespace

KF_API size_t kf_sana_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

KF_API int kf_sana_linattn_fwd_noalloc(const void* qkv, void* out, int64_t batch, int64_t heads,
                                       int64_t dim, int64_t seq_len, int64_t splits, float eps,
                                       int in_dtype, int out_dtype, void* stream) {
  if (!kf::dtype_valid(in_dtype) || !kf::dtype_valid(out_dtype)) return KF_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || seq_len <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (!valid_head_dim(dim)) return KF_ERR_UNSUPPORTED;
  if (qkv == nullptr || out == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || seq_len > (int64_t(1) << 30) || heads * dim > (int64_t(1) << 24) ||
      batch * seq_len * 3 * heads * dim > (int64_t(1) << 40))
    return KF_ERR_UNSUPPORTED;
  if (!kf::aligned(qkv, kf::dtype_size(in_dtype)) || !kf::aligned(out, kf::dtype_size(out_dtype)))
    return KF_ERR_MISALIGNED;
  const int B = static_cast<int>(batch), H = static_cast<int>(heads), d = static_cast<int>(dim);
  const int N = static_cast<int>(seq_len);
  const bool fast = d == kD && (in_dtype == KF_DTYPE_BF16 || in_dtype == KF_DTYPE_F16) &&
                    H * kD >= 64 && N >= kTok && kf::aligned(qkv, 16) && kf::aligned(out, 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (fast && (splits == -1 || (splits == 0 && fused_preferred(B, H, N)))) {
    // The one-launch schedule, chosen exactly as kf_sana_linattn_fwd chooses it: it keeps
    // whole heads in shared memory and needs no scratch at all.
    if (in_dtype == KF_DTYPE_BF16) return launch_fused<__nv_bfloat16>(qkv, out, B, H, N, eps, out_dtype, s, nullptr);
    return launch_fused<__half>(qkv, out, B, H, N, eps, out_dtype, s, nullptr);
  }
  if (fast) {
    // As many splits as requested (or the default) and the scratch holds.
    int S = fast_splits(B, H, N, splits);
    while (S > 1 && fast_layout(B, H, S).total > kNoAllocScratchBytes) --S;
    if (fast_layout(B, H, S).total > kNoAllocScratchBytes) return KF_ERR_WORKSPACE;
    uint8_t* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st != KF_OK) return st;
    if (in_dtype == KF_DTYPE_BF16)
      return launch_fast<__nv_bfloat16, kFastHeads>(qkv, out, scratch, B, H, N, S, eps, out_dtype, s, nullptr);
    return launch_fast<__half, kFastHeads>(qkv, out, scratch, B, H, N, S, eps, out_dtype, s, nullptr);
  }
  // Generic path: as many splits as requested (or the default) and the scratch holds.
  int S = generic_splits(batch, heads, seq_len, splits);
  while (S > 1 && layout_for(batch, heads, dim, S).total > kNoAllocScratchBytes) --S;
  const WorkspaceLayout lay = layout_for(batch, heads, dim, S);
  if (lay.total > kNoAllocScratchBytes) return KF_ERR_WORKSPACE;
  uint8_t* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != KF_OK) return st;
  float* partial = reinterpret_cast<float*>(scratch + lay.partial_off);
  float* final_vk = reinterpret_cast<float*>(scratch + lay.final_off);
  unsigned int* counters = reinterpret_cast<unsigned int*>(scratch + lay.counter_off);
  // The arrival counters must start at zero; the array keeps whatever the last call left.
  KF_CUDA_TRY(cudaMemsetAsync(counters, 0, static_cast<size_t>(batch) * heads * sizeof(unsigned int), s));
  switch (in_dtype) {
    case KF_DTYPE_F32:
      return launch_generic<float>(qkv, out, partial, final_vk, counters, B, H, d, N, S, eps, out_dtype, s, nullptr);
    case KF_DTYPE_F16:
      return launch_generic<__half>(qkv, out, partial, final_vk, counters, B, H, d, N, S, eps, out_dtype, s, nullptr);
    default:
      return launch_generic<__nv_bfloat16>(qkv, out, partial, final_vk, counters, B, H, d, N, S, eps, out_dtype, s, nullptr);
  }
}
