// SANA linear attention fused with its QKV projection, for sm_100a: the grouped kernels of
// SANA_LinearAttention/custom.py:595-868 (grouped_full64_kv_vk_producer and
// partial_reduce_joint_qout, written there for B=1, N=1024, C=1152 only), generalised to any
// batch, sequence length and head count (head dim 32, bf16 as there). q, k and v never exist in memory:
//
//  1. sana_proj_kv    grid (splits, head groups of 4, batch), 192 threads
//     Per 128-token tile: [K | V] of the group's 4 heads = x_tile W_kv^T on the tcgen05 tensor
//     cores (M128 N256 K16, fp32 accumulators in tensor memory, two buffers), then the
//     epilogue warps round K and V to the input dtype (the projection's output rounding), add
//     the QKV bias if any, stage relu(K) and V token-major in shared memory, and each warp
//     accumulates one head's VK += V^T relu(K), ksum += relu(K) (mma.sync, fp32) over the
//     CTA's tiles. Each split writes its fp32 partial [VK ; ksum] (33 x 32 per head).
//  2. sana_proj_qout  grid (token splits, head groups of 4, batch), 192 threads
//     B = [VK ; ksum] of the group's heads, the split partials summed in split order, as hi +
//     lo 16-bit halves in shared memory (so the fp32 sums keep ~16 mantissa bits). Per
//     128-token tile: Q = x_tile W_q^T on the tensor cores (M128 N128 K16); the epilogue writes
//     relu(cast(Q)) back to tensor memory as the A operand of D = relu(Q) B (M128 N48 K16, B
//     from shared memory) and stores out = D[:, :32] / (D[:, 32] + eps).
// Warp roles in both: warp 0 TMA producer, warp 1 MMA issuer (one thread), warps 2-5 epilogue
// (warp w reads tensor-memory lanes 32 (w % 4) ..., i.e. tokens 32 (w % 4) .. + 31 of a tile).
// Every wait is bounded; after a timeout the roles leave their loops, the producer and the MMA
// thread wait (bounded) for what they have in flight, and tensor memory is freed.
#include "kf_sm100.cuh"
#include "kf_tcgen05.cuh"

#include <climits>
#include <type_traits>

namespace {

__device__ unsigned int g_proj_attn_error = 0;

constexpr int kHd = 32;               // head dim
constexpr int kGroup = 4;             // heads per CTA
constexpr int kGC = kGroup * kHd;     // channels per group: 128
constexpr int kTokT = 128;            // tokens per tile
constexpr int kKB = 64;               // K elements per stage
constexpr int kRowsB = kHd + 1;       // VK rows + the ksum row
constexpr int kPT = 192;              // threads
constexpr int kTmaWarp = 0, kMmaW = 1;

__device__ __forceinline__ uint64_t dsw(uint32_t base, uint32_t off) {
  return kf::tc::desc_advance(kf::tc::desc_sw128(base, 16, 1024), off);
}

// ---- kernel 1 ------------------------------------------------------------------------------
struct KvCfg {
  static constexpr int kStages = 3;
  static constexpr int kABytes = kTokT * kKB * 2;        // 16 KB
  static constexpr int kBBytes = 2 * kGC * kKB * 2;       // 32 KB: 128 k rows, then 128 v rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStageOff = kStages * kStageBytes;     // staging: per head 128 tokens x (k | v)
  static constexpr int kHeadStage = kTokT * 128;             // 16 KB
  static constexpr int kBarOff = kStageOff + kGroup * kHeadStage;
  static constexpr int kSmemBytes = kBarOff + 256 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

template <typename T>
__global__ void __launch_bounds__(kPT, 1)
sana_proj_kv(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
             const T* __restrict__ qkv_bias, float* __restrict__ partial, int N, int C, int H, int tiles_per_split) {
  using Cf = KvCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cf::kBarOff);
  uint64_t* empty = full + Cf::kStages;
  uint64_t* acc_full = empty + Cf::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, grp = blockIdx.y, b = blockIdx.z, S = gridDim.x;
  const int ntiles = (N + kTokT - 1) / kTokT;
  const int t_begin = split * tiles_per_split;
  const int t_end = min(ntiles, t_begin + tiles_per_split);
  const int k_steps = (C + kKB - 1) / kKB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cf::kStages; ++s) {
      kf::mbar_init(&full[s], 1);
      kf::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      kf::mbar_init(&acc_full[i], 1);
      kf::mbar_init(&acc_empty[i], 4);
    }
    kf::mbar_init(drain, 1);
    *abort_flag = 0;
    kf::fence_mbar_init();
  }
  if (warp == kMmaW) kf::tc::tmem_alloc(tmem_slot, 512);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      kf::prefetch_tensormap(&tm_x);
      kf::prefetch_tensormap(&tm_w);
      int issued = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        for (int ks = 0; ks < k_steps; ++ks) {
          const int s = issued % Cf::kStages, use = issued / Cf::kStages;
          if (use > 0 && !(ok = kf::mbar_wait_or_abort<true>(&empty[s], (use - 1) & 1, &g_proj_attn_error, abort_flag)))
            break;
          uint8_t* a = smem + s * Cf::kStageBytes;
          kf::mbar_arrive_expect_tx(&full[s], Cf::kStageBytes);
          kf::tma_load_4d(a, &tm_x, &full[s], ks * kKB, t * kTokT, b, 0);
          kf::tma_load_2d(a + Cf::kABytes, &tm_w, &full[s], ks * kKB, C + grp * kGC);
          kf::tma_load_2d(a + Cf::kABytes + Cf::kBBytes / 2, &tm_w, &full[s], ks * kKB, 2 * C + grp * kGC);
          ++issued;
        }
      }
      for (int i = issued > Cf::kStages ? issued - Cf::kStages : 0; i < issued; ++i)
        (void)kf::mbar_wait_bounded(&full[i % Cf::kStages], (i / Cf::kStages) & 1, &g_proj_attn_error);
    }
  } else if (warp == kMmaW) {
    if (lane == 0) {
      constexpr uint32_t idesc = kf::tc::idesc_f16(std::is_same<T, __nv_bfloat16>::value ? 1 : 0, kTokT, 2 * kGC,
                                                   false, false);
      int consumed = 0, local = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t, ++local) {
        const int ab = local & 1, use = local >> 1;
        if (use > 0 && !(ok = kf::mbar_wait_or_abort<true>(&acc_empty[ab], (use - 1) & 1, &g_proj_attn_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t d = tmem + ab * 2 * kGC;
        for (int ks = 0; ks < k_steps; ++ks, ++consumed) {
          const int s = consumed % Cf::kStages;
          if (!(ok = kf::mbar_wait_or_abort<true>(&full[s], (consumed / Cf::kStages) & 1, &g_proj_attn_error, abort_flag)))
            break;
          kf::tc::fence_after_sync();
          const uint32_t a = kf::smem_u32(smem + s * Cf::kStageBytes), bb = a + Cf::kABytes;
#pragma unroll
          for (int k = 0; k < kKB / 16; ++k) kf::tc::mma_ss(d, dsw(a, k * 32), dsw(bb, k * 32), idesc, (ks | k) != 0);
          kf::tc::commit(&empty[s]);
        }
        if (!ok) break;
        kf::tc::commit(&acc_full[ab]);
      }
      kf::tc::commit(drain);
      (void)kf::mbar_wait_bounded(drain, 0, &g_proj_attn_error);
    }
  } else {
    // ---- epilogue: warp (quarter) stages tokens 32 quarter .. of every head, then owns head
    // `quarter` of the group for VK += V^T relu(K) over all 128 tokens ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // token within the tile / tensor-memory lane
    const int gid = lane >> 2, tig = lane & 3, sub = lane >> 3;
    const int head = grp * kGroup + quarter;
    float acc[2][4][4], ksum[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.f;
    }
    bool ok = true;
    int local = 0;
    for (int t = t_begin; t < t_end; ++t, ++local) {
      const int ab = local & 1;
      ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&acc_full[ab], (local >> 1) & 1, &g_proj_attn_error,
                                                          abort_flag));
      if (!ok) break;
      kf::tc::fence_after_sync();
      const uint32_t lanes = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + ab * 2 * kGC;
      const bool valid = t * kTokT + row < N;
#pragma unroll 1
      for (int hh = 0; hh < kGroup; ++hh) {
        uint32_t kr[32], vr[32];
        kf::tc::ld_32x32b_x32(lanes + hh * kHd, kr);
        kf::tc::ld_32x32b_x32(lanes + kGC + hh * kHd, vr);
        kf::tc::wait_ld();
        const int kc = C + (grp * kGroup + hh) * kHd, vc = 2 * C + (grp * kGroup + hh) * kHd;
        uint32_t kp[16], vp[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float k0 = __uint_as_float(kr[2 * i]), k1 = __uint_as_float(kr[2 * i + 1]);
          float v0 = __uint_as_float(vr[2 * i]), v1 = __uint_as_float(vr[2 * i + 1]);
          if (qkv_bias != nullptr && grp * kGroup + hh < H) {
            k0 += kf::Elem<T>::to_f(qkv_bias[kc + 2 * i]);
            k1 += kf::Elem<T>::to_f(qkv_bias[kc + 2 * i + 1]);
            v0 += kf::Elem<T>::to_f(qkv_bias[vc + 2 * i]);
            v1 += kf::Elem<T>::to_f(qkv_bias[vc + 2 * i + 1]);
          }
          kp[i] = kf::Mma<T>::relu2(kf::Mma<T>::from_f2(k0, k1));  // relu(cast(k)) = cast(relu(k))
          vp[i] = kf::Mma<T>::from_f2(v0, v1);
          if (!valid) kp[i] = vp[i] = 0u;  // tokens past N (zero rows of x, but a bias would leak)
        }
        // Token-major rows of 128 bytes: k in 16-byte chunks 0-3, v in chunks 4-7 (128-byte swizzle).
        uint8_t* st = smem + KvCfg::kStageOff + hh * KvCfg::kHeadStage + row * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          *reinterpret_cast<uint4*>(st + ((c ^ (row & 7)) << 4)) = make_uint4(kp[4 * c], kp[4 * c + 1], kp[4 * c + 2], kp[4 * c + 3]);
          *reinterpret_cast<uint4*>(st + (((4 + c) ^ (row & 7)) << 4)) =
              make_uint4(vp[4 * c], vp[4 * c + 1], vp[4 * c + 2], vp[4 * c + 3]);
        }
      }
      // The accumulator is read: the MMAs of tile t + 2 may use it.
      kf::tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) kf::mbar_arrive(&acc_empty[ab]);
      kf::named_bar_sync(1, 128);  // the staging tiles are complete
      const uint32_t hbase = kf::smem_u32(smem + KvCfg::kStageOff + quarter * KvCfg::kHeadStage);
#pragma unroll 1
      for (int ks = 0; ks < kTokT / 16; ++ks) {
        uint32_t a[2][4], bf[4][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          // A = V^T (M = v channel, K = token): transposed loads of the token-major v chunks.
          const int r = ks * 16 + (lane & 7) + (sub >> 1) * 8;
          kf::ldsm_x4_t(hbase + kf::swz128(r, 4 + mt * 2 + (sub & 1)), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
        }
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          // B = relu(K) (K = token, N = k channel), two n-tiles per load.
          const int r = ks * 16 + (lane & 7) + (sub & 1) * 8;
          kf::ldsm_x4_t(hbase + kf::swz128(r, np * 2 + (sub >> 1)), bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0],
                        bf[2 * np + 1][1]);
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const float2 x = kf::Mma<T>::to_f2(bf[nt][0]), y = kf::Mma<T>::to_f2(bf[nt][1]);
          ksum[nt] += (x.x + x.y) + (y.x + y.y);
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) kf::Mma<T>::run(acc[mt][nt], a[mt], bf[nt]);
      }
      kf::named_bar_sync(1, 128);  // every head's staging tile has been read
    }
    // This split's partial [VK ; ksum] of head `head` (nothing after a timeout).
    if (ok && head < H) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 1);
        ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 2);
      }
      float* dst = partial + ((static_cast<size_t>(b) * H + head) * S + split) * (kRowsB * kHd);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int r = mt * 16 + gid, c = nt * 8 + tig * 2;
          *reinterpret_cast<float2*>(dst + r * kHd + c) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
          *reinterpret_cast<float2*>(dst + (r + 8) * kHd + c) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
        }
      if (tig == 0) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) dst[kHd * kHd + nt * 8 + gid] = ksum[nt];
      }
    }
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaW) {
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, 512);
  }
}

// ---- kernel 2 ------------------------------------------------------------------------------
constexpr int kBRows = 48;                 // B rows per head: 32 VK rows, ksum, 15 zero
constexpr int kBImage = kBRows * 128;      // (32 hi + 32 lo) 16-bit values per row
struct QoutCfg {
  static constexpr int kStages = 5;
  static constexpr int kABytes = kTokT * kKB * 2;   // 16 KB
  static constexpr int kBBytes = kGC * kKB * 2;      // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBImgOff = kStages * kStageBytes;
  static constexpr int kOutOff = kBImgOff + kGroup * kBImage;  // 4 warps x 2 buffers x 32 x 32 outputs
  static constexpr int kOutChunk = 32 * kHd * 2;
  static constexpr int kBarOff = kOutOff + 4 * 2 * kOutChunk;
  static constexpr int kSmemBytes = kBarOff + 256 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};
// Tensor memory: Q accumulators at 0 and 128; head h's D at 256 + 64 h (48 columns) and its A at
// 256 + 64 h + 48 (16 columns of packed 16-bit pairs).
__device__ __forceinline__ uint32_t qo_slot(int h) { return 256u + 64u * h; }

template <typename T>
__global__ void __launch_bounds__(kPT, 1)
sana_proj_qout(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
               const __grid_constant__ CUtensorMap tm_out, const T* __restrict__ qkv_bias,
               const float* __restrict__ partial, int N, int C, int H, int S, int tiles_per_cta, float eps) {
  using Cf = QoutCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cf::kBarOff);
  uint64_t* empty = full + Cf::kStages;
  uint64_t* acc_full = empty + Cf::kStages;  // [2] Q of a tile computed
  uint64_t* acc_empty = acc_full + 2;        // [2] Q read by the 4 epilogue warps
  uint64_t* a_ready = acc_empty + 2;         // A of a tile written (and D of the previous tile read)
  uint64_t* d_full = a_ready + 1;            // D of a tile computed
  uint64_t* drain = d_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.y, b = blockIdx.z;
  const int ntiles = (N + kTokT - 1) / kTokT;
  const int t_begin = blockIdx.x * tiles_per_cta;
  const int t_end = min(ntiles, t_begin + tiles_per_cta);
  const int k_steps = (C + kKB - 1) / kKB;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cf::kStages; ++s) {
      kf::mbar_init(&full[s], 1);
      kf::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      kf::mbar_init(&acc_full[i], 1);
      kf::mbar_init(&acc_empty[i], 4);
    }
    kf::mbar_init(a_ready, 4);
    kf::mbar_init(d_full, 1);
    kf::mbar_init(drain, 1);
    *abort_flag = 0;
    kf::fence_mbar_init();
  }
  if (warp == kMmaW) kf::tc::tmem_alloc(tmem_slot, 512);
  // B images of the group's heads: the S split partials summed in split order; hi + lo halves.
  for (int task = threadIdx.x; task < kGroup * kBRows * 4; task += kPT) {
    const int hh = task / (kBRows * 4), n = (task / 4) % kBRows, kg = task % 4;
    const int h = grp * kGroup + hh;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (h < H && n < kRowsB) {
      const float* src = partial + (static_cast<size_t>(b) * H + h) * S * (kRowsB * kHd) + n * kHd + kg * 8;
      for (int sp = 0; sp < S; ++sp) {
        const float4 x0 = __ldcg(reinterpret_cast<const float4*>(src + sp * (kRowsB * kHd)));
        const float4 x1 = __ldcg(reinterpret_cast<const float4*>(src + sp * (kRowsB * kHd) + 4));
        v[0] += x0.x; v[1] += x0.y; v[2] += x0.z; v[3] += x0.w;
        v[4] += x1.x; v[5] += x1.y; v[6] += x1.z; v[7] += x1.w;
      }
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      hi[e] = kf::Mma<T>::from_f2(v[2 * e], v[2 * e + 1]);
      const float2 hf = kf::Mma<T>::to_f2(hi[e]);
      lo[e] = kf::Mma<T>::from_f2(v[2 * e] - hf.x, v[2 * e + 1] - hf.y);
    }
    uint8_t* rowp = smem + Cf::kBImgOff + hh * kBImage + n * 128;
    *reinterpret_cast<uint4*>(rowp + ((kg ^ (n & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(rowp + (((4 + kg) ^ (n & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
  kf::fence_proxy_async_smem();  // the tensor cores read B through the async proxy
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      kf::prefetch_tensormap(&tm_x);
      kf::prefetch_tensormap(&tm_w);
      int issued = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        for (int ks = 0; ks < k_steps; ++ks) {
          const int s = issued % Cf::kStages, use = issued / Cf::kStages;
          if (use > 0 && !(ok = kf::mbar_wait_or_abort<true>(&empty[s], (use - 1) & 1, &g_proj_attn_error, abort_flag)))
            break;
          uint8_t* a = smem + s * Cf::kStageBytes;
          kf::mbar_arrive_expect_tx(&full[s], Cf::kStageBytes);
          kf::tma_load_4d(a, &tm_x, &full[s], ks * kKB, t * kTokT, b, 0);
          kf::tma_load_2d(a + Cf::kABytes, &tm_w, &full[s], ks * kKB, grp * kGC);
          ++issued;
        }
      }
      for (int i = issued > Cf::kStages ? issued - Cf::kStages : 0; i < issued; ++i)
        (void)kf::mbar_wait_bounded(&full[i % Cf::kStages], (i / Cf::kStages) & 1, &g_proj_attn_error);
    }
  } else if (warp == kMmaW) {
    if (lane == 0) {
      constexpr uint32_t idq = kf::tc::idesc_f16(kBf16 ? 1 : 0, kTokT, kGC, false, false);
      constexpr uint32_t idd = kf::tc::idesc_f16(kBf16 ? 1 : 0, kTokT, kBRows, false, false);
      const uint32_t bimg = kf::smem_u32(smem + Cf::kBImgOff);
      int consumed = 0, local = 0, d_issued = 0;
      bool ok = true;
      // D = relu(Q) B of tile j, once its A is written (and the previous D has been read).
      auto issue_d = [&](int j) -> bool {
        if (!kf::mbar_wait_or_abort<true>(a_ready, j & 1, &g_proj_attn_error, abort_flag)) return false;
        kf::tc::fence_after_sync();
#pragma unroll
        for (int hh = 0; hh < kGroup; ++hh) {
          const uint32_t slot = tmem + qo_slot(hh);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)  // hi k 0-15, hi k 16-31, lo k 0-15, lo k 16-31
            kf::tc::mma_ts(slot, slot + 48 + (ks & 1) * 8, kf::tc::desc_sw128(bimg + hh * kBImage + ks * 32, 16, 1024),
                           idd, ks > 0 ? 1u : 0u);
        }
        kf::tc::commit(d_full);
        ++d_issued;
        return true;
      };
      for (int t = t_begin; ok && t < t_end; ++t, ++local) {
        const int ab = local & 1, use = local >> 1;
        if (use > 0 && !(ok = kf::mbar_wait_or_abort<true>(&acc_empty[ab], (use - 1) & 1, &g_proj_attn_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t d = tmem + ab * kGC;
        for (int ks = 0; ks < k_steps; ++ks, ++consumed) {
          const int s = consumed % Cf::kStages;
          if (!(ok = kf::mbar_wait_or_abort<true>(&full[s], (consumed / Cf::kStages) & 1, &g_proj_attn_error, abort_flag)))
            break;
          kf::tc::fence_after_sync();
          const uint32_t a = kf::smem_u32(smem + s * Cf::kStageBytes), bb = a + Cf::kABytes;
#pragma unroll
          for (int k = 0; k < kKB / 16; ++k) kf::tc::mma_ss(d, dsw(a, k * 32), dsw(bb, k * 32), idq, (ks | k) != 0);
          kf::tc::commit(&empty[s]);
        }
        if (!ok) break;
        kf::tc::commit(&acc_full[ab]);
        if (local > 0 && !(ok = issue_d(local - 1))) break;
      }
      if (ok && local > 0) ok = issue_d(local - 1);
      kf::tc::commit(drain);
      (void)kf::mbar_wait_bounded(drain, 0, &g_proj_attn_error);
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    int local = 0;
    // out of tile j: D / (D[:, 32] + eps) for the group's heads. Each warp's 32 tokens x 32
    // channels of a head go through shared memory (64-byte swizzle: 16-byte piece v of row r at
    // v ^ ((r >> 1) & 3)) into one TMA store, which clips tokens past N.
    uint8_t* out_stage = smem + Cf::kOutOff + quarter * 2 * Cf::kOutChunk;
    const uint32_t swz = (lane >> 1) & 3;
    int chunks = 0;
    auto store_out = [&](int j) -> bool {
      if (!__all_sync(0xffffffffu, kf::mbar_wait_or_abort(d_full, j & 1, &g_proj_attn_error, abort_flag))) return false;
      kf::tc::fence_after_sync();
      const int tok0 = (t_begin + j) * kTokT + quarter * 32;
#pragma unroll 1
      for (int hh = 0; hh < kGroup; ++hh) {
        uint32_t dr[32], den[2];
        kf::tc::ld_32x32b_x32(tmem + lanes + qo_slot(hh), dr);
        kf::tc::ld_32x32b_x2(tmem + lanes + qo_slot(hh) + 32, den);
        kf::tc::wait_ld();
        const int h = grp * kGroup + hh;
        if (h >= H || tok0 >= N) continue;  // warp-uniform
        uint8_t* st = out_stage + (chunks & 1) * Cf::kOutChunk;
        // The store issued from this buffer two chunks ago has finished reading it.
        if (chunks >= 2 && lane == 0) kf::tma_store_wait_read1();
        __syncwarp();
        const float inv = __frcp_rn(__uint_as_float(den[0]) + eps);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 o;
          o.x = kf::Mma<T>::from_f2(__uint_as_float(dr[8 * v]) * inv, __uint_as_float(dr[8 * v + 1]) * inv);
          o.y = kf::Mma<T>::from_f2(__uint_as_float(dr[8 * v + 2]) * inv, __uint_as_float(dr[8 * v + 3]) * inv);
          o.z = kf::Mma<T>::from_f2(__uint_as_float(dr[8 * v + 4]) * inv, __uint_as_float(dr[8 * v + 5]) * inv);
          o.w = kf::Mma<T>::from_f2(__uint_as_float(dr[8 * v + 6]) * inv, __uint_as_float(dr[8 * v + 7]) * inv);
          *reinterpret_cast<uint4*>(st + lane * 64 + ((v ^ swz) << 4)) = o;
        }
        kf::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          kf::tma_store_3d(&tm_out, st, h * kHd, tok0, b);
          kf::tma_store_commit();
        }
        ++chunks;
      }
      return true;
    };
    for (int t = t_begin; t < t_end; ++t, ++local) {
      const int ab = local & 1;
      ok = __all_sync(0xffffffffu, kf::mbar_wait_or_abort(&acc_full[ab], (local >> 1) & 1, &g_proj_attn_error,
                                                          abort_flag));
      if (!ok) break;
      // A is single-buffered: the previous tile's D must be computed and read before it is rewritten.
      if (local > 0 && !(ok = store_out(local - 1))) break;
      kf::tc::fence_after_sync();
#pragma unroll 1
      for (int hh = 0; hh < kGroup; ++hh) {
        uint32_t qr[32];
        kf::tc::ld_32x32b_x32(tmem + lanes + ab * kGC + hh * kHd, qr);
        kf::tc::wait_ld();
        const int qc = (grp * kGroup + hh) * kHd;
        const bool bias = qkv_bias != nullptr && grp * kGroup + hh < H;
        uint32_t ap[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float q0 = __uint_as_float(qr[2 * i]), q1 = __uint_as_float(qr[2 * i + 1]);
          if (bias) {
            q0 += kf::Elem<T>::to_f(qkv_bias[qc + 2 * i]);
            q1 += kf::Elem<T>::to_f(qkv_bias[qc + 2 * i + 1]);
          }
          ap[i] = kf::Mma<T>::relu2(kf::Mma<T>::from_f2(q0, q1));
        }
        kf::tc::st_32x32b_x16(tmem + lanes + qo_slot(hh) + 48, ap);
      }
      kf::tc::wait_st();
      kf::tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        kf::mbar_arrive(&acc_empty[ab]);
        kf::mbar_arrive(a_ready);
      }
    }
    if (ok && local > 0) (void)store_out(local - 1);
    // Shared memory outlives the stores in flight, and they complete before the kernel ends.
    if (lane == 0) kf::tma_store_wait_all0();
    __syncwarp();
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaW) {
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int kf_internal_proj_attn_error(unsigned int* code) {
  unsigned int v = 0;
  KF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_proj_attn_error, sizeof(v)));
  if (v != 0) {
    const unsigned int zero = 0;
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_proj_attn_error, &zero, sizeof(zero)));
  }
  *code = v;
  return KF_OK;
}

namespace {

// Token splits of kernel 1 (each split covers whole 128-token tiles). One CTA fits per SM, so
// the kernel takes waves x tiles-per-split tile times: the split count minimising that, the
// smallest on ties (fewer partials). B = 2, C = 2240 (36 units of 128 tiles): 4 splits, one
// wave of 144 CTAs and 32 tiles each; 5 splits would take two waves of 26.
int kv_splits(int64_t B, int64_t G, int64_t ntiles) {
  const int64_t units = B * G;
  const int64_t sms = static_cast<int64_t>(kf_host::current_device_sms());
  int64_t best = 1, best_cost = INT64_MAX;
  for (int64_t s = 1; s <= ntiles && s <= 4 * sms; ++s) {
    const int64_t waves = (units * s + sms - 1) / sms;
    const int64_t cost = waves * ((ntiles + s - 1) / s);
    if (cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return static_cast<int>(best);
}

template <typename T>
int launch_proj_attn(const CUtensorMap& tm_x, const CUtensorMap& tm_w, const CUtensorMap& tm_out, const void* qkv_bias,
                     float* partial, int B, int N, int C, float eps, cudaStream_t s) {
  const int H = C / kHd, G = (H + kGroup - 1) / kGroup, ntiles = (N + kTokT - 1) / kTokT;
  const int S = kv_splits(B, G, ntiles);
  const int tps = (ntiles + S - 1) / S;
  const T* bias = static_cast<const T*>(qkv_bias);
  {
    auto k1 = sana_proj_kv<T>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(k1), kPT, KvCfg::kSmemBytes, nullptr);
    if (prep != KF_OK) return prep;
    k1<<<dim3(S, G, B), kPT, KvCfg::kSmemBytes, s>>>(tm_x, tm_w, bias, partial, N, C, H, tps);
    KF_LAUNCH_CHECK();
  }
  {
    auto k2 = sana_proj_qout<T>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(k2), kPT, QoutCfg::kSmemBytes, nullptr);
    if (prep != KF_OK) return prep;
    // Token tiles per CTA: about one CTA per SM over the (batch, head group, tile) items.
    const int64_t items = static_cast<int64_t>(B) * G * ntiles;
    const int64_t sms = kf_host::current_device_sms();
    const int tpc = static_cast<int>(std::min<int64_t>(ntiles, std::max<int64_t>(1, (items + sms - 1) / sms)));
    const int splits2 = (ntiles + tpc - 1) / tpc;
    k2<<<dim3(splits2, G, B), kPT, QoutCfg::kSmemBytes, s>>>(tm_x, tm_w, tm_out, bias, partial, N, C, H, S, tpc,
                                                             eps);
    KF_LAUNCH_CHECK();
  }
  return KF_OK;
}

}  // namespace

KF_API size_t kf_sana_proj_attn_workspace_size(int64_t batch, int64_t seq_len, int64_t channels) {
  if (batch <= 0 || seq_len <= 0 || channels <= 0 || channels % kHd != 0) return 0;
  const int64_t H = channels / kHd, G = (H + kGroup - 1) / kGroup, ntiles = (seq_len + kTokT - 1) / kTokT;
  const int S = kv_splits(batch, G, ntiles);
  return static_cast<size_t>(batch) * H * S * kRowsB * kHd * sizeof(float);
}

KF_API int kf_sana_proj_attn_fwd(const void* x, const void* qkv_weight, const void* qkv_bias, void* out,
                                 void* workspace, size_t workspace_bytes, int64_t batch, int64_t seq_len,
                                 int64_t channels, float eps, int dtype, void* stream) {
  // bf16 only (as the reference's grouped kernels): fp16 would need the power-of-two scaling of
  // [K^T V ; ksum] that the attention kernels apply to keep the B halves in fp16's range.
  if (dtype != KF_DTYPE_BF16) return KF_ERR_UNSUPPORTED;
  if (batch <= 0 || seq_len <= 0 || channels <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (channels % kHd != 0 || channels < 64) return KF_ERR_UNSUPPORTED;
  if (x == nullptr || qkv_weight == nullptr || out == nullptr || workspace == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || seq_len >= (int64_t(1) << 30) || channels >= (int64_t(1) << 20)) return KF_ERR_UNSUPPORTED;
  if (workspace_bytes < kf_sana_proj_attn_workspace_size(batch, seq_len, channels)) return KF_ERR_WORKSPACE;
  if (!kf::aligned(x, 16) || !kf::aligned(qkv_weight, 16) || !kf::aligned(out, 16) || !kf::aligned(workspace, 16) ||
      (qkv_bias != nullptr && !kf::aligned(qkv_bias, 4)))
    return KF_ERR_MISALIGNED;
  const int B = static_cast<int>(batch), N = static_cast<int>(seq_len), C = static_cast<int>(channels);
  const int H = C / kHd, G = (H + kGroup - 1) / kGroup, ntiles = (N + kTokT - 1) / kTokT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const CUtensorMapDataType type = kf_host::map_type(dtype);
  // x [B, N, C] as (channel, token, batch, 1): boxes of 64 channels x 128 tokens, zero past N.
  CUtensorMap tm_x, tm_w, tm_out;
  {
    // out [B, N, C] as (channel, token, batch): stores of 32 channels (one head) x 32 tokens.
    const uint64_t dims[3] = {static_cast<uint64_t>(C), static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
    const uint64_t strides[2] = {static_cast<uint64_t>(C) * 2, static_cast<uint64_t>(N) * C * 2};
    const uint32_t box[3] = {kHd, 32, 1};
    if (!kf_host::encode_tiled(&tm_out, type, 3, out, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B)) return KF_ERR_CUDA;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(C), static_cast<uint64_t>(N), static_cast<uint64_t>(B), 1};
    const uint64_t strides[3] = {static_cast<uint64_t>(C) * 2, static_cast<uint64_t>(N) * C * 2,
                                 static_cast<uint64_t>(B) * N * C * 2};
    const uint32_t box[4] = {kKB, kTokT, 1, 1};
    if (!kf_host::encode_tiled(&tm_x, type, 4, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return KF_ERR_CUDA;
  }
  {
    // W_qkv [3C, C] (nn.Linear layout): boxes of 64 input channels x 128 output rows.
    const uint64_t dims[2] = {static_cast<uint64_t>(C), static_cast<uint64_t>(3 * C)};
    const uint64_t strides[1] = {static_cast<uint64_t>(C) * 2};
    const uint32_t box[2] = {kKB, kGC};
    if (!kf_host::encode_tiled(&tm_w, type, 2, qkv_weight, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return KF_ERR_CUDA;
  }
  float* partial = static_cast<float*>(workspace);
  return launch_proj_attn<__nv_bfloat16>(tm_x, tm_w, tm_out, qkv_bias, partial, B, N, C, eps, s);
}
