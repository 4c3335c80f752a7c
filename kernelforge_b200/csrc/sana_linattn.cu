// SANA ReLU linear attention over packed QKV for sm_100a.
//
// Computes LiteLA.attn_matmul (SANA_LinearAttention/original.py:99-117) as the reference's
// split-sequence kernels do (SANA_LinearAttention/custom.py:98-388), in two launches:
//
//  1. sana_vk_producer   grid (splits, head groups, batch)
//     Each CTA streams its token range of K and V for G heads through a TMA/mbarrier ring
//     (SWIZZLE_128B boxes of 64 tokens x 2 heads) and accumulates, per head (one warp),
//         VK[r][c] += v[t][r] * relu(k[t][c])      (mma.sync m16n8k16, fp32 accumulators)
//         ksum[c]  += relu(k[t][c])                (fp32, from the same B fragments)
//     It writes fp32 partials; the last CTA to finish a (batch, head group) -- an atomic
//     arrival counter, no waiting -- sums the partials in split order (deterministic) into the
//     final VK/ksum and resets the counter for the next call.
//  2. sana_out_epilogue  grid (token tiles, head groups, batch)
//     out[t][r] = (VK relu(q_t))_r / (ksum . relu(q_t) + eps). VK and ksum are split into
//     hi + lo 16-bit halves (two MMAs) so the epilogue keeps ~16 mantissa bits of the fp32
//     sums; ksum is the 33rd row of the B operand, like the reference's ones-row padding.
//     The output tile is staged in shared memory and written with a TMA store.
//
// Intensity is ~16 flop/byte: the path is HBM-bound, K/V are read once by (1), Q read once
// and out written once by (2). d = 32 is below tcgen05's minimum M (64), so the tensor work
// uses the warp-level MMA; at the measured rates it is far from the bound.
// Shapes outside the fast path (fp32 input, head dims other than 32, tiny tensors) run the
// generic kernels below (same workspace protocol, CUDA-core fp32 arithmetic).
#include "kf_sm100.cuh"

#include <algorithm>
#include <type_traits>

namespace {

__device__ unsigned int g_sana_error = 0;

constexpr int kD = 32;                 // fast-path head dim
constexpr int kTok = 64;               // tokens per tile / TMA box
constexpr int kBoxBytes = kTok * 128;  // 64 tokens x 128 bytes
constexpr int kRows = kD + 1;          // 32 VK rows + the ksum row
constexpr int kMaxG = 4;

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

constexpr int kMaxClusterSplits = 8;  // portable thread-block cluster size

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

// Fast path: the splits of a (batch, head pair) form one cluster (<= 8 CTAs). Default: about
// two producer CTAs per SM.
constexpr int kFastHeads = 2;
int fast_splits(int64_t B, int64_t H, int64_t N, int64_t requested) {
  const int64_t tiles = std::max<int64_t>(1, ceil_div(N, kTok));
  int64_t s = requested;
  if (s <= 0) {
    const int64_t units = B * ceil_div(H, kFastHeads);
    const int64_t target = static_cast<int64_t>(kf_host::current_device_sms()) * 2;
    s = (target + units / 2) / std::max<int64_t>(units, 1);
  }
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({s, tiles, kMaxClusterSplits})));
}

struct WorkspaceLayout {
  size_t partial_off, final_off, counter_off, total;
};
size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// [partials: B*H*S*(d+1)*d fp32 | final: B*H*(d+1)*d fp32 | counters: B*H u32]. The fast path
// uses only `final`; the generic path uses all three.
WorkspaceLayout layout_for(int64_t B, int64_t H, int64_t d, int64_t S) {
  WorkspaceLayout l;
  const size_t per_head = static_cast<size_t>(d + 1) * d;
  l.partial_off = 0;
  l.final_off = align256(static_cast<size_t>(B * H * S) * per_head * sizeof(float));
  l.counter_off = l.final_off + align256(static_cast<size_t>(B * H) * per_head * sizeof(float));
  l.total = l.counter_off + align256(static_cast<size_t>(B * H) * sizeof(unsigned int));
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
// Fast path, kernel 1: K^T V and ksum per split; the S splits of a (batch, head group) are one
// thread-block cluster and reduce their partials through distributed shared memory.
// ------------------------------------------------------------------------------------------
template <typename T, int G, int STAGES>
__global__ void __launch_bounds__(G * 32)
sana_vk_producer(const __grid_constant__ CUtensorMap qkv_map, float* __restrict__ final_vk, int H,
                 int tiles, int tiles_per_split) {
  constexpr int kThreads = G * 32;
  constexpr int kPairs = G / 2;
  constexpr int kStageBytes = 2 * kPairs * kBoxBytes;  // K boxes, then V boxes
  constexpr int kHeadElems = kRows * kD;
  static_assert(STAGES * kStageBytes >= G * kHeadElems * 4, "reduction buffer must fit the stages");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);

  const int split = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x;  // == cluster size
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
  // Partials of this split -> own shared memory (the stage ring is idle: every issued load
  // was waited for). After a timeout the ring may still be written by TMA: leave it alone.
  float* red = reinterpret_cast<float*>(smem);
  if (!aborted) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 1);
      ksum[nt] += __shfl_xor_sync(0xffffffffu, ksum[nt], 2);
    }
    float* dst = red + warp * kHeadElems;
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
  // Every CTA of the cluster reaches both cluster barriers, also after a timeout, so no CTA can
  // wait for one that has left.
  __syncthreads();
  kf::cluster_sync_all();
  if (!aborted) {
    // CTA `rank` sums its slice of the G heads' elements over the S splits, in split order.
    constexpr int kTotal = G * kHeadElems;
    const int per = (kTotal + S - 1) / S;
    const int rank = static_cast<int>(kf::cluster_ctarank());
    const int e_end = min(kTotal, (rank + 1) * per);
    const uint32_t red_addr = kf::smem_u32(red);
    for (int e = rank * per + threadIdx.x; e < e_end; e += kThreads) {
      // Issue all remote loads first, then add in split order (deterministic).
      float part[kMaxClusterSplits];
#pragma unroll
      for (int r = 0; r < kMaxClusterSplits; ++r)
        part[r] = r < S ? kf::ld_shared_cluster_f32(kf::mapa_shared(red_addr + e * 4, r)) : 0.f;
      float sum = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxClusterSplits; ++r) sum += part[r];
      const int h = h0 + e / kHeadElems;
      if (h < H) final_vk[(static_cast<size_t>(b) * H + h) * kHeadElems + e % kHeadElems] = sum;
    }
  }
  kf::cluster_sync_all();  // shared memory stays alive until every remote read is done
}

// ------------------------------------------------------------------------------------------
// Fast path, kernel 2: normalised output. Persistent CTAs walk a contiguous range of
// (batch, head group, 64-token tile) items with a two-deep TMA load / store ring.
// ------------------------------------------------------------------------------------------
template <typename T, typename O, int G>
__global__ void __launch_bounds__(G * 32)
sana_out_epilogue(const __grid_constant__ CUtensorMap qkv_map,
                  const __grid_constant__ CUtensorMap out_map, const float* __restrict__ final_vk,
                  int H, int C, int head_groups, int tiles_out, int total_items, int items_per_cta,
                  float eps) {
  constexpr int kPairs = G / 2;
  constexpr int kQBytes = kPairs * kBoxBytes;
  constexpr int kOutBoxes = (G * kD * static_cast<int>(sizeof(O))) / 128;
  constexpr int kOutBytes = kOutBoxes * kBoxBytes;
  constexpr int kChPerBox = 128 / static_cast<int>(sizeof(O));
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* qbuf[2] = {smem, smem + kQBytes};
  uint8_t* obuf[2] = {smem + 2 * kQBytes, smem + 2 * kQBytes + kOutBytes};
  float* vk_s = reinterpret_cast<float*>(smem + 2 * kQBytes + 2 * kOutBytes);  // G heads x 33 x 32
  __shared__ uint64_t bars[2];
  __shared__ uint64_t vk_bar;

  const int first = blockIdx.x * items_per_cta;
  const int last = min(total_items, first + items_per_cta);
  if (first >= last) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int pair = warp >> 1, g = warp & 1;

  auto issue = [&](int item, int buf) {
    const int unit = item / tiles_out, tt = item % tiles_out;
    const int b = unit / head_groups, hg = unit % head_groups;
    kf::mbar_arrive_expect_tx(&bars[buf], kQBytes);
#pragma unroll
    for (int p = 0; p < kPairs; ++p)
      kf::tma_load_4d(qbuf[buf] + p * kBoxBytes, &qkv_map, &bars[buf], (hg * G + 2 * p) * kD, 0,
                      tt * kTok, b);
  };
  if (threadIdx.x == 0) {
    kf::prefetch_tensormap(&qkv_map);
    kf::prefetch_tensormap(&out_map);
    kf::mbar_init(&bars[0], 1);
    kf::mbar_init(&bars[1], 1);
    kf::mbar_init(&vk_bar, 1);
    kf::fence_mbar_init();
    issue(first, 0);
    if (first + 1 < last) issue(first + 1, 1);
  }
  __syncthreads();
  // Q does not depend on the producer; K^T V does: wait for the producer grid from here on.
  kf::pdl_wait_primary();
  uint32_t vk_phase = 0;

  // B operand: VK^T (K = q channel, N = output row) as hi/lo halves; n-tile 4 row 0 = ksum.
  uint32_t bhi[2][5][2], blo[2][5][2];
  float eps_scaled = eps;
  int cur_unit = -1;
  for (int it = first, i = 0; it < last; ++it, ++i) {
    const int unit = it / tiles_out, tt = it % tiles_out;
    const int b = unit / head_groups, hg = unit % head_groups;
    const int h0 = hg * G;
    if (unit != cur_unit) {
      cur_unit = unit;
      const int nheads = min(G, H - h0);
      if (threadIdx.x == 0) {
        const uint32_t bytes = static_cast<uint32_t>(nheads * kRows * kD * sizeof(float));
        kf::mbar_arrive_expect_tx(&vk_bar, bytes);
        kf::bulk_load(vk_s, final_vk + (static_cast<size_t>(b) * H + h0) * kRows * kD, bytes, &vk_bar);
      }
      const bool vk_ok = kf::mbar_wait_bounded(&vk_bar, vk_phase, &g_sana_error);
      vk_phase ^= 1u;
      if (!__syncthreads_and(vk_ok)) break;
      const int h = h0 + warp;
      const bool valid = h < H;
      const float* src = vk_s + min(warp, nheads - 1) * kRows * kD;
      float v[2][5][2][2];
      float vmax = 0.f;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
#pragma unroll
        for (int nt = 0; nt < 5; ++nt)
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int r = nt * 8 + gid;
            const int c = ks * 16 + half * 8 + tig * 2;
            float2 x = make_float2(0.f, 0.f);
            if (valid && r <= kD) x = *reinterpret_cast<const float2*>(src + r * kD + c);
            v[ks][nt][half][0] = x.x;
            v[ks][nt][half][1] = x.y;
            vmax = fmaxf(vmax, fmaxf(fabsf(x.x), fabsf(x.y)));
          }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
      const float scale = operand_scale(vmax, std::is_same<T, __half>::value);
      eps_scaled = eps * scale;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
#pragma unroll
        for (int nt = 0; nt < 5; ++nt)
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const float x0 = v[ks][nt][half][0] * scale, x1 = v[ks][nt][half][1] * scale;
            const uint32_t hi = kf::Mma<T>::from_f2(x0, x1);
            const float2 hf = kf::Mma<T>::to_f2(hi);
            bhi[ks][nt][half] = hi;
            blo[ks][nt][half] = kf::Mma<T>::from_f2(x0 - hf.x, x1 - hf.y);
          }
      __syncthreads();  // vk_s is free for the next unit's copy
    }
    const int buf = i & 1;
    if (threadIdx.x == 0 && i >= 2) kf::tma_store_wait_read1();  // store of item i-2 has read obuf[buf]
    const bool ok = kf::mbar_wait_bounded(&bars[buf], (i >> 1) & 1, &g_sana_error);
    if (!__syncthreads_and(ok)) break;

    const uint32_t qbase = kf::smem_u32(qbuf[buf] + pair * kBoxBytes);
    uint8_t* otile = obuf[buf];
#pragma unroll
    for (int mt = 0; mt < kTok / 16; ++mt) {
      uint32_t a[2][4];
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int row = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int chunk = g * 4 + ks * 2 + (lane >> 4);
        kf::ldsm_x4(qbase + kf::swz128(row, chunk), a[ks][0], a[ks][1], a[ks][2], a[ks][3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) a[ks][j] = kf::Mma<T>::relu2(a[ks][j]);
      }
      float acc[5][4];
#pragma unroll
      for (int nt = 0; nt < 5; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
#pragma unroll
        for (int nt = 0; nt < 5; ++nt) {
          kf::Mma<T>::run(acc[nt], a[ks], bhi[ks][nt]);
          kf::Mma<T>::run(acc[nt], a[ks], blo[ks][nt]);
        }
      // Column 32 (n-tile 4, tig 0, first element) holds the denominators of rows gid, gid + 8.
      const float inv0 = __frcp_rn(__shfl_sync(0xffffffffu, acc[4][0], lane & ~3) + eps_scaled);
      const float inv1 = __frcp_rn(__shfl_sync(0xffffffffu, acc[4][2], lane & ~3) + eps_scaled);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int cc = warp * kD + nt * 8 + tig * 2;  // channel within the CTA's G heads
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const int row = mt * 16 + gid + rh * 8;
          const float inv = rh ? inv1 : inv0;
          const float v0 = acc[nt][rh * 2] * inv;
          const float v1 = acc[nt][rh * 2 + 1] * inv;
          const int box = cc / kChPerBox;
          const int colb = (cc % kChPerBox) * static_cast<int>(sizeof(O));
          uint8_t* p = otile + box * kBoxBytes + kf::swz128(row, colb >> 4) + (colb & 15);
          if constexpr (sizeof(O) == 4) {
            *reinterpret_cast<float2*>(p) = make_float2(v0, v1);
          } else {
            *reinterpret_cast<uint32_t*>(p) = kf::Mma<O>::from_f2(v0, v1);
          }
        }
      }
    }
    kf::fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
      for (int box = 0; box < kOutBoxes; ++box) {
        const int c0 = h0 * kD + box * kChPerBox;
        if (c0 < C) kf::tma_store_3d(&out_map, otile + box * kBoxBytes, c0, tt * kTok, b);
      }
      kf::tma_store_commit();
      if (it + 2 < last) issue(it + 2, buf);
    }
  }
  if (threadIdx.x == 0) kf::tma_store_wait_read0();  // smem outlives the stores' reads
}

// ------------------------------------------------------------------------------------------
// Generic path (fp32 input, any head dim dividing 128, small tensors): CUDA-core fp32.
// Split partials go to the workspace; the last CTA of a (batch, head) to arrive -- an atomic
// counter, no waiting -- sums them in split order and resets the counter for the next call.
// ------------------------------------------------------------------------------------------
constexpr int kGenThreads = 256;
constexpr int kGenTok = 32;

template <typename T>
__global__ void __launch_bounds__(kGenThreads)
sana_vk_generic(const T* __restrict__ qkv, float* __restrict__ partial, float* __restrict__ final_vk,
                unsigned int* __restrict__ counters, int H, int d, int N, int tiles_per_split) {
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
        kv = fmaxf(kf::Elem<T>::to_f(row[C]), 0.f);
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

template <typename T, typename O>
__global__ void __launch_bounds__(kGenThreads)
sana_out_generic(const T* __restrict__ qkv, const float* __restrict__ final_vk, O* __restrict__ out,
                 int H, int d, int N, float eps) {
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
    if (tok < N)
      qv = fmaxf(kf::Elem<T>::to_f(qkv[(static_cast<int64_t>(b) * N + tok) * 3 * C + static_cast<int64_t>(h) * d + c]), 0.f);
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
// Host side
// ------------------------------------------------------------------------------------------
constexpr int kFastStages = 3;

template <typename T, int G>
int launch_fast(const void* qkv, void* out, float* final_vk, int B, int H, int N, int S, float eps,
                int out_dtype, cudaStream_t stream) {
  const int C = H * kD;
  const int in_dtype = std::is_same<T, __half>::value ? KF_DTYPE_F16 : KF_DTYPE_BF16;
  const size_t es = 2;
  CUtensorMap qkv_map, out_map;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(C), 3, static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
    const uint64_t strides[3] = {C * es, 3 * C * es, static_cast<uint64_t>(N) * 3 * C * es};
    const uint32_t box[4] = {64, 1, kTok, 1};
    if (!kf_host::encode_tiled(&qkv_map, kf_host::map_type(in_dtype), 4, qkv, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B))
      return KF_ERR_CUDA;
  }
  {
    const size_t os = kf::dtype_size(out_dtype);
    const uint64_t dims[3] = {static_cast<uint64_t>(C), static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
    const uint64_t strides[2] = {C * os, static_cast<uint64_t>(N) * C * os};
    const uint32_t box[3] = {static_cast<uint32_t>(128 / os), kTok, 1};
    if (!kf_host::encode_tiled(&out_map, kf_host::map_type(out_dtype), 3, out, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B))
      return KF_ERR_CUDA;
  }
  const int HG = (H + G - 1) / G;
  const int tiles = (N + kTok - 1) / kTok;
  const int tps = (tiles + S - 1) / S;
  {
    auto kernel = sana_vk_producer<T, G, kFastStages>;
    const int smem = kFastStages * 2 * (G / 2) * kBoxBytes + kFastStages * 8 + 1024;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), G * 32, smem, nullptr);
    if (prep != KF_OK) return prep;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, HG, B);
    cfg.blockDim = dim3(G * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, qkv_map, final_vk, H, tiles, tps));
  }
  auto run = [&](auto kernel, int obytes) -> int {
    const int smem = 2 * (G / 2) * kBoxBytes + 2 * (G * kD * obytes / 128) * kBoxBytes +
                     G * kRows * kD * 4 + 1024;
    int occ = 1;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), G * 32, smem, &occ);
    if (prep != KF_OK) return prep;
    const int total = B * HG * tiles;
    const int grid_cap = kf_host::current_device_sms() * occ;
    const int per = (total + grid_cap - 1) / grid_cap;
    const int grid = (total + per - 1) / per;
    // Programmatic dependent launch: overlaps this grid's prologue with the producer's tail.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(G * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KF_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, qkv_map, out_map, static_cast<const float*>(final_vk), H, C,
                                   HG, tiles, total, per, eps));
    return KF_OK;
  };
  switch (out_dtype) {
    case KF_DTYPE_F32: return run(sana_out_epilogue<T, float, G>, 4);
    case KF_DTYPE_F16: return run(sana_out_epilogue<T, __half, G>, 2);
    default: return run(sana_out_epilogue<T, __nv_bfloat16, G>, 2);
  }
}

template <typename T>
int launch_generic(const void* qkv, void* out, float* partial, float* final_vk,
                   unsigned int* counters, int B, int H, int d, int N, int S, float eps,
                   int out_dtype, cudaStream_t stream) {
  const T* q = static_cast<const T*>(qkv);
  const int nelem = (d + 1) * d;
  const int tiles = (N + kTok - 1) / kTok;
  const int tps = (tiles + S - 1) / S;
  {
    const int smem = (nelem + 2 * kGenTok * d) * static_cast<int>(sizeof(float));
    auto kernel = sana_vk_generic<T>;
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kGenThreads, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<dim3(S, H, B), kGenThreads, smem, stream>>>(q, partial, final_vk, counters, H, d, N, tps);
    KF_LAUNCH_CHECK();
  }
  const int smem = (nelem + kGenTok * d + kGenTok) * static_cast<int>(sizeof(float));
  const dim3 grid((N + kGenTok - 1) / kGenTok, H, B);
  auto run = [&](auto kernel, auto* optr) -> int {
    const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kGenThreads, smem, nullptr);
    if (prep != KF_OK) return prep;
    kernel<<<grid, kGenThreads, smem, stream>>>(q, final_vk, optr, H, d, N, eps);
    KF_LAUNCH_CHECK();
    return KF_OK;
  };
  switch (out_dtype) {
    case KF_DTYPE_F32: return run(sana_out_generic<T, float>, static_cast<float*>(out));
    case KF_DTYPE_F16: return run(sana_out_generic<T, __half>, static_cast<__half*>(out));
    default: return run(sana_out_generic<T, __nv_bfloat16>, static_cast<__nv_bfloat16*>(out));
  }
}

bool valid_head_dim(int64_t d) { return d > 0 && d <= 128 && 128 % d == 0; }

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
  return layout_for(batch, heads, dim, generic_splits(batch, heads, seq_len, splits)).total;
}

KF_API int kf_sana_linattn_fwd(const void* qkv, void* out, void* workspace, size_t workspace_bytes,
                               int64_t batch, int64_t heads, int64_t dim, int64_t seq_len,
                               int64_t splits, float eps, int in_dtype, int out_dtype,
                               void* stream) {
  if (!kf::dtype_valid(in_dtype) || !kf::dtype_valid(out_dtype)) return KF_ERR_UNSUPPORTED;
  if (batch <= 0 || heads <= 0 || seq_len <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (!valid_head_dim(dim)) return KF_ERR_UNSUPPORTED;
  if (qkv == nullptr || out == nullptr || workspace == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return KF_ERR_INVALID_ARGUMENT;
  // TMA coordinates and kernel indices are 32-bit.
  if (batch > 65535 || seq_len > (int64_t(1) << 30) || heads * dim > (int64_t(1) << 24) ||
      batch * seq_len * 3 * heads * dim > (int64_t(1) << 40))
    return KF_ERR_UNSUPPORTED;
  const int S_gen = generic_splits(batch, heads, seq_len, splits);
  const WorkspaceLayout lay = layout_for(batch, heads, dim, S_gen);
  if (workspace_bytes < lay.total) return KF_ERR_WORKSPACE;
  if (!kf::aligned(workspace, 256)) return KF_ERR_MISALIGNED;
  if (!kf::aligned(qkv, kf::dtype_size(in_dtype)) || !kf::aligned(out, kf::dtype_size(out_dtype)))
    return KF_ERR_MISALIGNED;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* partial = reinterpret_cast<float*>(ws + lay.partial_off);
  float* final_vk = reinterpret_cast<float*>(ws + lay.final_off);
  unsigned int* counters = reinterpret_cast<unsigned int*>(ws + lay.counter_off);
  const int B = static_cast<int>(batch), H = static_cast<int>(heads), d = static_cast<int>(dim);
  const int N = static_cast<int>(seq_len);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const bool fast = d == kD && (in_dtype == KF_DTYPE_BF16 || in_dtype == KF_DTYPE_F16) &&
                    H * kD >= 64 && N >= kTok && kf::aligned(qkv, 16) && kf::aligned(out, 16);
  if (fast) {
    // Two heads (one 128-byte TMA box) per CTA measured at or above four heads on every
    // benchmark shape.
    const int S = fast_splits(B, H, N, splits);
    if (in_dtype == KF_DTYPE_BF16)
      return launch_fast<__nv_bfloat16, kFastHeads>(qkv, out, final_vk, B, H, N, S, eps, out_dtype, s);
    return launch_fast<__half, kFastHeads>(qkv, out, final_vk, B, H, N, S, eps, out_dtype, s);
  }
  switch (in_dtype) {
    case KF_DTYPE_F32:
      return launch_generic<float>(qkv, out, partial, final_vk, counters, B, H, d, N, S_gen, eps, out_dtype, s);
    case KF_DTYPE_F16:
      return launch_generic<__half>(qkv, out, partial, final_vk, counters, B, H, d, N, S_gen, eps, out_dtype, s);
    default:
      return launch_generic<__nv_bfloat16>(qkv, out, partial, final_vk, counters, B, H, d, N, S_gen, eps, out_dtype, s);
  }
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

// Device address of the scratch array on the current device. In host code the array's name is
// only a host-side stand-in, so the address comes from cudaGetSymbolAddress, once per device.
int noalloc_scratch(uint8_t** out) {
  static uint8_t* addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return KF_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return KF_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sana_noalloc_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return KF_ERR_CUDA;
    }
    addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = addr[dev];
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
  const size_t per_head = static_cast<size_t>(d + 1) * d * sizeof(float);
  const bool fast = d == kD && (in_dtype == KF_DTYPE_BF16 || in_dtype == KF_DTYPE_F16) &&
                    H * kD >= 64 && N >= kTok && kf::aligned(qkv, 16) && kf::aligned(out, 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (fast) {
    // Only the reduced K^T V / ksum (B*H*33*32 floats) is needed.
    if (static_cast<size_t>(batch) * heads * per_head > kNoAllocScratchBytes) return KF_ERR_WORKSPACE;
    uint8_t* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st != KF_OK) return st;
    float* final_vk = reinterpret_cast<float*>(scratch);
    const int S = fast_splits(B, H, N, splits);
    if (in_dtype == KF_DTYPE_BF16)
      return launch_fast<__nv_bfloat16, kFastHeads>(qkv, out, final_vk, B, H, N, S, eps, out_dtype, s);
    return launch_fast<__half, kFastHeads>(qkv, out, final_vk, B, H, N, S, eps, out_dtype, s);
  }
  // Generic path: as many splits as the default asks for and the scratch holds.
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
      return launch_generic<float>(qkv, out, partial, final_vk, counters, B, H, d, N, S, eps, out_dtype, s);
    case KF_DTYPE_F16:
      return launch_generic<__half>(qkv, out, partial, final_vk, counters, B, H, d, N, S, eps, out_dtype, s);
    default:
      return launch_generic<__nv_bfloat16>(qkv, out, partial, final_vk, counters, B, H, d, N, S, eps, out_dtype, s);
  }
}
