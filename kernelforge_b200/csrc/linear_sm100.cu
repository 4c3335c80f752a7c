// Projection GEMM with a fused bias for sm_100a:
//
//   y[M, N] = x[M, K] W^T (+ bias[N])       x, W, y, bias: fp16 or bf16, fp32 accumulation
//
// the nn.Linear arithmetic of SANA's packed QKV projection (SANA_LinearAttention/custom.py:23-85,
// `_qkv_projection`: x [B*N, C] -> qkv [B*N, 3C], which is the packed [B, N, 3, C] layout the
// attention kernel reads) and of its bias-fused output projection (custom.py:457-523,
// `_output_projection`). W is either nn.Linear's [N, K] (K contiguous) or the reference's
// prepacked WeightT [K, N] (N contiguous); both are tensor-core operands as they lie in memory
// (K-major and MN-major), so no transpose is ever made.
//
// One persistent CTA per SM walks the output tiles (128 rows x BN columns, BN = 256 unless 192
// or 128 saves more than an eighth of N in padding). Warp roles:
//   warp 0      TMA producer: 128 x 64 tiles of x and BN x 64 tiles of W through a ring of
//               shared-memory stages (128-byte swizzle), one mbarrier pair per stage;
//   warp 1      MMA issuer (one thread): four tcgen05.mma kind::f16 M128 N=BN K16 per stage into
//               one of two tensor-memory accumulators, so the epilogue of tile i overlaps the
//               main loop of tile i+1;
//   warps 2-5   epilogue: each warp reads its 32 accumulator lanes (rows) with tcgen05.ld, 32
//               columns at a time, adds the bias in fp32, rounds once to the output dtype, writes
//               the 32 x 32 chunk to shared memory (64-byte swizzle, conflict-free) and stores it
//               with one TMA store (double-buffered per warp; the TMA clips rows past M and
//               columns past N). Per-thread row stores would touch 32 rows per instruction.
// Every wait is bounded (kf::mbar_wait_or_abort): a timeout records KF_ERR_DEVICE_TIMEOUT in
// g_linear_error, the roles leave their loops, the producer waits (bounded) for its copies in
// flight, the MMA thread for its MMAs, and the tensor memory is freed.
//
// fp32 inputs run a CUDA-core kernel with fp32 FMAs (no TF32 rounding), tiled through shared
// memory: correct for any shape, not tuned.
#include "kf_sm100.cuh"
#include "kf_tcgen05.cuh"

#include <type_traits>

namespace {

__device__ unsigned int g_linear_error = 0;

constexpr int kBM = 128;  // x rows per tile = accumulator lanes
constexpr int kBK = 64;   // K elements per stage: one 128-byte swizzle row of 16-bit values
constexpr int kThreads = 192;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;

template <int BN>
struct LinearCfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 192 ? 5 : 6);
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccStride = BN <= 128 ? 128 : 256;  // accumulator b at column b * kAccStride
  static constexpr int kTmemCols = 2 * kAccStride;            // a power of two
  static constexpr int kOutOffset = kStages * kStageBytes;     // 4 warps x 2 buffers x 32 x 32 outputs
  static constexpr int kOutChunkBytes = 32 * 32 * 2;
  static constexpr int kBarOffset = kOutOffset + 4 * 2 * kOutChunkBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // barriers + 1024-byte alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ uint64_t dsw(uint32_t base, uint32_t off, uint32_t lbo) {
  return kf::tc::desc_advance(kf::tc::desc_sw128(base, lbo, 1024), off);
}

template <typename T, int BN, bool kWeightKN>
__global__ void __launch_bounds__(kThreads, 1)
linear_sm100_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_y, const T* __restrict__ bias, int M, int N, int K) {
  using C = LinearCfg<BN>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (kf::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2]: the MMAs of the accumulator's tile are done
  uint64_t* acc_empty = acc_full + 2;       // [2]: the four epilogue warps have read it
  uint64_t* drain = acc_empty + 2;          // the MMA thread's last commit before teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + kBM - 1) / kBM;
  const int tiles = m_tiles * ((N + BN - 1) / BN);
  const int k_steps = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
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
  if (warp == kMmaWarp) kf::tc::tmem_alloc(tmem_slot, C::kTmemCols);
  kf::tc::fence_before_sync();
  __syncthreads();
  kf::tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      kf::prefetch_tensormap(&tm_x);
      kf::prefetch_tensormap(&tm_w);
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mt = t % m_tiles, nt = t / m_tiles;
        for (int ks = 0; ks < k_steps; ++ks) {
          const int s = issued % C::kStages;
          const int use = issued / C::kStages;
          // Stage s is free once the MMAs of its previous use have read it.
          if (use > 0 && !(ok = kf::mbar_wait_or_abort<true>(&empty[s], (use - 1) & 1, &g_linear_error, abort_flag)))
            break;
          uint8_t* a_dst = smem + s * C::kStageBytes;
          uint8_t* b_dst = a_dst + C::kABytes;
          kf::mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          kf::tma_load_2d(a_dst, &tm_x, &full[s], ks * kBK, mt * kBM);
          if (kWeightKN) {
            // W^T [K, N]: BN / 64 boxes of 64 K rows x 64 N values (MN-major operand).
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              kf::tma_load_2d(b_dst + j * 64 * kBK * 2, &tm_w, &full[s], nt * BN + j * 64, ks * kBK);
          } else {
            kf::tma_load_2d(b_dst, &tm_w, &full[s], ks * kBK, nt * BN);  // W [N, K]: K-major
          }
          ++issued;
        }
      }
      // Nothing in flight on exit: the last use of every stage has landed (already true unless a
      // wait gave up).
      for (int i = issued > C::kStages ? issued - C::kStages : 0; i < issued; ++i)
        (void)kf::mbar_wait_bounded(&full[i % C::kStages], (i / C::kStages) & 1, &g_linear_error);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = kf::tc::idesc_f16(kBf16 ? 1 : 0, kBM, BN, false, kWeightKN);
      int consumed = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++local) {
        const int ab = local & 1;
        const int use = local >> 1;
        // The accumulator is free once the epilogue has read tile local-2 out of it.
        if (use > 0 && !(ok = kf::mbar_wait_or_abort<true>(&acc_empty[ab], (use - 1) & 1, &g_linear_error, abort_flag)))
          break;
        kf::tc::fence_after_sync();
        const uint32_t d = tmem + ab * C::kAccStride;
        for (int ks = 0; ks < k_steps; ++ks, ++consumed) {
          const int s = consumed % C::kStages;
          if (!(ok = kf::mbar_wait_or_abort<true>(&full[s], (consumed / C::kStages) & 1, &g_linear_error, abort_flag)))
            break;
          kf::tc::fence_after_sync();
          const uint32_t a = kf::smem_u32(smem + s * C::kStageBytes);
          const uint32_t b = a + C::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // K step of 16: 32 bytes along a K-major row, or 16 rows (2048 bytes) of an MN-major
            // block, whose 64-wide N blocks lie 64 x 128 bytes apart.
            const uint64_t bdesc = kWeightKN ? dsw(b, k * 2048, 64 * kBK * 2) : dsw(b, k * 32, 16);
            kf::tc::mma_ss(d, dsw(a, k * 32, 16), bdesc, idesc, (ks | k) != 0);
          }
          kf::tc::commit(&empty[s]);
        }
        if (!ok) break;
        kf::tc::commit(&acc_full[ab]);
      }
      // No MMA in flight on exit.
      kf::tc::commit(drain);
      (void)kf::mbar_wait_bounded(drain, 0, &g_linear_error);
    }
  } else {
    const int quarter = warp & 3;  // tensor-memory lanes [32 quarter, 32 quarter + 32)
    uint8_t* out_stage = smem + C::kOutOffset + quarter * 2 * C::kOutChunkBytes;
    // Row `lane` of a staged chunk is 64 bytes; 64-byte swizzle: 16-byte piece v sits at
    // v ^ ((lane >> 1) & 3), so each quarter-warp phase of the 16-byte stores hits all 32 banks.
    const uint32_t swz = (lane >> 1) & 3;
    int chunks = 0;  // chunks this warp has stored (buffer chunks & 1)
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int ab = local & 1;
      bool ok = kf::mbar_wait_or_abort(&acc_full[ab], (local >> 1) & 1, &g_linear_error, abort_flag);
      // Warp-uniform outcome: the tcgen05 copies below are .sync.aligned.
      if (!__all_sync(0xffffffffu, ok)) break;
      kf::tc::fence_after_sync();
      const int mt = t % m_tiles, nt = t / m_tiles;
      const int row0 = mt * kBM + quarter * 32;  // first row of this warp's chunks
      const uint32_t acc = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + ab * C::kAccStride;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        const int col0 = nt * BN + cc * 32;
        if (col0 >= N) break;  // warp-uniform
        uint32_t r[32];
        kf::tc::ld_32x32b_x32(acc + cc * 32, r);
        kf::tc::wait_ld();
        if (row0 >= M) continue;  // warp-uniform: the whole chunk lies past the last row
        uint8_t* st = out_stage + (chunks & 1) * C::kOutChunkBytes;
        // The store issued from this buffer two chunks ago has finished reading it.
        if (chunks >= 2 && lane == 0) kf::tma_store_wait_read1();
        __syncwarp();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int c = col0 + v * 8;
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[v * 8 + e]);
          if (bias != nullptr && c < N) {  // N is a multiple of 8
            const uint4 bv = *reinterpret_cast<const uint4*>(bias + c);
            const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 bf = kf::Mma<T>::to_f2(bw[e]);
              f[2 * e] += bf.x;
              f[2 * e + 1] += bf.y;
            }
          }
          uint4 o;
          o.x = kf::Mma<T>::from_f2(f[0], f[1]);
          o.y = kf::Mma<T>::from_f2(f[2], f[3]);
          o.z = kf::Mma<T>::from_f2(f[4], f[5]);
          o.w = kf::Mma<T>::from_f2(f[6], f[7]);
          *reinterpret_cast<uint4*>(st + lane * 64 + ((v ^ swz) << 4)) = o;
        }
        kf::fence_proxy_async_smem();  // the TMA reads the chunk through the async proxy
        __syncwarp();
        if (lane == 0) {
          kf::tma_store_2d(&tm_y, st, col0, row0);
          kf::tma_store_commit();
        }
        ++chunks;
      }
      kf::tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) kf::mbar_arrive(&acc_empty[ab]);
    }
    // Shared memory outlives the stores in flight, and they complete before the kernel ends.
    if (lane == 0) kf::tma_store_wait_all0();
    __syncwarp();
  }
  kf::tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    kf::tc::fence_after_sync();
    kf::tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// fp32: 64 x 64 output tiles, 256 threads with 4 x 4 outputs each, K in steps of 16 through
// shared memory. W is [N, K] or, with kWeightKN, [K, N].
constexpr int kFBM = 64, kFBN = 64, kFBK = 16;
template <bool kWeightKN>
__global__ void __launch_bounds__(256)
linear_f32_kernel(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
                  float* __restrict__ y, int M, int N, int K) {
  __shared__ float xs[kFBK][kFBM + 4];
  __shared__ float ws[kFBK][kFBN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kFBM, n0 = blockIdx.x * kFBN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kFBK) {
    for (int i = threadIdx.x; i < kFBM * kFBK; i += 256) {
      const int r = i / kFBK, kk = i % kFBK;
      const int gm = m0 + r, gk = k0 + kk;
      xs[kk][r] = (gm < M && gk < K) ? x[static_cast<int64_t>(gm) * K + gk] : 0.f;
    }
    for (int i = threadIdx.x; i < kFBN * kFBK; i += 256) {
      int cn, kk;
      if (kWeightKN) {
        kk = i / kFBN;
        cn = i % kFBN;
      } else {
        cn = i / kFBK;
        kk = i % kFBK;
      }
      const int gn = n0 + cn, gk = k0 + kk;
      float v = 0.f;
      if (gn < N && gk < K) v = kWeightKN ? w[static_cast<int64_t>(gk) * N + gn] : w[static_cast<int64_t>(gn) * K + gk];
      ws[kk][cn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kFBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn < N) y[static_cast<int64_t>(gm) * N + gn] = acc[i][j] + (bias != nullptr ? bias[gn] : 0.f);
    }
  }
}

// Output tile width: 256 (measured fastest on the SANA shapes, even padding C = 1152 to 1280)
// unless a narrower tile saves more than an eighth of N in padding.
int pick_bn(int64_t N) {
  auto pad = [&](int bn) { return (N + bn - 1) / bn * bn - N; };
  int best = 256;
  for (int bn : {192, 128})
    if ((pad(best) - pad(bn)) * 8 > N) best = bn;
  return best;
}

template <typename T, int BN, bool kWeightKN>
int launch_tc(const void* x, const void* w, const void* bias, void* y, int M, int N, int K, int dtype,
              cudaStream_t stream) {
  using C = LinearCfg<BN>;
  const CUtensorMapDataType type = kf_host::map_type(dtype);
  CUtensorMap tm_x, tm_w, tm_y;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
    const uint32_t box[2] = {32, 32};
    if (!kf_host::encode_tiled(&tm_y, type, 2, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B)) return KF_ERR_CUDA;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {kBK, kBM};
    if (!kf_host::encode_tiled(&tm_x, type, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return KF_ERR_CUDA;
  }
  if (kWeightKN) {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
    const uint32_t box[2] = {64, kBK};
    if (!kf_host::encode_tiled(&tm_w, type, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return KF_ERR_CUDA;
  } else {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {kBK, static_cast<uint32_t>(BN)};
    if (!kf_host::encode_tiled(&tm_w, type, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return KF_ERR_CUDA;
  }
  auto kernel = linear_sm100_kernel<T, BN, kWeightKN>;
  const int prep = kf_host::prepare_kernel(reinterpret_cast<const void*>(kernel), kThreads, C::kSmemBytes, nullptr);
  if (prep != KF_OK) return prep;
  const int64_t tiles = ((M + kBM - 1) / kBM) * static_cast<int64_t>((N + BN - 1) / BN);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, kf_host::current_device_sms()));
  kernel<<<grid, kThreads, C::kSmemBytes, stream>>>(tm_x, tm_w, tm_y, static_cast<const T*>(bias), M, N, K);
  KF_LAUNCH_CHECK();
  return KF_OK;
}

template <typename T, bool kWeightKN>
int dispatch_bn(const void* x, const void* w, const void* bias, void* y, int M, int N, int K, int dtype,
                cudaStream_t s) {
  switch (pick_bn(N)) {
    case 128: return launch_tc<T, 128, kWeightKN>(x, w, bias, y, M, N, K, dtype, s);
    case 192: return launch_tc<T, 192, kWeightKN>(x, w, bias, y, M, N, K, dtype, s);
    default: return launch_tc<T, 256, kWeightKN>(x, w, bias, y, M, N, K, dtype, s);
  }
}

}  // namespace

int kf_internal_linear_error(unsigned int* code) {
  unsigned int v = 0;
  KF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_linear_error, sizeof(v)));
  if (v != 0) {
    const unsigned int zero = 0;
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_linear_error, &zero, sizeof(zero)));
  }
  *code = v;
  return KF_OK;
}

KF_API int kf_linear_fwd(const void* x, const void* weight, const void* bias, void* y, int64_t rows,
                         int64_t in_features, int64_t out_features, int weight_layout, int dtype, void* stream) {
  if (!kf::dtype_valid(dtype)) return KF_ERR_UNSUPPORTED;
  if (rows < 0 || in_features <= 0 || out_features <= 0) return KF_ERR_INVALID_ARGUMENT;
  if (weight_layout != 0 && weight_layout != 1) return KF_ERR_INVALID_ARGUMENT;
  if (rows == 0) return KF_OK;  // empty input: nothing is read or written
  if (x == nullptr || weight == nullptr || y == nullptr) return KF_ERR_INVALID_ARGUMENT;
  if (rows >= (int64_t(1) << 31) || in_features >= (int64_t(1) << 31) || out_features >= (int64_t(1) << 31))
    return KF_ERR_UNSUPPORTED;
  const int M = static_cast<int>(rows), K = static_cast<int>(in_features), N = static_cast<int>(out_features);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == KF_DTYPE_F32) {
    if (!kf::aligned(x, 4) || !kf::aligned(weight, 4) || !kf::aligned(y, 4) || (bias && !kf::aligned(bias, 4)))
      return KF_ERR_MISALIGNED;
    const dim3 grid((N + kFBN - 1) / kFBN, (M + kFBM - 1) / kFBM);
    if (grid.y > 65535) return KF_ERR_UNSUPPORTED;
    const float* xf = static_cast<const float*>(x);
    const float* wf = static_cast<const float*>(weight);
    const float* bf = static_cast<const float*>(bias);
    if (weight_layout == 1)
      linear_f32_kernel<true><<<grid, 256, 0, s>>>(xf, wf, bf, static_cast<float*>(y), M, N, K);
    else
      linear_f32_kernel<false><<<grid, 256, 0, s>>>(xf, wf, bf, static_cast<float*>(y), M, N, K);
    KF_LAUNCH_CHECK();
    return KF_OK;
  }
  // Tensor-core path: TMA needs 16-byte aligned rows, the epilogue stores 8-element vectors.
  if (K % 8 != 0 || N % 8 != 0) return KF_ERR_UNSUPPORTED;
  if (!kf::aligned(x, 16) || !kf::aligned(weight, 16) || !kf::aligned(y, 16) || (bias && !kf::aligned(bias, 16)))
    return KF_ERR_MISALIGNED;
  if (dtype == KF_DTYPE_BF16)
    return weight_layout == 1 ? dispatch_bn<__nv_bfloat16, true>(x, weight, bias, y, M, N, K, dtype, s)
                              : dispatch_bn<__nv_bfloat16, false>(x, weight, bias, y, M, N, K, dtype, s);
  return weight_layout == 1 ? dispatch_bn<__half, true>(x, weight, bias, y, M, N, K, dtype, s)
                            : dispatch_bn<__half, false>(x, weight, bias, y, M, N, K, dtype, s);
}
