// sm_100a primitives written as inline PTX: mbarriers, TMA (cp.async.bulk.tensor, single-CTA
// copies only), ldmatrix and legacy-shape mma.sync, plus host-side tensor-map encoding
// through the driver entry point (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "kf_common.cuh"

namespace kf {

// ------------------------------------------------------------------------------------------
// Shared-memory addresses and mbarriers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records KF_ERR_DEVICE_TIMEOUT in *err) when the phase has
// not completed within timeout_ns. Every caller of a wait in this project uses this form.
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;  // 4 s: far above any legitimate wait
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0 && globaltimer_ns() - start > kWaitTimeoutNs) {
      atomicCAS(err, 0u, static_cast<unsigned int>(KF_ERR_DEVICE_TIMEOUT));
      return false;
    }
  }
}

// Relaxed-semantics probe of a phase. Threads that keep asynchronous tensor-core or TMA work
// in flight (the MMA issuer, the TMA producer) use it: an acquire-semantics try_wait in such a
// thread stalls its issue for hundreds of cycles even when the phase has long completed.
// Ordering for them comes from the producers of each phase: TMA completes a transaction only
// after its bytes are in shared memory, tcgen05.commit arrives only after the MMAs' reads, and
// the softmax threads run tcgen05.wait::st + tcgen05.fence::before_thread_sync before arriving
// (the consumer issues tcgen05.fence::after_thread_sync after the wait).
__device__ __forceinline__ bool mbar_try_wait_relaxed(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.relaxed.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Probe with acquire semantics at cluster scope: the phase may have been completed by arrivals
// from other CTAs of the cluster, whose writes the waiter then reads.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait that also gives up as soon as another thread of the CTA has set *abort (a
// shared-memory flag), so a CTA whose roles synchronise with each other never waits out one
// timeout per remaining step after the first failure. A timeout sets *abort itself.
// kPoll: probe with test_wait (no suspension) instead of try_wait.
template <bool kRelaxed = false, bool kPoll = false>
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, unsigned int* err,
                                                   volatile int* abort) {
  auto probe = [&]() {
    return kPoll ? mbar_test_wait(bar, parity)
                 : (kRelaxed ? mbar_try_wait_relaxed(bar, parity) : mbar_try_wait(bar, parity));
  };
  if (probe()) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (probe()) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - start > kWaitTimeoutNs) {
        atomicCAS(err, 0u, static_cast<unsigned int>(KF_ERR_DEVICE_TIMEOUT));
        *abort = 1;
        return false;
      }
    }
  }
}

// mbar_wait_or_abort for a phase that other CTAs of the cluster complete (their arrivals
// release their writes): probes with acquire at cluster scope.
__device__ __forceinline__ bool mbar_wait_cluster_or_abort(uint64_t* bar, uint32_t parity, unsigned int* err,
                                                           volatile int* abort) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - start > kWaitTimeoutNs) {
        atomicCAS(err, 0u, static_cast<unsigned int>(KF_ERR_DEVICE_TIMEOUT));
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------
// Thread-block clusters: distributed shared memory and mbarrier arrivals across CTAs
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Cluster index and cluster count along x (clusters tile the grid in blockIdx order).
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Shared-memory address (shared::cta window) -> the same offset in CTA `rank` of the cluster
// (shared::cluster window).
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// One arrival on an mbarrier of any CTA of the cluster. Release at cluster scope: writes this
// thread made, or saw through a CTA barrier before it, are visible to whoever acquires the phase.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arrival with no ordering of this thread's memory operations (a "done reading" signal whose
// reads have already returned their values).
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 16-byte store into a CTA of the cluster (shared::cluster address) whose completion counts 16
// bytes on that CTA's mbarrier `cluster_mbar`; the waiter of that phase sees the data.
__device__ __forceinline__ void st_async_f4(uint32_t cluster_addr, float4 v, uint32_t cluster_mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   cluster_addr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cluster_mbar)
               : "memory");
}
// Orders this thread's earlier shared-memory writes before its later operations at cluster
// scope (before the CTA barrier that hands them to the thread that arrives remotely).
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}
// Every thread of every CTA of the cluster (each warp converged). Used once, right after the
// mbarriers are initialised and before any CTA waits on anything, so every thread reaches it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32) that use barrier `id` (1..15; 0 is
// __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 f32x2 arithmetic: two lanes of work per instruction)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// ------------------------------------------------------------------------------------------
// TMA (tensor copies through the async proxy). Every load here is a plain single-CTA copy.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_all0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Tensor reduction shared -> global through TMA: the box at (c0, c1) of the 2-D fp32 map gets the
// shared tile added to it, at L2. Completion is tracked by the issuing thread's bulk group
// (tma_store_wait_read0 before the tile's shared memory is rewritten).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}

// Programmatic dependent launch: the primary grid lets its dependent grid start launching;
// the dependent waits for the primary's completion (and memory) before consuming its output.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Byte offset of 16-byte chunk `chunk` in row `row` of a tile written by TMA with
// CU_TENSOR_MAP_SWIZZLE_128B (rows of 128 bytes, tile base 1024-byte aligned).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + (((chunk ^ (row & 7u)) & 7u) << 4);
}

// ------------------------------------------------------------------------------------------
// ldmatrix / mma.sync (m16n8k16, fp32 accumulate)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float* d, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  static __device__ __forceinline__ uint32_t relu2(uint32_t v) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&v);
    x = __hmax2(x, __float2bfloat162_rn(0.f));
    return *reinterpret_cast<uint32_t*>(&x);
  }
  static __device__ __forceinline__ float2 to_f2(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  // Exactly rounded (round to nearest even) products of two packed pairs.
  static __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    __nv_bfloat162 x = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&x);
  }
};
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float* d, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  static __device__ __forceinline__ uint32_t relu2(uint32_t v) {
    __half2 x = *reinterpret_cast<__half2*>(&v);
    x = __hmax2(x, __float2half2_rn(0.f));
    return *reinterpret_cast<uint32_t*>(&x);
  }
  static __device__ __forceinline__ float2 to_f2(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2*>(&v));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    __half2 x = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&x);
  }
};

}  // namespace kf

// ------------------------------------------------------------------------------------------
// Host: tensor-map encoding through the driver entry point.
// ------------------------------------------------------------------------------------------
namespace kf_host {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Encodes a tiled map. dims/strides are innermost-first; strides are in bytes for dims 1..
inline bool encode_tiled(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank,
                         const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                         const uint32_t* box, CUtensorMapSwizzle swizzle) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return false;
  uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, rank, const_cast<void*>(base), dims, strides_bytes, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline CUtensorMapDataType map_type(int dtype) {
  switch (dtype) {
    case KF_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    case KF_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  }
}

// Per-device cache of kernel preparation. The dynamic shared-memory opt-in is a per-function
// attribute: it is only ever raised (to the largest size requested so far), so launches of the
// same kernel with different sizes stay valid. Occupancy is cached per (function, size). The
// runtime queries cost microseconds; each is done once.
struct KernelPrep {
  const void* fn = nullptr;
  int smem = -1;       // occupancy entries: size; attribute entries: largest opt-in so far
  int occupancy = 0;
};
// CTAs per SM of a kernel that allocates `tmem_cols` tensor-memory columns per CTA. The
// runtime's occupancy query assumes such a kernel may hold all 512 columns and answers 1; here
// the limits are shared memory, registers, threads and the columns the kernel allocates.
inline int tmem_kernel_occupancy(const void* fn, int threads, int smem, int tmem_cols) {
  cudaFuncAttributes a{};
  int dev = 0, smem_sm = 0, reserved = 0, regs_sm = 0, threads_sm = 0;
  if (cudaFuncGetAttributes(&a, fn) != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  const int warps = (threads + 31) / 32;
  const int regs_per_warp = (a.numRegs * 32 + 255) / 256 * 256;  // allocation unit: 256 registers
  int occ = 512 / tmem_cols;
  occ = std::min(occ, smem_sm / (smem + static_cast<int>(a.sharedSizeBytes) + reserved));
  if (regs_per_warp > 0) occ = std::min(occ, regs_sm / (regs_per_warp * warps));
  occ = std::min(occ, threads_sm / threads);
  return std::max(occ, 1);
}

// Id of the CUDA context current on this thread (cuCtxGetId), or 0 when none is current or it
// was destroyed (cudaDeviceReset). Ids are unique for the life of the process, so state that
// belongs to a context (function attributes, module symbol addresses) can be cached under it.
inline unsigned long long context_id() {
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetId fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<GetId>(nullptr);
    }
    return reinterpret_cast<GetId>(p);
  }();
  unsigned long long id = 0;
  if (fn == nullptr || fn(nullptr, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Opt the kernel in to `smem` bytes of dynamic shared memory (cached per device and context:
// a new context, after a cudaDeviceReset, starts without the opt-ins) and, when asked, report
// how many CTAs of it fit on an SM (a property of the device, cached per device). tmem_cols > 0:
// the kernel allocates that many tensor-memory columns per CTA.
inline int prepare_kernel(const void* fn, int threads, int smem, int* occupancy_out, int tmem_cols = 0) {
  constexpr int kSlots = 256;
  static KernelPrep attr_cache[64][kSlots];
  static unsigned long long attr_ctx[64] = {};
  static KernelPrep occ_cache[64][kSlots];
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return KF_ERR_CUDA;
  }
  bool cached_dev = dev >= 0 && dev < 64;
  if (cached_dev) {
    const unsigned long long ctx = context_id();
    if (ctx == 0) {
      cached_dev = false;  // no context yet: the runtime creates one on the calls below
    } else if (attr_ctx[dev] != ctx) {
      for (int i = 0; i < kSlots; ++i) attr_cache[dev][i] = KernelPrep{};
      attr_ctx[dev] = ctx;
    }
  }
  // 1. shared-memory opt-in
  KernelPrep* attr = nullptr;
  if (cached_dev) {
    for (int i = 0; i < kSlots; ++i) {
      KernelPrep& c = attr_cache[dev][i];
      if (c.fn == fn || c.fn == nullptr) {
        attr = &c;
        break;
      }
    }
  }
  if (attr == nullptr || attr->fn == nullptr || attr->smem < smem) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      return KF_ERR_CUDA;
    }
    // Kernels with large tiles want every CTA slot the shared memory allows: ask for the
    // largest shared-memory carveout (the default may keep a bigger L1 and fit fewer CTAs).
    if (smem >= (64 << 10) &&
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                             static_cast<int>(cudaSharedmemCarveoutMaxShared)) != cudaSuccess) {
      (void)cudaGetLastError();
      return KF_ERR_CUDA;
    }
    if (attr != nullptr) {
      attr->smem = smem;
      attr->fn = fn;
    }
  }
  // 2. occupancy for this size
  if (occupancy_out == nullptr) return KF_OK;
  KernelPrep* occ_slot = nullptr;
  if (cached_dev) {
    for (int i = 0; i < kSlots; ++i) {
      KernelPrep& c = occ_cache[dev][i];
      if (c.fn == fn && c.smem == smem) {
        *occupancy_out = c.occupancy;
        return KF_OK;
      }
      if (c.fn == nullptr) {
        occ_slot = &c;
        break;
      }
    }
  }
  int occ = 0;
  if (tmem_cols > 0) {
    occ = tmem_kernel_occupancy(fn, threads, smem, tmem_cols);
  } else if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem) != cudaSuccess || occ <= 0) {
    (void)cudaGetLastError();
    occ = 1;
  }
  if (occ_slot != nullptr) {
    occ_slot->occupancy = occ;
    occ_slot->smem = smem;
    occ_slot->fn = fn;
  }
  *occupancy_out = occ;
  return KF_OK;
}

inline int current_device_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      sms = 148;
    }
    cache[dev] = sms;
  }
  return cache[dev];
}

}  // namespace kf_host
