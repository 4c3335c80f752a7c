// ABI-level helpers: status strings, version, the device error words of the modules, and a
// self-test of the bounded-wait path.
#include "kf_common.cuh"
#include "kf_sm100.cuh"

int kf_internal_sana_error(unsigned int* code);
int kf_internal_fa_error(unsigned int* code);
int kf_internal_fa_bwd_error(unsigned int* code);
int kf_internal_linear_error(unsigned int* code);
int kf_internal_proj_attn_error(unsigned int* code);

KF_API const char* kf_status_string(int status) {
  switch (status) {
    case KF_OK: return "ok";
    case KF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case KF_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case KF_ERR_MISALIGNED: return "misaligned pointer or stride";
    case KF_ERR_WORKSPACE: return "workspace missing or too small";
    case KF_ERR_CUDA: return "CUDA runtime or launch error";
    case KF_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired";
    default: return "unknown status";
  }
}

KF_API int kf_abi_version(void) { return 2; }  // 2: kf_fa_bwd takes `deterministic`

namespace {

__device__ unsigned int g_selftest_error = 0;

// One warp waits on an mbarrier that nothing ever arrives on, through the same bounded wait the
// kernels use: it gives up after kf::kWaitTimeoutNs, records KF_ERR_DEVICE_TIMEOUT and returns.
__global__ void selftest_bounded_wait_kernel() {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    kf::mbar_init(&bar, 1);
    kf::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)kf::mbar_wait_bounded(&bar, 0, &g_selftest_error);
}

int selftest_error(unsigned int* code) {
  unsigned int v = 0;
  KF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_selftest_error, sizeof(v)));
  if (v != 0) {
    const unsigned int zero = 0;
    KF_CUDA_TRY(cudaMemcpyToSymbol(g_selftest_error, &zero, sizeof(zero)));
  }
  *code = v;
  return KF_OK;
}

}  // namespace

KF_API int kf_selftest_bounded_wait(void* stream) {
  selftest_bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  KF_LAUNCH_CHECK();
  return KF_OK;
}

KF_API int kf_query_device_error(void* stream, int* code) {
  if (code == nullptr) return KF_ERR_INVALID_ARGUMENT;
  *code = KF_OK;
  KF_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  unsigned int sana = 0;
  int st = kf_internal_sana_error(&sana);
  if (st != KF_OK) return st;
  if (sana != 0 && *code == KF_OK) *code = static_cast<int>(sana);
  unsigned int fa = 0;
  st = kf_internal_fa_error(&fa);
  if (st != KF_OK) return st;
  if (fa != 0 && *code == KF_OK) *code = static_cast<int>(fa);
  unsigned int fa_bwd = 0;
  st = kf_internal_fa_bwd_error(&fa_bwd);
  if (st != KF_OK) return st;
  if (fa_bwd != 0 && *code == KF_OK) *code = static_cast<int>(fa_bwd);
  unsigned int linear = 0;
  st = kf_internal_linear_error(&linear);
  if (st != KF_OK) return st;
  if (linear != 0 && *code == KF_OK) *code = static_cast<int>(linear);
  unsigned int proj_attn = 0;
  st = kf_internal_proj_attn_error(&proj_attn);
  if (st != KF_OK) return st;
  if (proj_attn != 0 && *code == KF_OK) *code = static_cast<int>(proj_attn);
  unsigned int self = 0;
  st = selftest_error(&self);
  if (st != KF_OK) return st;
  if (self != 0 && *code == KF_OK) *code = static_cast<int>(self);
  return KF_OK;
}
