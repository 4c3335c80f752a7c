// ABI-level helpers: status strings, version, and the device error words of the modules.
#include "kf_common.cuh"

int kf_internal_sana_error(unsigned int* code);
int kf_internal_fa_error(unsigned int* code);
int kf_internal_fa_bwd_error(unsigned int* code);

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

KF_API int kf_abi_version(void) { return 1; }

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
  return KF_OK;
}
