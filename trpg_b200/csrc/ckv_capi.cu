// Status strings, per-thread error text and version of the C ABI.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include "ckv_common.cuh"

namespace ckv {
namespace {
thread_local char g_last_error[256] = {0};
}

void set_last_error(const char *msg) {
  strncpy(g_last_error, msg ? msg : "", sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = 0;
}

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return CKV_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(err),
           cudaGetErrorString(err));
  return CKV_ERR_CUDA;
}
}  // namespace ckv

extern "C" const char *ckv_status_string(int status) {
  switch (status) {
    case CKV_OK: return "ok";
    case CKV_ERR_INVALID: return "invalid argument (pointer, size, stride or alignment)";
    case CKV_ERR_UNSUPPORTED: return "unsupported shape for this build";
    case CKV_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case CKV_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

extern "C" const char *ckv_last_error(void) { return ckv::g_last_error; }

extern "C" int ckv_version(void) { return (1 << 16) | 0; }
