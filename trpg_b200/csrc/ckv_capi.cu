// Status strings, per-thread error text and version of the C ABI.
#include <cuda.h>
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

namespace {
using CtxGetCurrent = CUresult (*)(CUcontext *);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long *);

template <class F>
F driver_fn(const char *name) {
  void *ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(ptr);
}
}  // namespace

unsigned long long context_id() {
  static const CtxGetCurrent get_current = driver_fn<CtxGetCurrent>("cuCtxGetCurrent");
  static const CtxGetId get_id = driver_fn<CtxGetId>("cuCtxGetId");
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
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
