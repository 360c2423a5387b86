// Attention without device allocations, for callers that cannot call
// cudaMalloc (or any allocating routine) at the point of the call.
//
// The split records and tickets that ckv_attention keeps in a caller-supplied
// workspace live here in one file-scope device array instead.  The array is
// part of the library image: every GPU that loads libtrpg_ckv.so holds
// CKV_STATIC_SCRATCH_BYTES of it until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "ckv_common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_scratch[CKV_STATIC_SCRATCH_BYTES];

// Device address of g_scratch in the current device's context.  In host code
// the name g_scratch is only a stand-in for the symbol, never a usable
// pointer, so the address comes from cudaGetSymbolAddress with the device
// current.  It is looked up once per device and context: the context id
// changes after a cudaDeviceReset, which also moves the array, and the next
// call looks it up again.
int scratch_address(void **out) {
  struct Entry {
    unsigned long long ctx;
    void *addr;
  };
  static std::mutex mu;
  static Entry cache[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ckv::cuda_status(e);
  if (dev < 0 || dev >= 64) return CKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long ctx = ckv::context_id();
  if (ctx == 0 || cache[dev].ctx != ctx || !cache[dev].addr) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return ckv::cuda_status(e);
    cache[dev].addr = p;
    cache[dev].ctx = ckv::context_id();   // the lookup made the context current
  }
  *out = cache[dev].addr;
  return CKV_OK;
}

}  // namespace

extern "C" int ckv_attention_static(const ckv_attn_args *args, ckv_stream_t stream) {
  if (!args) return CKV_ERR_INVALID;
  size_t need = 0;
  const int st = ckv_attention_workspace(args, &need);
  if (st != CKV_OK) return st;
  if (need > size_t(CKV_STATIC_SCRATCH_BYTES)) {
    ckv::set_last_error(
        "ckv_attention_static: request needs more scratch than the static buffer holds "
        "(CKV_STATIC_SCRATCH_BYTES); use ckv_attention with a caller workspace");
    return CKV_ERR_WORKSPACE;
  }
  void *ws = nullptr;
  const int sa = scratch_address(&ws);
  if (sa != CKV_OK) return sa;
  // The buffer keeps whatever the previous call left; clearing the ticket
  // region and the give-up word is left to ckv_attention (on the stream,
  // before the kernel) by not claiming they are already zero.
  ckv_attn_args a = *args;
  a.flags &= ~CKV_WS_COUNTERS_ZERO;
  return ckv_attention(&a, ws, size_t(CKV_STATIC_SCRATCH_BYTES), stream);
}

// ckv_attention_error with a NULL workspace: the give-up word of this
// device's static array, as the last ckv_attention_static call on it left it
// (each call clears it before its kernel runs).
int static_scratch_error(int *flag, ckv_stream_t stream) {
  void *ws = nullptr;
  const int sa = scratch_address(&ws);
  if (sa != CKV_OK) return sa;
  unsigned v = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CKV_CUDA_TRY(cudaMemcpyAsync(&v, ws, sizeof(v), cudaMemcpyDeviceToHost, st));
  CKV_CUDA_TRY(cudaStreamSynchronize(st));
  *flag = int(v);
  return CKV_OK;
}
