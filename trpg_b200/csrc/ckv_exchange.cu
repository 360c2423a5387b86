// Split-KV partials exchanged over peer memory: publish, wait, merge in one
// launch per rank (see the ckv_exchange_* declarations in ckv.h).
//
// Every value travels with the step that wrote it: the publishing rank
// stores each fp32 of its partial as one 8-byte word (value bits, step) into
// every rank's buffer, and a reader polls the words it needs until their
// step field is this step.  An aligned 8-byte store is seen whole or not at
// all, so no fence and no separate flag are needed (the low-latency scheme
// of flagged words).  Words of the previous use of a slot carry step - 2.
//
// Buffer layout (bytes):
//   [0, 256)    header: word 0 = error (1 after a wait gave up), word 1 = the
//               number of steps this buffer's rank has completed;
//   [256, ...)  words [2 slots][world][rows][D + 2] of (fp32 bits, step).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "ckv_common.cuh"

namespace ckv {
namespace {

constexpr size_t kHeader = 256, kData = kHeader;
constexpr int kThreads = 512;

struct ExchangeArgs {
  const float *partial;
  void *bufs[CKV_EXCHANGE_MAX_WORLD];
  void *out;
  long long spin_limit;
  int64_t rows;
  int head_dim, world, rank, phases;
};

__device__ __forceinline__ unsigned long long *slot_words(void *buf, unsigned slot, int r, int world,
                                                          size_t part) {
  return reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(buf) + kData) +
         (size_t(slot) * world + r) * part;
}
__device__ __forceinline__ void store_word(unsigned long long *p, float v, unsigned step) {
  const unsigned long long w = (uint64_t(step) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long load_word(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// The value of word `p` once it carries `step`; false if the wait gave up.
__device__ __forceinline__ bool wait_word(const unsigned long long *p, unsigned step, long long t0,
                                          long long limit, float &v) {
  unsigned long long w = load_word(p);
  while (unsigned(w >> 32) != step) {
    if (clock64() - t0 > limit) return false;
    __nanosleep(20);
    w = load_word(p);
  }
  v = __uint_as_float(unsigned(w));
  return true;
}

template <int DT>
__global__ void __launch_bounds__(kThreads) exchange_kernel(const ExchangeArgs a) {
  __shared__ unsigned s_step;
  const int tid = threadIdx.x;
  const int D = a.head_dim;
  const size_t part = size_t(a.rows) * (D + 2);      // words per rank's partial
  unsigned *hdr = static_cast<unsigned *>(a.bufs[a.rank]);
  if (tid == 0) {
    s_step = *reinterpret_cast<volatile unsigned *>(hdr + 1) + 1u;
  }
  __syncthreads();
  const unsigned step = s_step, slot = step & 1u;

  if (a.phases & 1) {
    // ---- publish: this rank's partial into slot [slot][rank] of every buffer
    for (size_t i = tid; i < part; i += kThreads) {
      const float v = a.partial[i];
      for (int j = 0; j < a.world; ++j) store_word(slot_words(a.bufs[j], slot, a.rank, a.world, part) + i, v, step);
    }
  }

  if (a.phases & 2) {
    // ---- merge once every rank's words of this step have arrived (the rule
    // of combine_kernel, ranks in order)
    const long long limit = a.spin_limit > 0 ? a.spin_limit : (1ll << 31);
    const long long t0 = clock64();
    const unsigned long long *base0 = slot_words(a.bufs[a.rank], slot, 0, a.world, part);
    typename Elem<DT>::T *out = static_cast<typename Elem<DT>::T *>(a.out);
    const int64_t total = a.rows * D;
    bool ok = true;
    for (int64_t idx = tid; idx < total && ok; idx += kThreads) {
      const int64_t row = idx / D;
      const int d = int(idx - row * D);
      const unsigned long long *base = base0 + row * (D + 2);
      float mk[CKV_EXCHANGE_MAX_WORLD], lk[CKV_EXCHANGE_MAX_WORLD], ov[CKV_EXCHANGE_MAX_WORLD];
      float M = -INFINITY;
      for (int k = 0; k < a.world && ok; ++k) {
        ok = wait_word(base + k * part + D, step, t0, limit, mk[k]) &&
             wait_word(base + k * part + D + 1, step, t0, limit, lk[k]) &&
             wait_word(base + k * part + d, step, t0, limit, ov[k]);
        if (ok) M = fmaxf(M, mk[k]);
      }
      if (!ok) break;
      float O = 0.f, L = 0.f;
      if (M != -INFINITY) {
        for (int k = 0; k < a.world; ++k) {
          const float wt = mk[k] == -INFINITY ? 0.f : ex2(mk[k] - M);
          O += wt * ov[k];
          L += wt * lk[k];
        }
      }
      out[row * D + d] = Elem<DT>::from_f32(O / L);
    }
    if (!ok) atomicOr(hdr, 1u);
    __syncthreads();
    if (tid == 0) *reinterpret_cast<volatile unsigned *>(hdr + 1) = step;
  }
}

bool al(const void *p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" size_t ckv_exchange_bytes(int world, int64_t rows, int head_dim) {
  if (world < 1 || world > CKV_EXCHANGE_MAX_WORLD || rows < 1 || head_dim < 2 || head_dim > 1024 ||
      head_dim % 2)
    return 0;
  const size_t b = kData + 2 * size_t(world) * size_t(rows) * size_t(head_dim + 2) * 8;
  return (b + 255) / 256 * 256;
}

extern "C" int ckv_exchange_alloc(int world, int64_t rows, int head_dim, void **buffer,
                                  unsigned char handle[64]) {
  const size_t n = ckv_exchange_bytes(world, rows, head_dim);
  if (!n || !buffer || !handle) return CKV_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  void *p = nullptr;
  CKV_CUDA_TRY(cudaMalloc(&p, n));
  cudaError_t e = cudaMemset(p, 0, n);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e);
  }
  memcpy(handle, &h, sizeof(h));
  *buffer = p;
  return CKV_OK;
}

extern "C" int ckv_exchange_open(const unsigned char handle[64], void **peer_buffer) {
  if (!handle || !peer_buffer) return CKV_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  CKV_CUDA_TRY(cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess));
  return CKV_OK;
}

extern "C" int ckv_exchange_close(void *peer_buffer) {
  if (!peer_buffer) return CKV_ERR_INVALID;
  CKV_CUDA_TRY(cudaIpcCloseMemHandle(peer_buffer));
  return CKV_OK;
}

extern "C" int ckv_exchange_free(void *buffer) {
  if (!buffer) return CKV_ERR_INVALID;
  CKV_CUDA_TRY(cudaFree(buffer));
  return CKV_OK;
}

extern "C" int ckv_exchange_combine(const float *partial, int64_t rows, int head_dim,
                                    void *const *buffers, int world, int rank, int phases,
                                    long long spin_limit, int dtype, void *out,
                                    ckv_stream_t stream) {
  if (!ckv_exchange_bytes(world, rows, head_dim) || !buffers || rank < 0 || rank >= world ||
      phases < 1 || phases > 3 || spin_limit < 0 || (dtype != CKV_BF16 && dtype != CKV_F16))
    return CKV_ERR_INVALID;
  if ((phases & 1) && (!partial || !al(partial, 4))) return CKV_ERR_INVALID;
  if ((phases & 2) && (!out || !al(out, 2))) return CKV_ERR_INVALID;
  ExchangeArgs a{};
  a.partial = partial;
  for (int j = 0; j < world; ++j) {
    if (!buffers[j] || !al(buffers[j], 256)) return CKV_ERR_INVALID;
    a.bufs[j] = buffers[j];
  }
  a.out = out;
  a.spin_limit = spin_limit;
  a.rows = rows;
  a.head_dim = head_dim;
  a.world = world;
  a.rank = rank;
  a.phases = phases;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CKV_BF16)
    exchange_kernel<CKV_BF16><<<1, kThreads, 0, st>>>(a);
  else
    exchange_kernel<CKV_F16><<<1, kThreads, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

extern "C" int ckv_exchange_error(void *buffer, int *flag, ckv_stream_t stream) {
  if (!buffer || !flag) return CKV_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned v = 0;
  CKV_CUDA_TRY(cudaMemcpyAsync(&v, buffer, sizeof(v), cudaMemcpyDeviceToHost, st));
  CKV_CUDA_TRY(cudaMemsetAsync(buffer, 0, sizeof(unsigned), st));
  CKV_CUDA_TRY(cudaStreamSynchronize(st));
  *flag = int(v);
  return CKV_OK;
}
