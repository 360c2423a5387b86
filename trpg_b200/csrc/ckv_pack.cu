// Quantize-on-append and dequantize kernels for the compressed KV cache.
//
// Arithmetic follows models/quantized_kv.py:19-25 (CPU quantizer: IEEE
// division, round half to even) and models/quantized_kv_kernels.py:11-21
// (Triton kernel: the same with floor(t + 0.5)); both are selectable.  All
// divisions are correctly rounded (__fdiv_rn) and no multiply-add is
// contracted, so results are bit-identical to the CPU reference.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ckv_common.cuh"

namespace ckv {
namespace {

template <int BITS>
__device__ __forceinline__ uint32_t quantize(float x, float low, float scale, int rounding) {
  constexpr float kMax = float((1 << BITS) - 1);
  float t = __fdiv_rn(__fsub_rn(x, low), scale);
  float r = rounding == CKV_ROUND_HALF_EVEN ? rintf(t) : floorf(__fadd_rn(t, 0.5f));
  r = fminf(fmaxf(r, 0.0f), kMax);
  return static_cast<uint32_t>(r);
}

template <int BITS>
__device__ __forceinline__ float group_scale(float mn, float mx) {
  return fmaxf(__fdiv_rn(__fsub_rn(mx, mn), float((1 << BITS) - 1)), 1e-8f);
}

// One thread per row of G contiguous 16-bit values.
template <int DT, int BITS, int G>
__global__ void __launch_bounds__(128) pack_rows_kernel(const typename Elem<DT>::T *__restrict__ x,
                                                        int64_t rows, int rounding,
                                                        uint8_t *__restrict__ codes,
                                                        float *__restrict__ meta) {
  using E = Elem<DT>;
  int64_t row = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const uint4 *src = reinterpret_cast<const uint4 *>(x + row * G);
  float v[G];
#pragma unroll
  for (int i = 0; i < G / 8; ++i) {
    uint4 w = src[i];
    const typename E::T *h = reinterpret_cast<const typename E::T *>(&w);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i * 8 + j] = E::to_f32(h[j]);
  }
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < G; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
  float scale = group_scale<BITS>(mn, mx);
  constexpr int OUTB = G * BITS / 8;
  uint4 *dst = reinterpret_cast<uint4 *>(codes + row * OUTB);
#pragma unroll
  for (int i = 0; i < OUTB / 16; ++i) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t word = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        int byte = i * 16 + k * 4 + b;
        uint32_t val;
        if constexpr (BITS == 8) {
          val = quantize<8>(v[byte], mn, scale, rounding);
        } else {
          val = quantize<4>(v[2 * byte], mn, scale, rounding) |
                (quantize<4>(v[2 * byte + 1], mn, scale, rounding) << 4);
        }
        word |= val << (8 * b);
      }
      w[k] = word;
    }
    dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  reinterpret_cast<float2 *>(meta)[row] = make_float2(scale, mn);
}

template <int DT, int BITS, int G>
__global__ void __launch_bounds__(256) unpack_rows_kernel(const uint8_t *__restrict__ codes,
                                                          const float *__restrict__ meta,
                                                          int64_t total,
                                                          typename Elem<DT>::T *__restrict__ out) {
  using E = Elem<DT>;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int64_t row = i / G;
  int col = int(i - row * G);
  uint32_t code;
  if constexpr (BITS == 8) {
    code = codes[i];
  } else {
    code = (codes[row * (G / 2) + col / 2] >> ((col & 1) * 4)) & 15u;
  }
  float2 m = reinterpret_cast<const float2 *>(meta)[row];
  out[i] = E::from_f32(__fmaf_rn(float(code), m.x, m.y));
}

// Direct-to-slab append.  Grid: (blocks of 128 tokens x D/32 slices, heads);
// block 256 threads.  Slice s of a block covers
//   keys:   channels 32s..32s+31 over the block's 128 tokens -- thread
//           (channel c = tid % 32, part = tid / 32) takes tokens 16 part..+15
//           of channel c, the eight parts meet in shared memory for the
//           channel's (min, max), and each part writes its 16 codes;
//   values: the 64 (token, 64-channel group) rows of tokens
//           (128 / (D/32)) s.. of the block -- four threads per row, 16
//           channels each, (min, max) over the four by shuffles.
// Every group's (min, max) is exact whatever the order of the comparisons,
// so the codes match a one-thread-per-group quantizer bit for bit.
template <int DT, int BITS, int D>
__global__ void __launch_bounds__(256) append_kernel(ckv_append_args a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int SLICES = D / 32;
  const int blk = blockIdx.x / SLICES, sl = blockIdx.x % SLICES, h = blockIdx.y, tid = threadIdx.x;
  const int64_t tok0 = int64_t(blk) * 128;
  const int unit = a.unit_offset + blk;
  const T *keys = static_cast<const T *>(a.keys) + h * a.k_stride_head + tok0 * a.k_stride_token;
  const T *values =
      static_cast<const T *>(a.values) + h * a.v_stride_head + tok0 * a.v_stride_token;
  __shared__ float2 part_mm[8][32];

  // ---- keys: 32 channels x 128 tokens -------------------------------------
  {
    const int c = 32 * sl + (tid & 31), part = tid >> 5;
    float v[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) v[t] = E::to_f32(keys[(16 * part + t) * a.k_stride_token + c]);
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int t = 1; t < 16; ++t) {
      mn = fminf(mn, v[t]);
      mx = fmaxf(mx, v[t]);
    }
    part_mm[part][tid & 31] = make_float2(mn, mx);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 m = part_mm[k][tid & 31];
      mn = fminf(mn, m.x);
      mx = fmaxf(mx, m.y);
    }
    const float scale = group_scale<BITS>(mn, mx);
    constexpr int KS = 128 * BITS / 8;   // key bytes per channel row
    uint8_t *row = a.key_data + h * a.kd_stride_head + int64_t(unit) * a.kd_stride_unit + c * KS;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if constexpr (BITS == 8) {
#pragma unroll
      for (int t = 0; t < 16; ++t) w[t >> 2] |= quantize<8>(v[t], mn, scale, a.rounding) << (8 * (t & 3));
      reinterpret_cast<uint4 *>(row)[part] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int t = 0; t < 16; ++t) w[t >> 3] |= quantize<4>(v[t], mn, scale, a.rounding) << (4 * (t & 7));
      reinterpret_cast<uint2 *>(row)[part] = make_uint2(w[0], w[1]);
    }
    if (part == 0) {
      float *m = a.key_meta + h * a.km_stride_head + int64_t(unit) * a.km_stride_unit + c * 2;
      reinterpret_cast<float2 *>(m)[0] = make_float2(scale, mn);
    }
  }

  // ---- values: 64 (token, group) rows, four threads per row ----------------
  {
    constexpr int NG = D / 64;
    constexpr int TPS = 128 / SLICES;     // tokens per slice
    const int rowi = tid >> 2, q = tid & 3;
    const int t = TPS * sl + rowi / NG, g = rowi % NG;
    const uint4 *src = reinterpret_cast<const uint4 *>(values + t * a.v_stride_token + g * 64 + 16 * q);
    float v[16];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 wv = src[i];
      const T *hv = reinterpret_cast<const T *>(&wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * i + j] = E::to_f32(hv[j]);
    }
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      mn = fminf(mn, v[i]);
      mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = group_scale<BITS>(mn, mx);
    const int64_t token = tok0 + t + int64_t(a.unit_offset) * 128;
    constexpr int VB = 64 * BITS / 8;   // value bytes per group
    uint8_t *dst = a.value_data + h * a.vd_stride_head + token * a.vd_stride_token + g * VB;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if constexpr (BITS == 8) {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i >> 2] |= quantize<8>(v[i], mn, scale, a.rounding) << (8 * (i & 3));
      reinterpret_cast<uint4 *>(dst)[q] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i >> 3] |= quantize<4>(v[i], mn, scale, a.rounding) << (4 * (i & 7));
      reinterpret_cast<uint2 *>(dst)[q] = make_uint2(w[0], w[1]);
    }
    if (q == 0) {
      float *m = a.value_meta + h * a.vm_stride_head + token * a.vm_stride_token + g * 2;
      reinterpret_cast<float2 *>(m)[0] = make_float2(scale, mn);
    }
  }
}

// In-place append to the exact window.  Grid: heads x tokens; block: one
// thread per 16-byte piece of a row (D / 8), copying that piece of the key
// row and of the value row.
__global__ void residual_append_kernel(ckv_residual_args a) {
  // Let the next kernel (typically the attention call over this window)
  // launch at once, but finish only after the previous kernel has: the new
  // rows may be its output, and a successor that waits for this kernel then
  // knows the earlier one is done too.
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x / a.tokens, t = blockIdx.x % a.tokens, k = threadIdx.x;
  const uint16_t *kn = static_cast<const uint16_t *>(a.keys_new) + h * a.kn_stride_head + t * a.kn_stride_token;
  const uint16_t *vn = static_cast<const uint16_t *>(a.values_new) + h * a.vn_stride_head + t * a.vn_stride_token;
  uint16_t *kd = static_cast<uint16_t *>(a.keys) + h * a.k_stride_head + int64_t(a.offset + t) * a.k_stride_token;
  uint16_t *vd = static_cast<uint16_t *>(a.values) + h * a.v_stride_head + int64_t(a.offset + t) * a.v_stride_token;
  reinterpret_cast<uint4 *>(kd)[k] = reinterpret_cast<const uint4 *>(kn)[k];
  reinterpret_cast<uint4 *>(vd)[k] = reinterpret_cast<const uint4 *>(vn)[k];
}

bool aligned(const void *p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

template <int DT, int BITS>
int launch_pack_rows(const void *x, int64_t rows, int group, int rounding, uint8_t *codes,
                     float *meta, cudaStream_t s) {
  using T = typename Elem<DT>::T;
  unsigned grid = unsigned((rows + 127) / 128);
  if (group == 128)
    pack_rows_kernel<DT, BITS, 128><<<grid, 128, 0, s>>>(static_cast<const T *>(x), rows, rounding,
                                                          codes, meta);
  else
    pack_rows_kernel<DT, BITS, 64><<<grid, 128, 0, s>>>(static_cast<const T *>(x), rows, rounding,
                                                         codes, meta);
  return cuda_status(cudaGetLastError());
}

template <int DT, int BITS>
int launch_unpack_rows(const uint8_t *codes, const float *meta, int64_t rows, int group, void *out,
                       cudaStream_t s) {
  using T = typename Elem<DT>::T;
  int64_t total = rows * group;
  unsigned grid = unsigned((total + 255) / 256);
  if (group == 128)
    unpack_rows_kernel<DT, BITS, 128><<<grid, 256, 0, s>>>(codes, meta, total, static_cast<T *>(out));
  else
    unpack_rows_kernel<DT, BITS, 64><<<grid, 256, 0, s>>>(codes, meta, total, static_cast<T *>(out));
  return cuda_status(cudaGetLastError());
}

template <int DT, int BITS>
int launch_append(const ckv_append_args &a, cudaStream_t s) {
  dim3 grid(unsigned(a.count / 128 * (a.head_dim / 32)), unsigned(a.heads));
  switch (a.head_dim) {
    case 64: append_kernel<DT, BITS, 64><<<grid, 256, 0, s>>>(a); break;
    case 128: append_kernel<DT, BITS, 128><<<grid, 256, 0, s>>>(a); break;
    case 256: append_kernel<DT, BITS, 256><<<grid, 256, 0, s>>>(a); break;
    default: return CKV_ERR_UNSUPPORTED;
  }
  return cuda_status(cudaGetLastError());
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" int ckv_pack_rows(const void *x, int dtype, int64_t rows, int group, int bits,
                             int rounding, uint8_t *codes, float *meta, ckv_stream_t stream) {
  if (rows < 0 || (group != 64 && group != 128) || (bits != 4 && bits != 8) ||
      (dtype != CKV_BF16 && dtype != CKV_F16) ||
      (rounding != CKV_ROUND_HALF_EVEN && rounding != CKV_ROUND_HALF_UP))
    return CKV_ERR_INVALID;
  if (rows == 0) return CKV_OK;
  if (!x || !codes || !meta || !aligned(x, 16) || !aligned(codes, 16) || !aligned(meta, 8))
    return CKV_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CKV_BF16)
    return bits == 8 ? launch_pack_rows<CKV_BF16, 8>(x, rows, group, rounding, codes, meta, s)
                     : launch_pack_rows<CKV_BF16, 4>(x, rows, group, rounding, codes, meta, s);
  return bits == 8 ? launch_pack_rows<CKV_F16, 8>(x, rows, group, rounding, codes, meta, s)
                   : launch_pack_rows<CKV_F16, 4>(x, rows, group, rounding, codes, meta, s);
}

extern "C" int ckv_unpack_rows(const uint8_t *codes, const float *meta, int64_t rows, int group,
                               int bits, int dtype, void *out, ckv_stream_t stream) {
  if (rows < 0 || (group != 64 && group != 128) || (bits != 4 && bits != 8) ||
      (dtype != CKV_BF16 && dtype != CKV_F16))
    return CKV_ERR_INVALID;
  if (rows == 0) return CKV_OK;
  if (!codes || !meta || !out || !aligned(meta, 8)) return CKV_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CKV_BF16)
    return bits == 8 ? launch_unpack_rows<CKV_BF16, 8>(codes, meta, rows, group, out, s)
                     : launch_unpack_rows<CKV_BF16, 4>(codes, meta, rows, group, out, s);
  return bits == 8 ? launch_unpack_rows<CKV_F16, 8>(codes, meta, rows, group, out, s)
                   : launch_unpack_rows<CKV_F16, 4>(codes, meta, rows, group, out, s);
}

extern "C" int ckv_pack_append(const ckv_append_args *args, ckv_stream_t stream) {
  if (!args) return CKV_ERR_INVALID;
  const ckv_append_args &a = *args;
  if ((a.bits != 4 && a.bits != 8) || (a.dtype != CKV_BF16 && a.dtype != CKV_F16) ||
      (a.rounding != CKV_ROUND_HALF_EVEN && a.rounding != CKV_ROUND_HALF_UP) || a.count < 0 ||
      a.count % 128 || a.heads <= 0 || a.unit_offset < 0)
    return CKV_ERR_INVALID;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return CKV_ERR_UNSUPPORTED;
  if (a.count == 0) return CKV_OK;
  if (!a.keys || !a.values || !a.key_data || !a.key_meta || !a.value_data || !a.value_meta)
    return CKV_ERR_INVALID;
  // 16-byte vector loads of value rows and stores of code rows.
  if (!aligned(a.values, 16) || (a.v_stride_token * 2) % 16 || (a.v_stride_head * 2) % 16 ||
      !aligned(a.key_data, 16) || (a.kd_stride_unit % 16) || (a.kd_stride_head % 16) ||
      !aligned(a.value_data, 16) || (a.vd_stride_token % 16) || (a.vd_stride_head % 16) ||
      !aligned(a.key_meta, 8) || !aligned(a.value_meta, 8) || (a.km_stride_unit % 2) ||
      (a.km_stride_head % 2) || (a.vm_stride_token % 2) || (a.vm_stride_head % 2))
    return CKV_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a.dtype == CKV_BF16)
    return a.bits == 8 ? launch_append<CKV_BF16, 8>(a, s) : launch_append<CKV_BF16, 4>(a, s);
  return a.bits == 8 ? launch_append<CKV_F16, 8>(a, s) : launch_append<CKV_F16, 4>(a, s);
}

extern "C" int ckv_residual_append(const ckv_residual_args *args, ckv_stream_t stream) {
  if (!args) return CKV_ERR_INVALID;
  const ckv_residual_args &a = *args;
  if (a.heads < 1 || a.tokens < 0 || a.offset < 0 || a.head_dim < 8 || a.head_dim % 8 ||
      a.head_dim > 1024)
    return CKV_ERR_INVALID;
  if (a.tokens == 0) return CKV_OK;
  if (!a.keys_new || !a.values_new || !a.keys || !a.values) return CKV_ERR_INVALID;
  if (!aligned(a.keys_new, 16) || !aligned(a.values_new, 16) || !aligned(a.keys, 16) ||
      !aligned(a.values, 16))
    return CKV_ERR_INVALID;
  for (int64_t st : {a.kn_stride_head, a.kn_stride_token, a.vn_stride_head, a.vn_stride_token,
                     a.k_stride_head, a.k_stride_token, a.v_stride_head, a.v_stride_token})
    if (st % 8) return CKV_ERR_INVALID;
  if (int64_t(a.heads) * a.tokens > (int64_t(1) << 31) - 1) return CKV_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(a.heads * a.tokens));
  cfg.blockDim = dim3(unsigned(a.head_dim / 8));
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, residual_append_kernel, a));
  return CKV_OK;
}
