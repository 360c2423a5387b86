// Split-KV attention kernel, launch planning and C entry points.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <cmath>

#include <cudaTypedefs.h>

#include "ckv_attn.cuh"

namespace ckv {
namespace attn {

// Workspace layout: a 256-byte header (word 0 = error flag), then one ticket
// per (sequence, KV head), then the split records.  Every call leaves the
// tickets at zero.
constexpr int kMaxHeadsKV = 128;
constexpr size_t kCounterOff = 256;
constexpr size_t kCounterBytes = kCounterOff + size_t(CKV_MAX_SEQS) * kMaxHeadsKV * 4;

template <int BITS, int D, int NT, int DT, int MAXS>
__global__ void __launch_bounds__(THREADS, 1) attn_kernel(const __grid_constant__ Params<MAXS> p) {
  using C = Cfg<BITS, D, NT>;
  using T = typename Elem<DT>::T;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int s_seq, s_last;
  __shared__ __align__(8) uint64_t s_bar[WARPS][2];
  // 1024-byte aligned base: the 128-byte TMA swizzle needs aligned slots.
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  if (tid == 0) {
    int lo = 0, hi = p.num_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.seq[mid].cta_begin <= cta) lo = mid; else hi = mid - 1;
    }
    s_seq = lo;
  }
  __syncthreads();
  const int seq = s_seq;
  const SeqDev &sd = p.seq[seq];
  const int local = cta - sd.cta_begin;
  const int head = local / sd.cph, split = local % sd.cph;
  const int G = p.group, rows = p.rows, nq = p.nq;

  // ---- query fragments for both channel orders -----------------------------
  const uint32_t qfp = smem_u32(smem), qfr = qfp + C::QFRAG;
  const uint32_t bar0 = smem_u32(&s_bar[warp][0]), bar1 = smem_u32(&s_bar[warp][1]);
  if (lane == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar1, 1);
    mbar_fence_init();
  }
  {
    const uint16_t *q = static_cast<const uint16_t *>(sd.q);
    for (int x = tid; x < C::KSTEPS * NT * 32; x += THREADS) {
      const int ln = x & 31, nt = (x >> 5) % NT, s = (x >> 5) / NT;
      const int rr = ln >> 2, qq = ln & 3, row = 8 * nt + rr;
      uint2 vp = make_uint2(0, 0), vr = make_uint2(0, 0);
      if (row < rows) {
        const int n = row / G, g = row % G;
        const uint16_t *qrow = q + (head * G + g) * sd.q_h + n * sd.q_n;
        const int cp = 16 * s + qq, cr = 16 * s + 4 * qq;
        vp.x = qrow[cp] | (uint32_t(qrow[cp + 4]) << 16);
        vp.y = qrow[cp + 8] | (uint32_t(qrow[cp + 12]) << 16);
        vr.x = qrow[cr] | (uint32_t(qrow[cr + 1]) << 16);
        vr.y = qrow[cr + 2] | (uint32_t(qrow[cr + 3]) << 16);
      }
      *reinterpret_cast<uint2 *>(smem + x * 8) = vp;
      *reinterpret_cast<uint2 *>(smem + C::QFRAG + x * 8) = vr;
    }
  }
  __syncthreads();

  // ---- this warp's work items ---------------------------------------------
  const int np = sd.ue - sd.ub;
  const int nr = (sd.re - sd.rb + 15) / 16;
  const int ni = np + nr;
  const int ib = int(int64_t(split) * ni / sd.cph);
  const int ie = int(int64_t(split + 1) * ni / sd.cph);
  const int first = ib + warp;
  const int kt = ie > first ? (ie - first + WARPS - 1) / WARPS : 0;
  const int pend = ie < np ? ie : np;
  const int kp = pend > first ? (pend - first + WARPS - 1) / WARPS : 0;
  const int total = kp * C::SPB + (kt - kp) * 2;

  Warp<BITS, D, NT, DT> w;
  w.init(lane, qfp, qfr, qfp + C::QFRAG_AL + warp * C::WARP_BYTES, p.scale_log2);

  const T *rk = static_cast<const T *>(sd.rk) + head * sd.rk_h;
  const T *rv = static_cast<const T *>(sd.rv) + head * sd.rv_h;
  const int length = sd.length, packed = sd.packed;

  auto is_tma = [&](int s) { return s < kp * C::SPB; };
  auto issue = [&](int s) {
    const uint32_t slot = w.ring + (s & 1) * C::SLOT;
    const uint32_t bar = (s & 1) ? bar1 : bar0;
    if (is_tma(s)) {
      const int k = s / C::SPB, part = s % C::SPB;
      const int unit = sd.ub + first + k * WARPS;
      const int qq = part / (1 + C::VSQ), sub = part % (1 + C::VSQ);
      if (sub == 0)
        w.load_packed_k(sd, head, unit, qq, slot, qq == 0, bar);
      else
        w.load_packed_v(sd, head, unit * 128 + qq * C::QT + (sub - 1) * 32, slot, bar);
    } else {
      const int k = (s - kp * C::SPB) >> 1, part = (s - kp * C::SPB) & 1;
      const int t0 = sd.rb + (first + (kp + k) * WARPS - np) * 16;
      if (part == 0)
        w.load_resid(rk, sd.rk_t, t0, sd.re, slot, C::RKP);
      else
        w.load_resid(rv, sd.rv_t, t0, sd.re, slot, C::RVP);
    }
  };

  const int rr = lane >> 2;
  auto compute = [&](int s) {
    const uint32_t slot = w.ring + (s & 1) * C::SLOT;
    if (is_tma(s)) {
      const int part = s % C::SPB;
      const int sub = part % (1 + C::VSQ);
      if (sub == 0) {
        w.qk_packed(slot);
        w.template softmax<C::MTQ>(
            [&](int mt, int h) { return C::TPL * rr + 2 * mt + h; },
            [](int, int) { return true; }, [](int t) { return packed_pos(t); });
      } else {
        w.pv_packed(slot, 2 * (sub - 1));
      }
    } else {
      const int k = (s - kp * C::SPB) >> 1, part = (s - kp * C::SPB) & 1;
      if (part == 0) {
        const int t0 = sd.rb + (first + (kp + k) * WARPS - np) * 16;
        w.qk_resid(slot);
        w.template softmax<1>(
            [&](int, int h) { return rr + 8 * h; },
            [&](int t, int row) {
              const int ri = t0 + t;
              return ri < sd.re && (nq == 1 || packed + ri <= length - nq + row / G);
            },
            [](int t) { return resid_pos<C::CPL>(t); });
      } else {
        w.pv_resid(slot);
      }
    }
  };

  // Every slot commits one cp.async group (empty for TMA slots), so the
  // residual slots can wait with cp.async.wait_group 1; TMA slots wait on
  // their mbarrier phase.
  uint32_t phase = 0;  // bit k: parity of the next completion of ring slot k
  __syncwarp();
  if (total > 0) issue(0);
  cp_async_commit();
  if (total > 1) issue(1);
  cp_async_commit();
  int s = 0;
  for (; s < total; ++s) {
    if (is_tma(s)) {
      const int k = s & 1;
      if (!mbar_wait(k ? bar1 : bar0, (phase >> k) & 1)) {
        if (lane == 0) atomicOr(p.error, 1u);
        break;
      }
      phase ^= 1u << k;
    } else {
      cp_async_wait<1>();
    }
    __syncwarp();
    compute(s);
    __syncwarp();
    if (s + 2 < total) issue(s + 2);
    cp_async_commit();
  }
  if (s < total) {
    // A wait gave up: let the copies still in flight land (bounded) before
    // this CTA's shared memory is reused or released.
    for (int k2 = s; k2 < s + 2 && k2 < total; ++k2)
      if (is_tma(k2)) mbar_wait((k2 & 1) ? bar1 : bar0, (phase >> (k2 & 1)) & 1);
  }
  cp_async_wait<0>();

  // ---- warp -> CTA merge ----------------------------------------------------
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v = w.l[nt][j];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      w.l[nt][j] = v;
    }
  __syncthreads();  // ring memory becomes merge scratch
  constexpr int WR = 8 * NT;  // rows held by a warp
  float *mrg = reinterpret_cast<float *>(smem + C::QFRAG_AL);
  float *ml = mrg + WARPS * WR * D;
  {
    float *mw = mrg + warp * WR * D;
#pragma unroll
    for (int i = 0; i < C::MTV; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int row = 8 * nt + 2 * w.qd + (c & 1);
          mw[row * D + w.out_channel(i, c)] = w.acc[i][nt][c];
        }
    if (w.r == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int row = 8 * nt + 2 * w.qd + j;
          ml[(warp * WR + row) * 2] = w.m[nt][j];
          ml[(warp * WR + row) * 2 + 1] = w.l[nt][j];
        }
    }
  }
  __syncthreads();
  float *rec = p.rec + size_t(cta) * rows * D;
  float *recml = p.rec_ml + size_t(cta) * rows * 2;
  for (int idx = tid; idx < rows * D; idx += THREADS) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < WARPS; ++k) M = fmaxf(M, ml[(k * WR + row) * 2]);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int k = 0; k < WARPS; ++k) {
        const float mk = ml[(k * WR + row) * 2];
        const float wt = mk == -INFINITY ? 0.f : ex2(mk - M);
        O += wt * mrg[(k * WR + row) * D + d];
        L += wt * ml[(k * WR + row) * 2 + 1];
      }
    }
    rec[idx] = O;
    if (d == 0) {
      recml[row * 2] = M;
      recml[row * 2 + 1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[seq * p.hkv + head], 1u);
    s_last = prev == unsigned(sd.cph - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- last CTA of the pair: merge the pair's CTA records -------------------
  // Weights per (row, record) once, then every output element sums its
  // records with many independent 16-byte loads in flight.
  const int c0 = sd.cta_begin + head * sd.cph;
  const int cph = sd.cph;
  float *s_w = reinterpret_cast<float *>(smem + C::QFRAG_AL);  // [rows][cph] m, then weight
  float *s_l = s_w + rows * cph;                                 // [rows][cph] l
  float *s_row = s_l + rows * cph;                               // [rows] (M, L)
  for (int idx = tid; idx < rows * cph; idx += THREADS) {
    const int row = idx / cph, c = idx % cph;
    const float2 ml2 =
        __ldcg(reinterpret_cast<const float2 *>(p.rec_ml) + size_t(c0 + c) * rows + row);
    s_w[row * cph + c] = ml2.x;
    s_l[row * cph + c] = ml2.y;
  }
  __syncthreads();
  for (int row = warp; row < rows; row += WARPS) {
    float M = -INFINITY;
    for (int c = lane; c < cph; c += 32) M = fmaxf(M, s_w[row * cph + c]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int c = lane; c < cph; c += 32) {
      const float m = s_w[row * cph + c];
      const float wt = (m == -INFINITY) ? 0.f : ex2(m - M);
      s_w[row * cph + c] = wt;
      L += wt * s_l[row * cph + c];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) {
      s_row[2 * row] = M;
      s_row[2 * row + 1] = L;
    }
  }
  __syncthreads();
  constexpr int D4 = D / 4;
  const size_t rstride = size_t(rows) * D4;   // float4s per CTA record
  for (int idx = tid; idx < rows * D4; idx += THREADS) {
    const int row = idx / D4, d4 = idx % D4;
    const float4 *src = reinterpret_cast<const float4 *>(p.rec) + size_t(c0) * rstride + row * D4 + d4;
    const float *wr = s_w + row * cph;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int c = 0;
    for (; c + 16 <= cph; c += 16) {
      float4 v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = __ldcg(src + (c + k) * rstride);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float wt = wr[c + k];
        acc.x += wt * v[k].x; acc.y += wt * v[k].y; acc.z += wt * v[k].z; acc.w += wt * v[k].w;
      }
    }
    for (; c < cph; ++c) {
      const float4 v = __ldcg(src + c * rstride);
      const float wt = wr[c];
      acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
    }
    const float M = s_row[2 * row], L = s_row[2 * row + 1];
    const int n = row / G, g = row % G;
    const int64_t orow = int64_t(head * G + g) * nq + n;
    if (p.partial) {
      float *o = static_cast<float *>(sd.out) + orow * (D + 2);
      o[4 * d4] = acc.x; o[4 * d4 + 1] = acc.y; o[4 * d4 + 2] = acc.z; o[4 * d4 + 3] = acc.w;
      if (d4 == 0) {
        o[D] = M;
        o[D + 1] = L;
      }
    } else {
      T *o = static_cast<T *>(sd.out) + orow * D + 4 * d4;
      const float inv = 1.f / L;
      o[0] = Elem<DT>::from_f32(acc.x * inv);
      o[1] = Elem<DT>::from_f32(acc.y * inv);
      o[2] = Elem<DT>::from_f32(acc.z * inv);
      o[3] = Elem<DT>::from_f32(acc.w * inv);
    }
  }
  if (tid == 0) p.counters[seq * p.hkv + head] = 0u;
}

template <int DT>
__global__ void combine_kernel(const float *__restrict__ parts, int nparts, int64_t rows, int D,
                               typename Elem<DT>::T *__restrict__ out) {
  const int64_t row = blockIdx.x;
  const size_t stride = size_t(rows) * (D + 2);
  float M = -INFINITY;
  for (int k = 0; k < nparts; ++k) M = fmaxf(M, parts[k * stride + row * (D + 2) + D]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
      for (int k = 0; k < nparts; ++k) {
        const float *pr = parts + k * stride + row * (D + 2);
        const float wt = pr[D] == -INFINITY ? 0.f : ex2(pr[D] - M);
        O += wt * pr[d];
        L += wt * pr[D + 1];
      }
    }
    out[row * D + d] = Elem<DT>::from_f32(O / L);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct Plan {
  int grid = 0;
  int rows = 0;
  size_t rec_off = 0, ml_off = 0, bytes = 0;
  int cta_begin[CKV_MAX_SEQS];
  int cph[CKV_MAX_SEQS];
};

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && (sms = cache[dev].load(std::memory_order_relaxed)) > 0) return sms;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return 148;
  if (dev >= 0 && dev < 64) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

int seq_items(const ckv_seq &s) {
  return (s.unit_end - s.unit_begin) + (s.resid_end - s.resid_begin + 15) / 16;
}

// CTAs per (sequence, KV head): a whole number of waves of one CTA per SM,
// about two items per warp, shared out in proportion to each pair's items.
int make_plan(const ckv_attn_args &a, int D, Plan &pl) {
  const int sms = sm_count();
  int64_t total = 0;
  for (int i = 0; i < a.num_seqs; ++i) total += int64_t(seq_items(a.seqs[i])) * a.heads_kv;
  const int64_t per_wave = int64_t(sms) * WARPS * 2;
  const int64_t waves = std::max<int64_t>(1, (total + per_wave - 1) / per_wave);
  const int64_t target = int64_t(sms) * waves;
  int grid = 0;
  for (int i = 0; i < a.num_seqs; ++i) {
    const int items = seq_items(a.seqs[i]);
    int64_t c = total > 0 ? (target * items + total / 2) / total : 1;
    c = std::max<int64_t>(1, std::min<int64_t>({c, std::max(items, 1), int64_t(kMaxCph)}));
    pl.cph[i] = int(c);
    pl.cta_begin[i] = grid;
    grid += int(c) * a.heads_kv;
  }
  pl.grid = grid;
  pl.rows = a.nq * (a.heads_q / a.heads_kv);
  pl.rec_off = kCounterBytes;
  pl.ml_off = pl.rec_off + (size_t(grid) * pl.rows * D * 4 + 255) / 256 * 256;
  pl.bytes = pl.ml_off + (size_t(grid) * pl.rows * 2 * 4 + 255) / 256 * 256;
  return CKV_OK;
}

bool al(const void *p, int b) { return (reinterpret_cast<uintptr_t>(p) % b) == 0; }

// Kernel parameters (up to ~29 KB for a batched call), built per call on the
// host; one per thread so concurrent host threads do not share it (the
// launch copies it).
template <int MAXS>
Params<MAXS> &params_scratch() {
  thread_local Params<MAXS> p;
  return p;
}

int validate(const ckv_attn_args &a) {
  if (a.num_seqs < 1 || a.num_seqs > CKV_MAX_SEQS || !a.seqs) return CKV_ERR_INVALID;
  if (a.heads_kv < 1 || a.heads_kv > kMaxHeadsKV || a.heads_q < a.heads_kv ||
      a.heads_q % a.heads_kv || a.nq < 1)
    return CKV_ERR_INVALID;
  if ((a.bits != 4 && a.bits != 8) || (a.dtype != CKV_BF16 && a.dtype != CKV_F16) ||
      !std::isfinite(a.scale))
    return CKV_ERR_INVALID;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return CKV_ERR_UNSUPPORTED;
  if (a.nq * (a.heads_q / a.heads_kv) > 16) return CKV_ERR_UNSUPPORTED;
  const int D = a.head_dim;
  for (int i = 0; i < a.num_seqs; ++i) {
    const ckv_seq &s = a.seqs[i];
    if (!s.query || !s.out) return CKV_ERR_INVALID;
    if (s.packed_tokens < 0 || s.packed_tokens % 128 || s.length < s.packed_tokens ||
        s.length > INT32_MAX)
      return CKV_ERR_INVALID;
    if (s.unit_begin < 0 || s.unit_end < s.unit_begin || int64_t(s.unit_end) * 128 > s.packed_tokens)
      return CKV_ERR_INVALID;
    if (s.resid_begin < 0 || s.resid_end < s.resid_begin ||
        s.packed_tokens + s.resid_end > s.length)
      return CKV_ERR_INVALID;
    if (!a.partial && s.unit_end == s.unit_begin && s.resid_end == s.resid_begin)
      return CKV_ERR_INVALID;  // nothing to attend to
    if (a.nq > 1 && s.length - a.nq < s.packed_tokens) return CKV_ERR_INVALID;
    if (s.unit_end > s.unit_begin) {
      if (!s.key_data || !s.key_meta || !s.value_data || !s.value_meta) return CKV_ERR_INVALID;
      if (!al(s.key_data, 16) || s.kd_stride_head % 16 || s.kd_stride_unit % 16) return CKV_ERR_INVALID;
      if (!al(s.key_meta, 16) || s.km_stride_head % 4 || s.km_stride_unit % 4) return CKV_ERR_INVALID;
      if (!al(s.value_data, 16) || s.vd_stride_head % 16 || s.vd_stride_token % 16) return CKV_ERR_INVALID;
      // 1-D bulk copies of 32 tokens' value metadata need dense token rows.
      if (!al(s.value_meta, 16) || s.vm_stride_head % 4 || s.vm_stride_token != (D / 64) * 2)
        return CKV_ERR_INVALID;
    }
    if (s.resid_end > s.resid_begin) {
      if (!s.keys || !s.values || !al(s.keys, 16) || !al(s.values, 16)) return CKV_ERR_INVALID;
      if (s.rk_stride_head % 8 || s.rk_stride_token % 8 || s.rv_stride_head % 8 ||
          s.rv_stride_token % 8)
        return CKV_ERR_INVALID;
    }
    if (!al(s.query, 2) || !al(s.out, a.partial ? 4 : 2)) return CKV_ERR_INVALID;
  }
  return CKV_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// Tensor maps of one sequence's packed banks (only the units [0, unit_end)
// are described; TMA never reads past them).
template <int BITS, int D>
int encode_maps(const ckv_seq &s, int hkv, SeqDev &d) {
  using C = Cfg<BITS, D, 1>;
  auto enc = encode_fn();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled unavailable");
    return CKV_ERR_CUDA;
  }
  constexpr uint64_t S = 128 * BITS / 8;
  const cuuint64_t kdims[4] = {S, cuuint64_t(D), cuuint64_t(s.unit_end), cuuint64_t(hkv)};
  const cuuint64_t kstr[3] = {S, cuuint64_t(s.kd_stride_unit), cuuint64_t(s.kd_stride_head)};
  const cuuint32_t kbox[4] = {32, cuuint32_t(D), 1, 1};
  const cuuint32_t one[4] = {1, 1, 1, 1};
  CUresult r = enc(&d.tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(s.key_data), kdims,
                   kstr, kbox, one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("key tensor map rejected (bank strides)");
    return CKV_ERR_INVALID;
  }
  const cuuint64_t vdims[3] = {cuuint64_t(C::VROWB), cuuint64_t(s.unit_end) * 128, cuuint64_t(hkv)};
  const cuuint64_t vstr[2] = {cuuint64_t(s.vd_stride_token), cuuint64_t(s.vd_stride_head)};
  const cuuint32_t vbox[3] = {cuuint32_t(C::VBOX), 32, 1};
  const CUtensorMapSwizzle swz = C::VBOX == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : C::VBOX == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                 : CU_TENSOR_MAP_SWIZZLE_32B;
  r = enc(&d.tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(s.value_data), vdims, vstr,
          vbox, one, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("value tensor map rejected (bank strides)");
    return CKV_ERR_INVALID;
  }
  return CKV_OK;
}

template <int BITS, int D, int NT, int DT, int MAXS>
int launch(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  using C = Cfg<BITS, D, NT>;
  auto kern = attn_kernel<BITS, D, NT, DT, MAXS>;
  static std::atomic<int> configured[64];
  int dev = 0;
  CKV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CKV_ERR_INVALID;
  if (!configured[dev].load(std::memory_order_acquire)) {
    CKV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured[dev].store(1, std::memory_order_release);
  }
  Params<MAXS> &p = params_scratch<MAXS>();
  memset(&p, 0, sizeof(ParamsHead) + sizeof(SeqDev) * a.num_seqs);
  p.num_seqs = a.num_seqs;
  p.hkv = a.heads_kv;
  p.group = a.heads_q / a.heads_kv;
  p.nq = a.nq;
  p.rows = pl.rows;
  p.partial = a.partial;
  p.scale_log2 = float(double(a.scale) * 1.4426950408889634);
  p.error = reinterpret_cast<unsigned *>(ws);
  p.counters = reinterpret_cast<unsigned *>(ws + kCounterOff);
  p.rec = reinterpret_cast<float *>(ws + pl.rec_off);
  p.rec_ml = reinterpret_cast<float *>(ws + pl.ml_off);
  for (int i = 0; i < a.num_seqs; ++i) {
    const ckv_seq &s = a.seqs[i];
    SeqDev &d = p.seq[i];
    d.q = s.query; d.q_h = s.q_stride_head; d.q_n = s.q_stride_pos;
    if (s.unit_end > s.unit_begin) {
      const int st = encode_maps<BITS, D>(s, a.heads_kv, d);
      if (st != CKV_OK) return st;
    }
    d.km = s.key_meta; d.km_h = s.km_stride_head; d.km_u = s.km_stride_unit;
    d.vm = s.value_meta; d.vm_h = s.vm_stride_head; d.vm_t = s.vm_stride_token;
    d.rk = s.keys; d.rk_h = s.rk_stride_head; d.rk_t = s.rk_stride_token;
    d.rv = s.values; d.rv_h = s.rv_stride_head; d.rv_t = s.rv_stride_token;
    d.out = s.out;
    d.packed = int32_t(s.packed_tokens);
    d.length = int32_t(s.length);
    d.ub = s.unit_begin; d.ue = s.unit_end; d.rb = s.resid_begin; d.re = s.resid_end;
    d.cta_begin = pl.cta_begin[i];
    d.cph = pl.cph[i];
  }
  kern<<<pl.grid, THREADS, C::SMEM, st>>>(p);
  return cuda_status(cudaGetLastError());
}

template <int BITS, int D, int NT, int DT>
int dispatch_seqs(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  return a.num_seqs == 1 ? launch<BITS, D, NT, DT, 1>(a, pl, ws, st)
                         : launch<BITS, D, NT, DT, CKV_MAX_SEQS>(a, pl, ws, st);
}
template <int BITS, int D, int NT>
int dispatch_dt(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  return a.dtype == CKV_BF16 ? dispatch_seqs<BITS, D, NT, CKV_BF16>(a, pl, ws, st)
                             : dispatch_seqs<BITS, D, NT, CKV_F16>(a, pl, ws, st);
}
template <int BITS, int D>
int dispatch_nt(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  return pl.rows <= 8 ? dispatch_dt<BITS, D, 1>(a, pl, ws, st) : dispatch_dt<BITS, D, 2>(a, pl, ws, st);
}
template <int BITS>
int dispatch_d(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  switch (a.head_dim) {
    case 64: return dispatch_nt<BITS, 64>(a, pl, ws, st);
    case 128: return dispatch_nt<BITS, 128>(a, pl, ws, st);
    default: return dispatch_nt<BITS, 256>(a, pl, ws, st);
  }
}

}  // namespace attn
}  // namespace ckv

using namespace ckv;
using namespace ckv::attn;

extern "C" int ckv_attention_workspace(const ckv_attn_args *args, size_t *bytes) {
  if (!args || !bytes) return CKV_ERR_INVALID;
  const int v = validate(*args);
  if (v != CKV_OK) return v;
  Plan pl;
  make_plan(*args, args->head_dim, pl);
  *bytes = pl.bytes;
  return CKV_OK;
}

extern "C" int ckv_attention(const ckv_attn_args *args, void *workspace, size_t workspace_bytes,
                             ckv_stream_t stream) {
  if (!args) return CKV_ERR_INVALID;
  const int v = validate(*args);
  if (v != CKV_OK) return v;
  Plan pl;
  make_plan(*args, args->head_dim, pl);
  if (!workspace || workspace_bytes < pl.bytes || !al(workspace, 256)) return CKV_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  if (!(args->flags & CKV_WS_COUNTERS_ZERO))
    CKV_CUDA_TRY(cudaMemsetAsync(ws, 0, kCounterOff + size_t(args->num_seqs) * args->heads_kv * 4, st));
  return args->bits == 8 ? dispatch_d<8>(*args, pl, ws, st) : dispatch_d<4>(*args, pl, ws, st);
}

extern "C" int ckv_attention_error(const void *workspace, int *flag, ckv_stream_t stream) {
  if (!workspace || !flag) return CKV_ERR_INVALID;
  unsigned v = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CKV_CUDA_TRY(cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, st));
  CKV_CUDA_TRY(cudaStreamSynchronize(st));
  *flag = int(v);
  return CKV_OK;
}

extern "C" int ckv_combine_partials(const float *partials, int parts, int64_t rows, int head_dim,
                                    int dtype, void *out, ckv_stream_t stream) {
  if (!partials || !out || parts < 1 || rows < 0 || head_dim < 1 || head_dim > 1024)
    return CKV_ERR_INVALID;
  if (dtype != CKV_BF16 && dtype != CKV_F16) return CKV_ERR_INVALID;
  if (rows == 0) return CKV_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int threads = std::min(256, head_dim);
  if (dtype == CKV_BF16)
    combine_kernel<CKV_BF16><<<unsigned(rows), threads, 0, st>>>(
        partials, parts, rows, head_dim, static_cast<__nv_bfloat16 *>(out));
  else
    combine_kernel<CKV_F16><<<unsigned(rows), threads, 0, st>>>(partials, parts, rows, head_dim,
                                                                static_cast<__half *>(out));
  return cuda_status(cudaGetLastError());
}
