// ckv_prefill.cu -- packed multi-query prefill: lower-right causal attention
// of a query chunk (q_len rows, all query heads) over the quantized history
// plus the exact residual window that already holds the chunk.
//
// Semantics follow models/compressed_prefill_kernels.py:29-95 (the kernel
// behind models/compressed_prefill_attention.py:6-52):
//   * packed keys/values are dequantized exactly as
//     dtype(fma(float(code), scale, low)) (compressed_prefill_kernels.py:62,73);
//   * logits = (q . k) * (scale * log2 e), probabilities 2^(logit - m) with an
//     online max, P rounded to the query dtype before P.V, the denominator
//     summed from the fp32 probabilities (compressed_prefill_kernels.py:13-25);
//   * packed history precedes every query: no mask there (:46-47);
//   * residual token t (0-based in the window of R tokens) is visible to query
//     position n iff t <= R - q_len + n, lower-right alignment (:81-90);
//   * out = accum / denom, stored in the query dtype, [Hq, q_len, D] dense.
//
// B200 layout of the work: one CTA per (KV head, tile of 128 query rows),
// where a query row is (position n, group head g) in n-major order, so the
// G query heads that share a KV head share every dequantized K/V tile (the
// reference launches one program per query head and dequantizes G times).
// Eight warps, 16 rows each; logits and P.V on mma.sync m16n8k16 with fp32
// accumulators; K/V tiles of BT = 64 tokens staged in shared memory:
//   packed K   channel-major [D][BT]  (a bank row is one channel over a block)
//   residual K token-major   [BT][D]
//   V          token-major   [BT][D]
// K/V tiles are double-buffered: a packed tile's codes are read into
// registers before the previous tile's math and written out (dequantized)
// after it; residual tiles arrive by cp.async.
#include "ckv_common.cuh"

#include <algorithm>
#include <atomic>
#include <cmath>

namespace ckv {
namespace attn {
int sm_count();  // SMs of the current device (148 without one), ckv_attn.cu
}
namespace prefill {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int BM = 16 * kWarps;  // query rows per CTA

template <int D>
struct Cfg {
  static constexpr int BT = 64;  // tokens per K/V tile (divides 128)
  static constexpr int QS = D + 8;    // query tile row stride (elements)
  static constexpr int KCS = BT + 8;  // packed K, channel-major [D][BT]
  static constexpr int KRS = D + 8;   // residual K, token-major [BT][D]
  static constexpr int VS = D + 8;    // V, token-major [BT][D]
  static constexpr int Q_BYTES = BM * QS * 2;
  static constexpr int K_ELEMS = D * KCS > BT * KRS ? D * KCS : BT * KRS;
  static constexpr int K_BYTES = K_ELEMS * 2;
  static constexpr int V_BYTES = BT * VS * 2;
  static constexpr int SMEM = Q_BYTES + 2 * (K_BYTES + V_BYTES);
  // Per-thread share of one tile's loads (16-byte chunks of codes or rows).
  static constexpr int K_TASKS = D * (BT / 16) / kThreads;  // packed K: (channel, 16 tokens)
  static constexpr int V_TASKS = BT * (D / 16) / kThreads;  // packed V: (token, 16 channels)
  static_assert(K_TASKS * kThreads == D * (BT / 16), "K tile split");
  static_assert(V_TASKS * kThreads == BT * (D / 16), "V tile split");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct Params {
  const void *q;
  int64_t qhs, qts;
  const uint8_t *kd;
  int64_t kds_h, kds_u;
  const float *km;
  int64_t kms_h, kms_u;
  const uint8_t *vd;
  int64_t vds_h, vds_t;
  const float *vm;
  int64_t vms_h, vms_t;
  const void *rk;
  int64_t rks_h, rks_t;
  const void *rv;
  int64_t rvs_h, rvs_t;
  void *out;
  int qlen, packed, resid, groups;
  float scale_log2;
  int splits;        // history splits (grid z); > 1 writes partial records
  float *partials;   // [splits][Hq * qlen][D + 2] fp32 when splits > 1
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w));
}

// 16 codes (one per output element, in order) -> 16 dequantized elements,
// dtype(fma(code, scale, low)), packed two per word.
template <int BITS, int DT>
__device__ __forceinline__ void dequant16(const uint4 &raw, float scale, float low, uint4 &lo,
                                          uint4 &hi) {
  using E = Elem<DT>;
  uint32_t w[4];
  if constexpr (BITS == 8) {
    w[0] = raw.x, w[1] = raw.y, w[2] = raw.z, w[3] = raw.w;
  } else {
    // 8 bytes, two codes each, element 2j in the low nibble of byte j: spread
    // to one code per byte.
    const uint32_t a = raw.x, b = raw.y;
    const uint32_t al = a & 0x0F0F0F0Fu, ah = (a >> 4) & 0x0F0F0F0Fu;
    const uint32_t bl = b & 0x0F0F0F0Fu, bh = (b >> 4) & 0x0F0F0F0Fu;
    w[0] = prmt(al, ah, 0x5140u);  // bytes 0,1 of a: lo0 hi0 lo1 hi1
    w[1] = prmt(al, ah, 0x7362u);
    w[2] = prmt(bl, bh, 0x5140u);
    w[3] = prmt(bl, bh, 0x7362u);
  }
  // Paired fp32: code = (2^23 + code) - 2^23 exactly, then one rounding of
  // fma(code, scale, low) per element, as in the scalar form.
  const float2 sc = make_float2(scale, scale), lw = make_float2(low, low);
  const float2 nm = make_float2(-kMagic, -kMagic);
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 c01 = __fadd2_rn(make_float2(byte_magic<0>(w[i]), byte_magic<1>(w[i])), nm);
    const float2 c23 = __fadd2_rn(make_float2(byte_magic<2>(w[i]), byte_magic<3>(w[i])), nm);
    const float2 x01 = __ffma2_rn(c01, sc, lw), x23 = __ffma2_rn(c23, sc, lw);
    o[2 * i] = E::pack2(x01.x, x01.y);
    o[2 * i + 1] = E::pack2(x23.x, x23.y);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

// Codes and metadata of one packed tile, held in registers between the read
// from global memory and the dequantized write to shared memory.
template <int BITS, int D>
struct PackedRegs {
  uint4 k[Cfg<D>::K_TASKS];
  float2 km[Cfg<D>::K_TASKS];
  uint4 v[Cfg<D>::V_TASKS];
  float2 vm[Cfg<D>::V_TASKS];
};

template <int BITS, int D>
__device__ __forceinline__ void read_packed(const Params &p, int kvh, int t0, int tid,
                                            PackedRegs<BITS, D> &r) {
  using C = Cfg<D>;
  constexpr int SB = C::BT / 16;  // 16-token pieces of a channel row
  const int unit = t0 >> 7, s_off = t0 & 127;
  const uint8_t *kd = p.kd + kvh * p.kds_h + int64_t(unit) * p.kds_u;
  const float *km = p.km + kvh * p.kms_h + int64_t(unit) * p.kms_u;
#pragma unroll
  for (int j = 0; j < C::K_TASKS; ++j) {
    const int i = tid + j * kThreads, d = i / SB, s0 = s_off + (i % SB) * 16;
    if constexpr (BITS == 8) {
      r.k[j] = __ldg(reinterpret_cast<const uint4 *>(kd + d * 128 + s0));
    } else {
      const uint2 x = __ldg(reinterpret_cast<const uint2 *>(kd + d * 64 + s0 / 2));
      r.k[j] = make_uint4(x.x, x.y, 0u, 0u);
    }
    r.km[j] = __ldg(reinterpret_cast<const float2 *>(km + d * 2));
  }
  constexpr int CH = D / 16;  // 16-channel pieces of a token row
#pragma unroll
  for (int j = 0; j < C::V_TASKS; ++j) {
    const int i = tid + j * kThreads, t = t0 + i / CH, c0 = (i % CH) * 16;
    const uint8_t *vd = p.vd + kvh * p.vds_h + int64_t(t) * p.vds_t;
    if constexpr (BITS == 8) {
      r.v[j] = __ldg(reinterpret_cast<const uint4 *>(vd + (c0 >> 6) * 64 + (c0 & 63)));
    } else {
      const uint2 x = __ldg(reinterpret_cast<const uint2 *>(vd + (c0 >> 6) * 32 + (c0 & 63) / 2));
      r.v[j] = make_uint4(x.x, x.y, 0u, 0u);
    }
    r.vm[j] = __ldg(reinterpret_cast<const float2 *>(p.vm + kvh * p.vms_h + int64_t(t) * p.vms_t +
                                                     (c0 >> 6) * 2));
  }
}

template <int BITS, int D, int DT>
__device__ __forceinline__ void write_packed(const PackedRegs<BITS, D> &r, uint32_t ks,
                                             uint32_t vs, int tid) {
  using C = Cfg<D>;
  constexpr int SB = C::BT / 16;
#pragma unroll
  for (int j = 0; j < C::K_TASKS; ++j) {
    const int i = tid + j * kThreads, d = i / SB, sb = (i % SB) * 16;
    uint4 lo, hi;
    dequant16<BITS, DT>(r.k[j], r.km[j].x, r.km[j].y, lo, hi);
    const uint32_t a = ks + uint32_t(d * C::KCS + sb) * 2;
    sts128(a, lo);
    sts128(a + 16, hi);
  }
  constexpr int CH = D / 16;
  // Eight lanes write 32-byte pieces of one token row: lanes 4..7 store
  // their upper halves first, so each store instruction covers all 32 banks
  // once (with CH = 4 the two rows' padding already does that).
  const bool swap = CH >= 8 && (tid & 4);
#pragma unroll
  for (int j = 0; j < C::V_TASKS; ++j) {
    const int i = tid + j * kThreads, t = i / CH, c0 = (i % CH) * 16;
    uint4 lo, hi;
    dequant16<BITS, DT>(r.v[j], r.vm[j].x, r.vm[j].y, lo, hi);
    const uint32_t a = vs + uint32_t(t * C::VS + c0) * 2;
    sts128(swap ? a + 16 : a, swap ? hi : lo);
    sts128(swap ? a : a + 16, swap ? lo : hi);
  }
}

// Residual tile: rows [t0, t0 + BT) of the exact window by cp.async, zero
// past R (the copy then reads nothing and its address stays the row base).
template <int D>
__device__ __forceinline__ void issue_resid(const Params &p, int kvh, int t0, int tid, uint32_t ks,
                                            uint32_t vs) {
  using C = Cfg<D>;
  constexpr int CH = D / 8;
  const uint16_t *rk = static_cast<const uint16_t *>(p.rk) + kvh * p.rks_h;
  const uint16_t *rv = static_cast<const uint16_t *>(p.rv) + kvh * p.rvs_h;
  for (int i = tid; i < C::BT * CH; i += kThreads) {
    const int t = i / CH, c = (i % CH) * 8, tt = t0 + t;
    const bool ok = tt < p.resid;
    cp_async16(ks + uint32_t(t * C::KRS + c) * 2, ok ? rk + int64_t(tt) * p.rks_t + c : rk,
               ok ? 16 : 0);
    cp_async16(vs + uint32_t(t * C::VS + c) * 2, ok ? rv + int64_t(tt) * p.rvs_t + c : rv,
               ok ? 16 : 0);
  }
  cp_async_commit();
}

// One tile of BT tokens for this warp's 16 rows: logits, online softmax,
// P.V.  PACKED selects the channel-major K layout; otherwise K is token-major
// and the residual mask applies (token index tbase + column).
template <int D, int DT, bool PACKED>
__device__ __forceinline__ void tile_math(uint32_t qs, uint32_t ks, uint32_t vs, int warp,
                                          int lane, float (&o)[D / 8][4], float (&m)[2],
                                          float (&l)[2], float scale_log2, int tbase, int tlimit,
                                          const int (&vis)[2]) {
  using C = Cfg<D>;
  using E = Elem<DT>;
  constexpr int BT = C::BT;
  float s[BT / 8][4];
#pragma unroll
  for (int nt = 0; nt < BT / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
  const int li = lane >> 3, lr = lane & 7;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4(a, qs + uint32_t((warp * 16 + (lane & 15)) * C::QS + kk * 16 + (lane >> 4) * 8) * 2);
#pragma unroll
    for (int np = 0; np < BT / 16; ++np) {
      uint32_t b[4];
      if constexpr (PACKED) {
        ldsm_x4_t(b, ks + uint32_t((kk * 16 + (li & 1) * 8 + lr) * C::KCS + np * 16 +
                                   (li >> 1) * 8) * 2);
      } else {
        ldsm_x4(b, ks + uint32_t((np * 16 + (li >> 1) * 8 + lr) * C::KRS + kk * 16 +
                                 (li & 1) * 8) * 2);
      }
      mma16816<DT>(s[2 * np], a, b[0], b[1]);
      mma16816<DT>(s[2 * np + 1], a, b[2], b[3]);
    }
  }
  // Scale, mask, row max over the quad that shares a row.
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < BT / 8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x = s[nt][j] * scale_log2;
      if constexpr (!PACKED) {
        const int t = tbase + nt * 8 + 2 * (lane & 3) + (j & 1);
        if (t >= tlimit || t > vis[j >> 1]) x = -INFINITY;
      }
      s[nt][j] = x;
      mx[j >> 1] = fmaxf(mx[j >> 1], x);
    }
  float alpha[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    float nm = fmaxf(m[h], mx[h]);
    if (nm == -INFINITY) nm = 0.f;  // a row with nothing visible yet: no inf - inf
    alpha[h] = ex2(m[h] - nm);
    m[h] = nm;
  }
  float rs[2] = {0.f, 0.f};
#pragma unroll
  for (int nt = 0; nt < BT / 8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float e = ex2(s[nt][j] - m[j >> 1]);
      s[nt][j] = e;
      rs[j >> 1] += e;
    }
  l[0] = l[0] * alpha[0] + rs[0];
  l[1] = l[1] * alpha[1] + rs[1];
  // Once the row maxima settle (alpha exactly 1 for all of the warp's rows)
  // the rescale is the identity: skip it.
  if (!__all_sync(0xffffffffu, alpha[0] == 1.f && alpha[1] == 1.f)) {
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }
  }
#pragma unroll
  for (int kt = 0; kt < BT / 16; ++kt) {
    uint32_t a[4];
    a[0] = E::pack2(s[2 * kt][0], s[2 * kt][1]);
    a[1] = E::pack2(s[2 * kt][2], s[2 * kt][3]);
    a[2] = E::pack2(s[2 * kt + 1][0], s[2 * kt + 1][1]);
    a[3] = E::pack2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t b[4];
      ldsm_x4_t(b, vs + uint32_t((kt * 16 + (li & 1) * 8 + lr) * C::VS + dp * 16 + (li >> 1) * 8) *
                            2);
      mma16816<DT>(o[2 * dp], a, b[0], b[1]);
      mma16816<DT>(o[2 * dp + 1], a, b[2], b[3]);
    }
  }
}

template <int BITS, int D, int DT>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ Params p) {
  using C = Cfg<D>;
  using E = Elem<DT>;
  constexpr int BT = C::BT;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y;
  // Late query tiles see the most residual tokens: start them first.
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int G = p.groups, nrows = p.qlen * G, r0 = tile * BM;
  const uint32_t qs = smem_u32(smem);
  const uint32_t kbuf[2] = {qs + C::Q_BYTES, qs + C::Q_BYTES + C::K_BYTES + C::V_BYTES};
  const uint32_t vbuf[2] = {kbuf[0] + C::K_BYTES, kbuf[1] + C::K_BYTES};

  // Query tile (zero rows past the chunk).
  {
    constexpr int CH = D / 8;
    const uint16_t *q = static_cast<const uint16_t *>(p.q);
    for (int i = tid; i < BM * CH; i += kThreads) {
      const int r = i / CH, c = (i % CH) * 8, gr = r0 + r;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (gr < nrows) {
        const int pos = gr / G, h = kvh * G + gr % G;
        v = __ldg(reinterpret_cast<const uint4 *>(q + h * p.qhs + int64_t(pos) * p.qts + c));
      }
      sts128(qs + uint32_t(r * C::QS + c) * 2, v);
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  // Last residual token each of this thread's two rows may see.
  int vis[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = r0 + warp * 16 + (lane >> 2) + 8 * h;
    vis[h] = p.resid - p.qlen + gr / G;
  }
  // History split z of p.splits: an even share of this CTA's items, its
  // packed tiles followed by its residual tiles (up to its last visible
  // token).  The split with the most recent tokens launches first.
  const int z = p.splits - 1 - int(blockIdx.z), ntiles = p.packed / BT;
  const int last_row = min(r0 + BM, nrows) - 1;
  const int rstop = min(p.resid, p.resid - p.qlen + last_row / G + 1);
  const int total = ntiles + (rstop + BT - 1) / BT;
  const int a0 = int(int64_t(total) * z / p.splits), a1 = int(int64_t(total) * (z + 1) / p.splits);
  const int i0 = min(a0, ntiles), np = min(a1, ntiles) - i0;
  const int rb = max(a0, ntiles) - ntiles, nr = max(a1, ntiles) - ntiles - rb;

  // Packed history, double-buffered through registers.
  if (np > 0) {
    PackedRegs<BITS, D> pr;
    read_packed<BITS, D>(p, kvh, i0 * BT, tid, pr);
    write_packed<BITS, D, DT>(pr, kbuf[0], vbuf[0], tid);
    __syncthreads();
    for (int i = 0; i < np; ++i) {
      const int b = i & 1;
      if (i + 1 < np) read_packed<BITS, D>(p, kvh, (i0 + i + 1) * BT, tid, pr);
      tile_math<D, DT, true>(qs, kbuf[b], vbuf[b], warp, lane, o, m, l, p.scale_log2, 0, 0, vis);
      if (i + 1 < np) write_packed<BITS, D, DT>(pr, kbuf[b ^ 1], vbuf[b ^ 1], tid);
      __syncthreads();
    }
  }
  // Exact residual window, tiles [rb, rb + nr); tile i sits in buffer
  // (np + i) & 1, the next one lands while this one is used.
  if (nr > 0) issue_resid<D>(p, kvh, rb * BT, tid, kbuf[np & 1], vbuf[np & 1]);
  for (int i = 0; i < nr; ++i) {
    const int b = (np + i) & 1;
    if (i + 1 < nr) {
      issue_resid<D>(p, kvh, (rb + i + 1) * BT, tid, kbuf[b ^ 1], vbuf[b ^ 1]);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    tile_math<D, DT, false>(qs, kbuf[b], vbuf[b], warp, lane, o, m, l, p.scale_log2, (rb + i) * BT,
                            p.resid, vis);
    __syncthreads();
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  if (p.splits > 1) {
    // Partial record of output row (head, pos) for split z, the layout
    // ckv_combine_partials merges: sum 2^(s - m) v over this split's tokens,
    // then m (log2 domain) and l = sum 2^(s - m).
    const int64_t orows = int64_t(p.qlen) * G * gridDim.y;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int gr = r0 + warp * 16 + (lane >> 2) + 8 * h;
      if (gr >= nrows) continue;
      const int pos = gr / G, head = kvh * G + gr % G;
      float *rec = p.partials + (int64_t(z) * orows + int64_t(head) * p.qlen + pos) * (D + 2);
#pragma unroll
      for (int nt = 0; nt < D / 8; ++nt)
        *reinterpret_cast<float2 *>(rec + nt * 8 + 2 * (lane & 3)) =
            make_float2(o[nt][2 * h], o[nt][2 * h + 1]);
      // A row that saw no token in this split (a split of residual tiles all
      // past its position) records m = -inf: weight 0 in the merge.
      if ((lane & 3) == 0)
        *reinterpret_cast<float2 *>(rec + D) = make_float2(l[h] > 0.f ? m[h] : -INFINITY, l[h]);
    }
    return;
  }
  // out = accum / denom in the query dtype; rows past the chunk are dropped.
  uint16_t *out = static_cast<uint16_t *>(p.out);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = r0 + warp * 16 + (lane >> 2) + 8 * h;
    if (gr >= nrows) continue;
    const int pos = gr / G, head = kvh * G + gr % G;
    uint16_t *row = out + (int64_t(head) * p.qlen + pos) * D + 2 * (lane & 3);
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) {
      const uint32_t v =
          E::pack2(__fdiv_rn(o[nt][2 * h], l[h]), __fdiv_rn(o[nt][2 * h + 1], l[h]));
      *reinterpret_cast<uint32_t *>(row + nt * 8) = v;
    }
  }
}

bool al(const void *ptr, int b) { return (reinterpret_cast<uintptr_t>(ptr) % b) == 0; }

int validate(const ckv_prefill_args &a) {
  const ckv_seq &s = a.seq;
  if ((a.bits != 4 && a.bits != 8) || (a.dtype != CKV_BF16 && a.dtype != CKV_F16) ||
      !std::isfinite(a.scale))
    return CKV_ERR_INVALID;
  if (a.heads_kv < 1 || a.heads_q < a.heads_kv || a.heads_q % a.heads_kv || a.qlen < 1)
    return CKV_ERR_INVALID;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return CKV_ERR_UNSUPPORTED;
  if (a.heads_kv > 65535 || int64_t(a.qlen) * (a.heads_q / a.heads_kv) > (int64_t(1) << 30))
    return CKV_ERR_UNSUPPORTED;
  if (!s.query || !s.out || !s.keys || !s.values) return CKV_ERR_INVALID;
  if (s.packed_tokens < 128 || s.packed_tokens % 128 || s.length > INT32_MAX) return CKV_ERR_INVALID;
  const int64_t R = s.length - s.packed_tokens;
  if (R < a.qlen) return CKV_ERR_INVALID;  // the window holds the whole chunk
  // The whole history: no split-KV shard for prefill.
  if (s.unit_begin != 0 || int64_t(s.unit_end) * 128 != s.packed_tokens || s.resid_begin != 0 ||
      s.resid_end != R)
    return CKV_ERR_UNSUPPORTED;
  if (!s.key_data || !s.key_meta || !s.value_data || !s.value_meta) return CKV_ERR_INVALID;
  const int kq = a.bits == 8 ? 16 : 8;  // width of one code load
  if (!al(s.key_data, kq) || s.kd_stride_head % kq || s.kd_stride_unit % kq) return CKV_ERR_INVALID;
  if (!al(s.value_data, kq) || s.vd_stride_head % kq || s.vd_stride_token % kq) return CKV_ERR_INVALID;
  if (!al(s.key_meta, 8) || s.km_stride_head % 2 || s.km_stride_unit % 2) return CKV_ERR_INVALID;
  if (!al(s.value_meta, 8) || s.vm_stride_head % 2 || s.vm_stride_token % 2) return CKV_ERR_INVALID;
  for (const void *ptr : {s.query, s.keys, s.values})
    if (!al(ptr, 16)) return CKV_ERR_INVALID;
  for (int64_t st : {s.q_stride_head, s.q_stride_pos, s.rk_stride_head, s.rk_stride_token,
                     s.rv_stride_head, s.rv_stride_token})
    if (st % 8) return CKV_ERR_INVALID;
  if (!al(s.out, 4)) return CKV_ERR_INVALID;
  return CKV_OK;
}

// History splits: each CTA's items (packed tiles, then its residual tiles)
// are split so that the grid of (query tiles x KV heads x splits) fills
// whole waves of one CTA per SM -- a short grid up to one wave, a longer one
// (at most 4 splits) to fewer idle SMs in its last wave.  The fewest splits
// within 2% of the best fill win, at most one split per 64-token packed
// tile; the splits' partial records are then merged.
struct Plan {
  int tiles = 0, splits = 1;
  size_t bytes = 0;  // workspace for the partial records
};

Plan make_plan(const ckv_prefill_args &a) {
  Plan pl;
  const int64_t rows = int64_t(a.qlen) * (a.heads_q / a.heads_kv);
  pl.tiles = int((rows + BM - 1) / BM);
  const int64_t ctas = int64_t(pl.tiles) * a.heads_kv;
  const int sms = attn::sm_count();
  const int64_t ntiles = a.seq.packed_tokens / 64;
  const int64_t smax = std::min<int64_t>(ntiles, std::max<int64_t>(4, sms / std::max<int64_t>(ctas, 1)));
  double best = 0.0;
  for (int64_t sp = 1; sp <= smax; ++sp) {
    const int64_t n = ctas * sp, waves = (n + sms - 1) / sms;
    const double fill = double(n) / double(waves * sms);
    if (fill > best + 0.02) {
      best = fill;
      pl.splits = int(sp);
    }
  }
  if (pl.splits > 1)
    pl.bytes = size_t(pl.splits) * size_t(a.heads_q) * size_t(a.qlen) * size_t(a.head_dim + 2) * 4;
  return pl;
}

template <int BITS, int D, int DT>
int launch(const ckv_prefill_args &a, const Plan &pl, void *workspace, cudaStream_t st) {
  using C = Cfg<D>;
  auto kern = prefill_kernel<BITS, D, DT>;
  // The shared-memory opt-in is a per-device function attribute.
  static std::atomic<int> configured[64];
  int dev = 0;
  CKV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CKV_ERR_INVALID;
  if (!configured[dev].load(std::memory_order_acquire)) {
    CKV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured[dev].store(1, std::memory_order_release);
  }
  const ckv_seq &s = a.seq;
  Params p;
  p.q = s.query;
  p.qhs = s.q_stride_head;
  p.qts = s.q_stride_pos;
  p.kd = s.key_data;
  p.kds_h = s.kd_stride_head;
  p.kds_u = s.kd_stride_unit;
  p.km = s.key_meta;
  p.kms_h = s.km_stride_head;
  p.kms_u = s.km_stride_unit;
  p.vd = s.value_data;
  p.vds_h = s.vd_stride_head;
  p.vds_t = s.vd_stride_token;
  p.vm = s.value_meta;
  p.vms_h = s.vm_stride_head;
  p.vms_t = s.vm_stride_token;
  p.rk = s.keys;
  p.rks_h = s.rk_stride_head;
  p.rks_t = s.rk_stride_token;
  p.rv = s.values;
  p.rvs_h = s.rv_stride_head;
  p.rvs_t = s.rv_stride_token;
  p.out = s.out;
  p.qlen = a.qlen;
  p.packed = int(s.packed_tokens);
  p.resid = int(s.length - s.packed_tokens);
  p.groups = a.heads_q / a.heads_kv;
  p.scale_log2 = float(double(a.scale) * 1.4426950408889634);
  p.splits = pl.splits;
  p.partials = static_cast<float *>(workspace);
  const dim3 grid(unsigned(pl.tiles), unsigned(a.heads_kv), unsigned(pl.splits));
  kern<<<grid, kThreads, C::SMEM, st>>>(p);
  CKV_CUDA_TRY(cudaGetLastError());
  if (pl.splits == 1) return CKV_OK;
  return ckv_combine_partials(p.partials, pl.splits, int64_t(a.heads_q) * a.qlen, D, DT, s.out,
                              reinterpret_cast<ckv_stream_t>(st));
}

template <int BITS, int D>
int dispatch_dt(const ckv_prefill_args &a, const Plan &pl, void *ws, cudaStream_t st) {
  return a.dtype == CKV_BF16 ? launch<BITS, D, CKV_BF16>(a, pl, ws, st)
                             : launch<BITS, D, CKV_F16>(a, pl, ws, st);
}

template <int BITS>
int dispatch_d(const ckv_prefill_args &a, const Plan &pl, void *ws, cudaStream_t st) {
  switch (a.head_dim) {
    case 64: return dispatch_dt<BITS, 64>(a, pl, ws, st);
    case 128: return dispatch_dt<BITS, 128>(a, pl, ws, st);
    default: return dispatch_dt<BITS, 256>(a, pl, ws, st);
  }
}

}  // namespace prefill
}  // namespace ckv

extern "C" int ckv_prefill_workspace(const ckv_prefill_args *args, size_t *bytes) {
  using namespace ckv::prefill;
  if (!args || !bytes) return CKV_ERR_INVALID;
  const int v = validate(*args);
  if (v != CKV_OK) return v;
  *bytes = make_plan(*args).bytes;
  return CKV_OK;
}

extern "C" int ckv_prefill(const ckv_prefill_args *args, void *workspace, size_t workspace_bytes,
                           ckv_stream_t stream) {
  using namespace ckv::prefill;
  if (!args) return CKV_ERR_INVALID;
  const int v = validate(*args);
  if (v != CKV_OK) return v;
  const Plan pl = make_plan(*args);
  if (pl.bytes && (!workspace || workspace_bytes < pl.bytes || !al(workspace, 16)))
    return CKV_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return args->bits == 8 ? dispatch_d<8>(*args, pl, workspace, st)
                         : dispatch_d<4>(*args, pl, workspace, st);
}
