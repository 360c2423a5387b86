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

// ---------------------------------------------------------------------------
// 5th-generation tensor-core variant (tcgen05, D = 128 / 256).
//
// Same work split, dequantization, softmax rule, masks and partial records
// as prefill_kernel; the two products run on tcgen05.mma with both operands
// in shared memory and the fp32 accumulators in tensor memory:
//   S = Q K^T   M = 128 query rows, N = 64 tokens, K = D     -> TMEM columns [0, 64)
//   O += P V    M = 128 query rows, N = D,         K = 64    -> TMEM columns [256, 256 + D)
// Shared-memory tiles, 16-bit, in the canonical 128-byte-swizzled layouts
// (16-byte chunk c of a 128-byte row r stored at chunk c ^ (r & 7); 1024-byte
// atoms of 8 rows):
//   Q   K-major:  [D/64 blocks][128 rows][64 channels]
//   K   packed:   MN-major [D channel rows][64 tokens] (the bank's channel-major
//                 order, so dequantized codes are stored without a transpose);
//       window:   K-major  [D/64 blocks][64 token rows][64 channels] (the
//                 window's token-major order)
//   V   MN-major: [D/64 blocks][64 token rows][64 channels]
//   P   K-major:  [128 rows][64 tokens]
// One thread issues the MMAs; tcgen05.commit signals an mbarrier when they
// complete.  Warps 0-3 own the 128 accumulator lanes (thread = query row):
// each loads its row of S from tensor memory, runs the online softmax, writes
// its P row, and rescales its O row in tensor memory when its maximum grows.
// All eight warps dequantize; the next packed tile's codes are read into
// registers while this tile's products run.
namespace tc {

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;

template <int D>
struct TCfg {
  static constexpr int BT = 64;
  static constexpr int Q_BYTES = BM * D * 2;           // 128 rows
  static constexpr int KV_BYTES = D * BT * 2;          // one K or V tile
  static constexpr int P_BYTES = BM * BT * 2;
  static constexpr int OFF_Q = 0, OFF_K = Q_BYTES, OFF_V = OFF_K + KV_BYTES, OFF_P = OFF_V + KV_BYTES;
  static constexpr int SMEM = OFF_P + P_BYTES + 1024;  // + alignment slack
  static_assert(D % 64 == 0 && D <= 256, "head_dim");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Shared-memory matrix descriptor: start, leading / stride byte offsets
// (16-byte units), the sm_100 descriptor version (1), 128-byte swizzle (2).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulator, A and B of the query
// dtype, their major-ness (0 = K-major, 1 = MN-major), N and M.
template <int DT>
constexpr uint32_t idesc(int M, int N, int a_mn, int b_mn) {
  constexpr uint32_t fmt = DT == CKV_BF16 ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t id,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(id), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the tensor cores.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 32 consecutive fp32 columns of this thread's lane (32x32b shape; the whole
// warp must execute it).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte chunk `c` (0..7) of 128-byte row `r` in a swizzled tile.
__device__ __forceinline__ uint32_t swz128(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ unsigned g_error;   // set when a bounded wait gave up (ckv_prefill_error)

__device__ __forceinline__ void wait_bar(uint32_t bar, uint32_t parity) {
  if (!mbar_wait(bar, parity)) atomicOr(&g_error, 1u);
}

// A packed tile's codes (registers, read_packed's split) into K (MN-major,
// channel rows) and V (MN-major, token rows) in the swizzled layouts.
template <int BITS, int D, int DT>
__device__ __forceinline__ void write_packed_tc(const PackedRegs<BITS, D> &r, uint32_t ks,
                                                uint32_t vs, int tid) {
  using C = Cfg<D>;
  constexpr int SB = C::BT / 16;
#pragma unroll
  for (int j = 0; j < C::K_TASKS; ++j) {
    const int i = tid + j * kThreads, d = i / SB, c = (i % SB) * 2;   // chunks c, c + 1 of row d
    uint4 lo, hi;
    dequant16<BITS, DT>(r.k[j], r.km[j].x, r.km[j].y, lo, hi);
    sts128(ks + swz128(d, c), lo);
    sts128(ks + swz128(d, c + 1), hi);
  }
  constexpr int CH = D / 16;
#pragma unroll
  for (int j = 0; j < C::V_TASKS; ++j) {
    const int i = tid + j * kThreads, t = i / CH, c0 = (i % CH) * 16;
    uint4 lo, hi;
    dequant16<BITS, DT>(r.v[j], r.vm[j].x, r.vm[j].y, lo, hi);
    const uint32_t blk = vs + uint32_t(c0 >> 6) * (64 * 128);
    const int c = (c0 & 63) >> 3;
    sts128(blk + swz128(t, c), lo);
    sts128(blk + swz128(t, c + 1), hi);
  }
}

// Window tile: rows [t0, t0 + 64) of the exact K and V, zero past R, into K
// (K-major, token rows) and V (MN-major, token rows).
template <int D>
__device__ __forceinline__ void write_resid_tc(const Params &p, int kvh, int t0, int tid, uint32_t ks,
                                               uint32_t vs) {
  constexpr int CH = D / 8;   // 16-byte chunks of a row
  const uint16_t *rk = static_cast<const uint16_t *>(p.rk) + kvh * p.rks_h;
  const uint16_t *rv = static_cast<const uint16_t *>(p.rv) + kvh * p.rvs_h;
  for (int i = tid; i < 64 * CH; i += kThreads) {
    const int t = i / CH, c8 = i % CH, tt = t0 + t;
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (tt < p.resid) {
      kv = __ldg(reinterpret_cast<const uint4 *>(rk + int64_t(tt) * p.rks_t + c8 * 8));
      vv = __ldg(reinterpret_cast<const uint4 *>(rv + int64_t(tt) * p.rvs_t + c8 * 8));
    }
    const uint32_t blk = uint32_t(c8 >> 3) * (64 * 128);
    sts128(ks + blk + swz128(t, c8 & 7), kv);
    sts128(vs + blk + swz128(t, c8 & 7), vv);
  }
}

template <int BITS, int D, int DT>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ Params p) {
  using T = TCfg<D>;
  using E = Elem<DT>;
  constexpr int BT = T::BT;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t s_bar[2];   // S products done, O products done
  __shared__ uint32_t s_tmem;
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sb = smem_u32(smem);
  const uint32_t qs = sb + T::OFF_Q, ks = sb + T::OFF_K, vs = sb + T::OFF_V, ps = sb + T::OFF_P;
  const uint32_t bar_s = smem_u32(&s_bar[0]), bar_o = smem_u32(&s_bar[1]);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int kvh = blockIdx.y;
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int G = p.groups, nrows = p.qlen * G, r0 = tile * BM;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_fence_init();
  }
  // Query tile, K-major: row r, channels 64b + 8c.. at block b, chunk c.
  {
    constexpr int CH = D / 8;
    const uint16_t *q = static_cast<const uint16_t *>(p.q);
    for (int i = tid; i < BM * CH; i += kThreads) {
      const int r = i / CH, c8 = i % CH, gr = r0 + r;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (gr < nrows) {
        const int pos = gr / G, h = kvh * G + gr % G;
        v = __ldg(reinterpret_cast<const uint4 *>(q + h * p.qhs + int64_t(pos) * p.qts + c8 * 8));
      }
      sts128(qs + uint32_t(c8 >> 3) * (BM * 128) + swz128(r, c8 & 7), v);
    }
  }
  fence_async_smem();
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = s_tmem;

  // Items of this CTA's history split, as in prefill_kernel.
  const int z = p.splits - 1 - int(blockIdx.z), ntiles = p.packed / BT;
  const int last_row = min(r0 + BM, nrows) - 1;
  const int rstop = min(p.resid, p.resid - p.qlen + last_row / G + 1);
  const int total = ntiles + (rstop + BT - 1) / BT;
  const int a0 = int(int64_t(total) * z / p.splits), a1 = int(int64_t(total) * (z + 1) / p.splits);
  const int i0 = min(a0, ntiles), np = min(a1, ntiles) - i0;
  const int rb = max(a0, ntiles) - ntiles, nr = max(a1, ntiles) - ntiles - rb;

  // Row state (warps 0-3: thread tid owns query row tid of the tile).
  const bool row_owner = warp < 4;
  const int gr = r0 + tid;
  const int vis = p.resid - p.qlen + (row_owner ? gr : 0) / G;
  float m = -INFINITY, l = 0.f;
  const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;

  constexpr uint32_t ID_S_PACKED = idesc<DT>(BM, BT, 0, 1);
  constexpr uint32_t ID_S_RESID = idesc<DT>(BM, BT, 0, 0);
  constexpr uint32_t ID_O = idesc<DT>(BM, D, 0, 1);

  PackedRegs<BITS, D> pr;
  if (np > 0) read_packed<BITS, D>(p, kvh, i0 * BT, tid, pr);
  const int n_items = np + nr;
  bool o_live = false;   // O holds a product (the first one overwrites)
  for (int it = 0; it < n_items; ++it) {
    const bool packed = it < np;
    const int tbase = packed ? 0 : (rb + it - np) * BT;
    // ---- this tile into shared memory ------------------------------------------
    if (packed) {
      write_packed_tc<BITS, D, DT>(pr, ks, vs, tid);
      if (it + 1 < np) read_packed<BITS, D>(p, kvh, (i0 + it + 1) * BT, tid, pr);
    } else {
      write_resid_tc<D>(p, kvh, tbase, tid, ks, vs);
    }
    fence_async_smem();
    __syncthreads();
    // ---- S = Q K^T -----------------------------------------------------------------
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t da = sdesc(qs + uint32_t(kk >> 2) * (BM * 128) + uint32_t(kk & 3) * 32, 16, 1024);
        uint64_t db;
        if (packed)   // MN-major: channel rows 16kk.. (two 8-row groups)
          db = sdesc(ks + uint32_t(kk) * 2048, T::KV_BYTES, 1024);
        else          // K-major: token rows, channels 16kk.. in block kk / 4
          db = sdesc(ks + uint32_t(kk >> 2) * (64 * 128) + uint32_t(kk & 3) * 32, 16, 1024);
        umma(tmem, da, db, packed ? ID_S_PACKED : ID_S_RESID, kk > 0);
      }
      umma_commit(bar_s);
    }
    // ---- online softmax of the tile's S rows, P into shared memory -------------------
    if (row_owner) {
      wait_bar(bar_s, uint32_t(it & 1));
      __syncwarp();   // the tensor-memory loads are warp-collective
      fence_after();
      float s[BT];
      {
        float h[32];
        tmem_ld32(tmem + lane_base + 0, h);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[j] = h[j];
        tmem_ld32(tmem + lane_base + 32, h);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[32 + j] = h[j];
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < BT; ++j) {
        float x = s[j] * p.scale_log2;
        if (!packed) {
          const int t = tbase + j;
          if (t >= p.resid || t > vis) x = -INFINITY;
        }
        s[j] = x;
        mx = fmaxf(mx, x);
      }
      float nm = fmaxf(m, mx);
      if (nm == -INFINITY) nm = 0.f;   // nothing visible yet: no inf - inf
      const float alpha = ex2(m - nm);
      m = nm;
      if (__any_sync(0xffffffffu, o_live && alpha != 1.f)) {
        // Rescale the warp's O rows (the previous tile's products are
        // complete); rows that kept their maximum multiply by 1.
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          float o[32];
          tmem_ld32(tmem + lane_base + kOCol + c, o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= alpha;
          tmem_st32(tmem + lane_base + kOCol + c, o);
        }
      }
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < BT / 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float e0 = ex2(s[8 * c + 2 * k] - m), e1 = ex2(s[8 * c + 2 * k + 1] - m);
          rs += e0 + e1;
          w[k] = E::pack2(e0, e1);
        }
        sts128(ps + swz128(tid, c), make_uint4(w[0], w[1], w[2], w[3]));
      }
      l = l * alpha + rs;
      fence_async_smem();
      fence_before();
    }
    __syncthreads();
    // ---- O += P V ------------------------------------------------------------------
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int kk = 0; kk < BT / 16; ++kk) {
        const uint64_t da = sdesc(ps + uint32_t(kk) * 32, 16, 1024);
        const uint64_t db = sdesc(vs + uint32_t(kk) * 2048, 64 * 128, 1024);
        umma(tmem + kOCol, da, db, ID_O, (o_live || kk > 0) ? 1u : 0u);
      }
      umma_commit(bar_o);
    }
    o_live = true;
    // The tiles and P are rewritten next: wait for this tile's products.
    wait_bar(bar_o, uint32_t(it & 1));
    fence_after();
  }

  // ---- epilogue: warps 0-3 read their O rows (warp-collective loads; rows
  // past the chunk load and drop) ------------------------------------------------------
  if (row_owner) {
    __syncwarp();
    const bool live = gr < nrows;
    const int pos = gr / G, head = kvh * G + gr % G;
    const int64_t orows = int64_t(p.qlen) * G * gridDim.y;
    float *rec = p.partials + (int64_t(z) * orows + int64_t(head) * p.qlen + pos) * (D + 2);
    uint16_t *row = static_cast<uint16_t *>(p.out) + (int64_t(head) * p.qlen + pos) * D;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      float o[32];
      if (o_live) {
        tmem_ld32(tmem + lane_base + kOCol + c, o);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0.f;
      }
      if (!live) continue;
      // Records are D + 2 floats apart (8-byte aligned) and `out` is only
      // required to be 4-byte aligned: pairs, not wider stores.
      if (p.splits > 1) {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          *reinterpret_cast<float2 *>(rec + c + j) = make_float2(o[j], o[j + 1]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          *reinterpret_cast<uint32_t *>(row + c + j) = E::pack2(__fdiv_rn(o[j], l), __fdiv_rn(o[j + 1], l));
      }
    }
    // A row that saw no token in this split records m = -inf (weight 0).
    if (live && p.splits > 1) *reinterpret_cast<float2 *>(rec + D) = make_float2(l > 0.f ? m : -INFINITY, l);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// ---- pipelined variant -----------------------------------------------------------
// Warps 4-11 produce (dequantize the next tiles into a second K/V buffer);
// warps 0-3 run the softmax; thread 0 issues the products.  Two S buffers
// let S(t + 1) run on the tensor cores while the softmax of tile t runs, and
// P.V of tile t runs while the softmax of tile t + 1 starts.  K and V of a
// buffer are released separately (K when S of that tile completes, V when
// P.V does), so the producers refill K early.
//
// mbarriers (phase of tile t in buffer b = t & 1 is (t >> 1) & 1):
//   full_k[b], full_v[b]   producers -> issuer (one arrival per producer)
//   s_done[b]              S(t) complete: softmax may load it; K[b] free
//   o_done[b]              P.V(t) complete: V[b] and P free, O stable
constexpr int kProducers = 256;                    // warps 4-11
constexpr int kThreads2 = 4 * 32 + kProducers;    // + the softmax warps 0-3

template <int D>
struct TCfg2 {
  static constexpr int BT = 64;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = D * BT * 2;
  static constexpr int P_BYTES = BM * BT * 2;
  static constexpr int OFF_Q = 0, OFF_KV = Q_BYTES;             // K0 V0 K1 V1
  static constexpr int OFF_P = OFF_KV + 4 * KV_BYTES;
  static constexpr int SMEM = OFF_P + P_BYTES + 1024;
  static constexpr int K_TASKS = D * (BT / 16) / kProducers;    // (channel, 16 tokens)
  static constexpr int V_TASKS = BT * (D / 16) / kProducers;    // (token, 16 channels)
  static_assert(K_TASKS * kProducers == D * (BT / 16), "K tile split");
  static_assert(V_TASKS * kProducers == BT * (D / 16), "V tile split");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

template <int BITS, int D>
struct ProdRegs {
  uint4 k[TCfg2<D>::K_TASKS];
  float2 km[TCfg2<D>::K_TASKS];
  uint4 v[TCfg2<D>::V_TASKS];
  float2 vm[TCfg2<D>::V_TASKS];
};

template <int BITS, int D>
__device__ __forceinline__ void read_packed2(const Params &p, int kvh, int t0, int ptid, ProdRegs<BITS, D> &r) {
  using C = TCfg2<D>;
  constexpr int SB = C::BT / 16;
  const int unit = t0 >> 7, s_off = t0 & 127;
  const uint8_t *kd = p.kd + kvh * p.kds_h + int64_t(unit) * p.kds_u;
  const float *km = p.km + kvh * p.kms_h + int64_t(unit) * p.kms_u;
#pragma unroll
  for (int j = 0; j < C::K_TASKS; ++j) {
    const int i = ptid + j * kProducers, d = i / SB, s0 = s_off + (i % SB) * 16;
    if constexpr (BITS == 8) {
      r.k[j] = __ldg(reinterpret_cast<const uint4 *>(kd + d * 128 + s0));
    } else {
      const uint2 x = __ldg(reinterpret_cast<const uint2 *>(kd + d * 64 + s0 / 2));
      r.k[j] = make_uint4(x.x, x.y, 0u, 0u);
    }
    r.km[j] = __ldg(reinterpret_cast<const float2 *>(km + d * 2));
  }
  constexpr int CH = D / 16;
#pragma unroll
  for (int j = 0; j < C::V_TASKS; ++j) {
    const int i = ptid + j * kProducers, t = t0 + i / CH, c0 = (i % CH) * 16;
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
__device__ __forceinline__ void write_k2(const ProdRegs<BITS, D> &r, uint32_t ks, int ptid) {
  constexpr int SB = TCfg2<D>::BT / 16;
#pragma unroll
  for (int j = 0; j < TCfg2<D>::K_TASKS; ++j) {
    const int i = ptid + j * kProducers, d = i / SB, c = (i % SB) * 2;
    uint4 lo, hi;
    dequant16<BITS, DT>(r.k[j], r.km[j].x, r.km[j].y, lo, hi);
    sts128(ks + swz128(d, c), lo);
    sts128(ks + swz128(d, c + 1), hi);
  }
}
template <int BITS, int D, int DT>
__device__ __forceinline__ void write_v2(const ProdRegs<BITS, D> &r, uint32_t vs, int ptid) {
  constexpr int CH = D / 16;
#pragma unroll
  for (int j = 0; j < TCfg2<D>::V_TASKS; ++j) {
    const int i = ptid + j * kProducers, t = i / CH, c0 = (i % CH) * 16;
    uint4 lo, hi;
    dequant16<BITS, DT>(r.v[j], r.vm[j].x, r.vm[j].y, lo, hi);
    const uint32_t blk = vs + uint32_t(c0 >> 6) * (64 * 128);
    const int c = (c0 & 63) >> 3;
    sts128(blk + swz128(t, c), lo);
    sts128(blk + swz128(t, c + 1), hi);
  }
}
// Window rows [t0, t0 + 64) of K (K-major) or V (MN-major), zero past R.
template <int D>
__device__ __forceinline__ void write_resid2(const void *src, int64_t sh, int64_t st, int kvh, int t0,
                                             int resid, int ptid, uint32_t dst) {
  constexpr int CH = D / 8;
  const uint16_t *base = static_cast<const uint16_t *>(src) + kvh * sh;
  for (int i = ptid; i < 64 * CH; i += kProducers) {
    const int t = i / CH, c8 = i % CH, tt = t0 + t;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (tt < resid) v = __ldg(reinterpret_cast<const uint4 *>(base + int64_t(tt) * st + c8 * 8));
    sts128(dst + uint32_t(c8 >> 3) * (64 * 128) + swz128(t, c8 & 7), v);
  }
}

template <int BITS, int D, int DT>
__global__ void __launch_bounds__(kThreads2, 1) prefill_tc2_kernel(const __grid_constant__ Params p) {
  using T = TCfg2<D>;
  using E = Elem<DT>;
  constexpr int BT = T::BT;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // full_k[2] full_v[2] s_done[2] o_done[2]
  __shared__ __align__(8) uint64_t s_bar[8];
  __shared__ uint32_t s_tmem;
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sb = smem_u32(smem);
  const uint32_t qs = sb + T::OFF_Q, ps = sb + T::OFF_P;
  auto kbuf = [&](int b) { return sb + T::OFF_KV + uint32_t(2 * b) * T::KV_BYTES; };
  auto vbuf = [&](int b) { return sb + T::OFF_KV + uint32_t(2 * b + 1) * T::KV_BYTES; };
  auto bar = [&](int i) { return smem_u32(&s_bar[i]); };
  constexpr int FULL_K = 0, FULL_V = 2, S_DONE = 4, O_DONE = 6;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int kvh = blockIdx.y;
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int G = p.groups, nrows = p.qlen * G, r0 = tile * BM;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(FULL_K + b), kProducers);
      mbar_init(bar(FULL_V + b), kProducers);
      mbar_init(bar(S_DONE + b), 1);
      mbar_init(bar(O_DONE + b), 1);
    }
    mbar_fence_init();
  }
  {
    constexpr int CH = D / 8;
    const uint16_t *q = static_cast<const uint16_t *>(p.q);
    for (int i = tid; i < BM * CH; i += kThreads2) {
      const int r = i / CH, c8 = i % CH, gr = r0 + r;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (gr < nrows) {
        const int pos = gr / G, h = kvh * G + gr % G;
        v = __ldg(reinterpret_cast<const uint4 *>(q + h * p.qhs + int64_t(pos) * p.qts + c8 * 8));
      }
      sts128(qs + uint32_t(c8 >> 3) * (BM * 128) + swz128(r, c8 & 7), v);
    }
  }
  fence_async_smem();
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = s_tmem;

  const int z = p.splits - 1 - int(blockIdx.z), ntiles = p.packed / BT;
  const int last_row = min(r0 + BM, nrows) - 1;
  const int rstop = min(p.resid, p.resid - p.qlen + last_row / G + 1);
  const int total = ntiles + (rstop + BT - 1) / BT;
  const int a0 = int(int64_t(total) * z / p.splits), a1 = int(int64_t(total) * (z + 1) / p.splits);
  const int i0 = min(a0, ntiles), np = min(a1, ntiles) - i0;
  const int rb = max(a0, ntiles) - ntiles, nr = max(a1, ntiles) - ntiles - rb;
  const int n_items = np + nr;
  auto tile_base = [&](int t) { return (rb + t - np) * BT; };   // window tiles

  if (warp >= 4) {
    // ---- producers ----------------------------------------------------------------
    const int ptid = tid - 4 * 32;
    ProdRegs<BITS, D> pr;
    if (np > 0) read_packed2<BITS, D>(p, kvh, i0 * BT, ptid, pr);
    for (int t = 0; t < n_items; ++t) {
      const int b = t & 1;
      const uint32_t par = uint32_t(((t - 2) >> 1) & 1);
      if (t >= 2) wait_bar(bar(S_DONE + b), par);            // S(t - 2) read K[b]
      if (t < np) write_k2<BITS, D, DT>(pr, kbuf(b), ptid);
      else write_resid2<D>(p.rk, p.rks_h, p.rks_t, kvh, tile_base(t), p.resid, ptid, kbuf(b));
      fence_async_smem();
      mbar_arrive(bar(FULL_K + b));
      if (t >= 2) wait_bar(bar(O_DONE + b), par);            // P.V(t - 2) read V[b]
      if (t < np) write_v2<BITS, D, DT>(pr, vbuf(b), ptid);
      else write_resid2<D>(p.rv, p.rvs_h, p.rvs_t, kvh, tile_base(t), p.resid, ptid, vbuf(b));
      fence_async_smem();
      mbar_arrive(bar(FULL_V + b));
      if (t + 1 < np) read_packed2<BITS, D>(p, kvh, (i0 + t + 1) * BT, ptid, pr);
    }
  } else {
    // ---- softmax warps (thread tid owns query row tid); thread 0 issues ------------
    const int gr = r0 + tid;
    const int vis = p.resid - p.qlen + gr / G;
    float m = -INFINITY, l = 0.f;
    const uint32_t lane_base = uint32_t(32 * warp) << 16;
    constexpr uint32_t ID_S_PACKED = idesc<DT>(BM, BT, 0, 1);
    constexpr uint32_t ID_S_RESID = idesc<DT>(BM, BT, 0, 0);
    constexpr uint32_t ID_O = idesc<DT>(BM, D, 0, 1);
    auto issue_s = [&](int t) {
      const int b = t & 1;
      wait_bar(bar(FULL_K + b), uint32_t((t >> 1) & 1));
      fence_after();
      const uint32_t ks = kbuf(b);
      const bool packed = t < np;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t da = sdesc(qs + uint32_t(kk >> 2) * (BM * 128) + uint32_t(kk & 3) * 32, 16, 1024);
        const uint64_t db = packed ? sdesc(ks + uint32_t(kk) * 2048, T::KV_BYTES, 1024)
                                   : sdesc(ks + uint32_t(kk >> 2) * (64 * 128) + uint32_t(kk & 3) * 32, 16, 1024);
        umma(tmem + uint32_t(b * BT), da, db, packed ? ID_S_PACKED : ID_S_RESID, kk > 0);
      }
      umma_commit(bar(S_DONE + b));
    };
    if (tid == 0 && n_items > 0) issue_s(0);
    for (int t = 0; t < n_items; ++t) {
      const int b = t & 1;
      const bool packed = t < np;
      const int tbase = packed ? 0 : tile_base(t);
      wait_bar(bar(S_DONE + b), uint32_t((t >> 1) & 1));
      __syncwarp();
      fence_after();
      float s[BT];
      {
        float h[32];
        tmem_ld32(tmem + lane_base + uint32_t(b * BT), h);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[j] = h[j];
        tmem_ld32(tmem + lane_base + uint32_t(b * BT) + 32, h);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[32 + j] = h[j];
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < BT; ++j) {
        float x = s[j] * p.scale_log2;
        if (!packed) {
          const int tt = tbase + j;
          if (tt >= p.resid || tt > vis) x = -INFINITY;
        }
        s[j] = x;
        mx = fmaxf(mx, x);
      }
      float nm = fmaxf(m, mx);
      if (nm == -INFINITY) nm = 0.f;
      const float alpha = ex2(m - nm);
      m = nm;
      float rs = 0.f;
      uint32_t w[BT / 2];
#pragma unroll
      for (int k = 0; k < BT / 2; ++k) {
        const float e0 = ex2(s[2 * k] - m), e1 = ex2(s[2 * k + 1] - m);
        rs += e0 + e1;
        w[k] = E::pack2(e0, e1);
      }
      l = l * alpha + rs;
      // S of the next tile runs on the tensor cores while this one finishes.
      if (tid == 0 && t + 1 < n_items) issue_s(t + 1);
      if (t >= 1) {
        // P.V(t - 1) must be complete: it reads P, and O is rescaled below.
        wait_bar(bar(O_DONE + ((t - 1) & 1)), uint32_t(((t - 1) >> 1) & 1));
        __syncwarp();
        fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(tmem + lane_base + kOCol + c, o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] *= alpha;
            tmem_st32(tmem + lane_base + kOCol + c, o);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < BT / 8; ++c)
        sts128(ps + swz128(tid, c), make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]));
      fence_async_smem();
      fence_before();
      named_sync(1, 4 * 32);
      if (tid == 0) {
        wait_bar(bar(FULL_V + b), uint32_t((t >> 1) & 1));
        fence_after();
#pragma unroll
        for (int kk = 0; kk < BT / 16; ++kk) {
          const uint64_t da = sdesc(ps + uint32_t(kk) * 32, 16, 1024);
          const uint64_t db = sdesc(vbuf(b) + uint32_t(kk) * 2048, 64 * 128, 1024);
          umma(tmem + kOCol, da, db, ID_O, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar(O_DONE + b));
      }
    }
    // ---- epilogue --------------------------------------------------------------------
    const bool o_live = n_items > 0;
    if (o_live) {
      const int t = n_items - 1;
      wait_bar(bar(O_DONE + (t & 1)), uint32_t((t >> 1) & 1));
    }
    __syncwarp();
    fence_after();
    const bool live = gr < nrows;
    const int pos = gr / G, head = kvh * G + gr % G;
    const int64_t orows = int64_t(p.qlen) * G * gridDim.y;
    float *rec = p.partials + (int64_t(z) * orows + int64_t(head) * p.qlen + pos) * (D + 2);
    uint16_t *row = static_cast<uint16_t *>(p.out) + (int64_t(head) * p.qlen + pos) * D;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      float o[32];
      if (o_live) {
        tmem_ld32(tmem + lane_base + kOCol + c, o);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0.f;
      }
      if (!live) continue;
      if (p.splits > 1) {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          *reinterpret_cast<float2 *>(rec + c + j) = make_float2(o[j], o[j + 1]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          *reinterpret_cast<uint32_t *>(row + c + j) = E::pack2(__fdiv_rn(o[j], l), __fdiv_rn(o[j + 1], l));
      }
    }
    if (live && p.splits > 1) *reinterpret_cast<float2 *>(rec + D) = make_float2(l > 0.f ? m : -INFINITY, l);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc

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

Params make_params(const ckv_prefill_args &a, const Plan &pl, void *workspace);

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
  const Params p = make_params(a, pl, workspace);
  const dim3 grid(unsigned(pl.tiles), unsigned(a.heads_kv), unsigned(pl.splits));
  kern<<<grid, kThreads, C::SMEM, st>>>(p);
  CKV_CUDA_TRY(cudaGetLastError());
  if (pl.splits == 1) return CKV_OK;
  return ckv_combine_partials(p.partials, pl.splits, int64_t(a.heads_q) * a.qlen, D, DT, a.seq.out,
                              reinterpret_cast<ckv_stream_t>(st));
}

Params make_params(const ckv_prefill_args &a, const Plan &pl, void *workspace) {
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
  return p;
}

// The tcgen05 kernel for D = 128 and 256 when `use_tc`; D = 64 stays on mma.sync.
template <int BITS, int D, int DT>
int launch_tc(const ckv_prefill_args &a, const Plan &pl, void *workspace, cudaStream_t st) {
  using T = tc::TCfg<D>;
  auto kern = tc::prefill_tc_kernel<BITS, D, DT>;
  static std::atomic<int> configured[64];
  int dev = 0;
  CKV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CKV_ERR_INVALID;
  if (!configured[dev].load(std::memory_order_acquire)) {
    CKV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM));
    configured[dev].store(1, std::memory_order_release);
  }
  const Params p = make_params(a, pl, workspace);
  const dim3 grid(unsigned(pl.tiles), unsigned(a.heads_kv), unsigned(pl.splits));
  kern<<<grid, kThreads, T::SMEM, st>>>(p);
  CKV_CUDA_TRY(cudaGetLastError());
  if (pl.splits == 1) return CKV_OK;
  return ckv_combine_partials(p.partials, pl.splits, int64_t(a.heads_q) * a.qlen, D, DT, a.seq.out,
                              reinterpret_cast<ckv_stream_t>(st));
}

template <int BITS, int D, int DT>
int launch_tc2(const ckv_prefill_args &a, const Plan &pl, void *workspace, cudaStream_t st) {
  using T = tc::TCfg2<D>;
  auto kern = tc::prefill_tc2_kernel<BITS, D, DT>;
  static std::atomic<int> configured[64];
  int dev = 0;
  CKV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CKV_ERR_INVALID;
  if (!configured[dev].load(std::memory_order_acquire)) {
    CKV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM));
    configured[dev].store(1, std::memory_order_release);
  }
  const Params p = make_params(a, pl, workspace);
  const dim3 grid(unsigned(pl.tiles), unsigned(a.heads_kv), unsigned(pl.splits));
  kern<<<grid, tc::kThreads2, T::SMEM, st>>>(p);
  CKV_CUDA_TRY(cudaGetLastError());
  if (pl.splits == 1) return CKV_OK;
  return ckv_combine_partials(p.partials, pl.splits, int64_t(a.heads_q) * a.qlen, D, DT, a.seq.out,
                              reinterpret_cast<ckv_stream_t>(st));
}

// 0: mma.sync; 1: tcgen05, phases in order; 2: tcgen05, pipelined.
std::atomic<int> g_use_tc{2};

template <int BITS, int D, int DT>
int launch_any(const ckv_prefill_args &a, const Plan &pl, void *workspace, cudaStream_t st) {
  if constexpr (D >= 128) {
    const int mode = g_use_tc.load(std::memory_order_relaxed);
    if (mode == 2) return launch_tc2<BITS, D, DT>(a, pl, workspace, st);
    if (mode == 1) return launch_tc<BITS, D, DT>(a, pl, workspace, st);
  }
  return launch<BITS, D, DT>(a, pl, workspace, st);
}

template <int BITS, int D>
int dispatch_dt(const ckv_prefill_args &a, const Plan &pl, void *ws, cudaStream_t st) {
  return a.dtype == CKV_BF16 ? launch_any<BITS, D, CKV_BF16>(a, pl, ws, st)
                             : launch_any<BITS, D, CKV_F16>(a, pl, ws, st);
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

extern "C" int ckv_prefill_error(int *flag, ckv_stream_t stream) {
  if (!flag) return CKV_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned v = 0;
  CKV_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, ckv::prefill::tc::g_error, sizeof(v), 0,
                                         cudaMemcpyDeviceToHost, st));
  const unsigned zero = 0;
  CKV_CUDA_TRY(cudaMemcpyToSymbolAsync(ckv::prefill::tc::g_error, &zero, sizeof(zero), 0,
                                       cudaMemcpyHostToDevice, st));
  CKV_CUDA_TRY(cudaStreamSynchronize(st));
  *flag = int(v);
  return CKV_OK;
}

extern "C" int ckv_prefill_set_tensor_cores(int on) {
  if (on < 0 || on > 2) return CKV_ERR_INVALID;
  ckv::prefill::g_use_tc.store(on);
  return CKV_OK;
}
