// Split-KV GQA attention over the compressed KV cache (sm_100a).
//
// One launch covers every (sequence, KV head) pair of a call.  Each pair is
// split across `cph` CTAs; each CTA splits its share across WARPS warps; each
// warp streams its own work items through a private two-slot ring in shared
// memory and keeps its own online-softmax state.  Packed tiles arrive by TMA
// (cp.async.bulk.tensor from per-sequence tensor maps, metadata by 1-D bulk
// copies) signalled on one mbarrier per slot; the exact residual arrives by
// 16-byte cp.async.  Warps merge inside the CTA, CTAs merge in the last CTA of
// the pair (atomic ticket), all in one launch.
//
// Work items:
//   packed block  -- 128 tokens of one KV head, consumed in "quarters" of
//                    32 (Q8) or 64 (Q4) tokens: a K slot (all channels of the
//                    quarter's tokens) then one or two V slots of 32 tokens.
//   residual item -- 16 exact bf16/fp16 tokens of the recent window.
//
// Numerics follow models/compressed_kv_kernels.py:_partial (:12-77): a code
// is dequantized as fma(code, scale, low) and rounded to the query dtype
// (:47,68); logits are the fp32 dot product times scale*log2(e) (:51); the
// softmax runs in the exp2 domain with a running max (:53-58); P is rounded
// to the query dtype before P.V (:72) while the denominator sums the fp32
// probabilities (:73); partials merge with 2^(m_s - max m) weights (:85-89).
//
// Tensor-core use: mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate) with
// tokens or channels on M and the query rows (n, g) on N.  QK^T is
// S^T[token][row] = K^T[token][channel] q^T[channel][row]; PV is
// O^T[channel][row] = V^T[channel][token] P^T[token][row].  Codes are
// dequantized straight into A fragments in registers.  Because the reduction
// order inside an MMA is free, channels and tokens are permuted so that every
// shared-memory read is conflict-free without a swizzle:
//   * K slot rows are channels (32 bytes each); A-fragment k-index 2qd+e
//     maps to channel 16s+qd+4e', so the four lanes of a row group read rows
//     8 words apart.
//   * V slot rows are tokens, loaded as 128-byte boxes with the TMA 128-byte
//     swizzle (16-byte chunk c of row t lands at chunk c ^ (t & 7)); with the
//     natural PV token order (k-index 2qd+b <-> token 2qd+b) the 8 lanes of a
//     quarter-warp read 8 different chunks.
//   * P is stored permuted so each lane's B fragment is one 8-byte load.
#pragma once

#include <cuda.h>

#include "ckv_common.cuh"

namespace ckv {
namespace attn {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int PPITCH = 160;          // bytes per P row (<= 64 tokens), 40 words

struct alignas(64) SeqDev {
  CUtensorMap tk;   // key codes   [H][units][D][S] bytes, box 32 bytes x D channels
  CUtensorMap tv;   // value codes [H][tokens][D*bits/8] bytes, box VBOX bytes x 32 tokens
  const void *q;
  const float *km;
  const float *vm;
  const void *rk;
  const void *rv;
  void *out;
  int64_t q_h, q_n;
  int64_t km_h, km_u, vm_h, vm_t;
  int64_t rk_h, rk_t, rv_h, rv_t;
  int32_t packed, length;
  int32_t ub, ue, rb, re;
  int32_t cta_begin, cph;
};

struct ParamsHead {
  int32_t num_seqs, hkv, group, nq, rows;
  int32_t partial;
  float scale_log2;
  float *rec;           // [grid][rows][D]
  float *rec_ml;        // [grid][rows][2]
  unsigned *counters;   // [num_seqs * hkv]
  unsigned *error;      // set to 1 when a wait gives up
};

// Kernel parameters: a single-sequence call passes a ~300-byte block, a
// batched call the full table (launch cost grows with parameter size).
template <int MAXS>
struct alignas(64) Params : ParamsHead {
  SeqDev seq[MAXS];
};

constexpr int kMaxCph = 256;  // CTAs per (sequence, KV head), bounded by the merge scratch

template <int BITS, int D, int NT>
struct Cfg {
  static constexpr int KSTEPS = D / 16;
  static constexpr int QT = BITS == 8 ? 32 : 64;        // tokens per K slot
  static constexpr int QPB = 128 / QT;                  // K slots per block
  static constexpr int TPL = QT / 8;                    // tokens per lane in a K slot
  static constexpr int MTQ = QT / 16;                   // m-tiles per K slot
  static constexpr int VSQ = QT / 32;                   // V slots per K slot
  static constexpr int SPB = QPB * (1 + VSQ);           // slots per packed block
  static constexpr int KSLOT = D * 32;                  // K slot bytes (TMA box 32 B x D)
  static constexpr int KMETA = D * 8;                   // key (scale, low) of one block
  static constexpr int VROWB = D * BITS / 8;            // bytes of one token's value codes
  static constexpr int VBOX = VROWB < 128 ? VROWB : 128; // TMA box width (bytes)
  static constexpr int NVB = VROWB / VBOX;              // boxes per value slot
  static constexpr int VSWZ = VBOX == 128 ? 7 : (VBOX == 64 ? 3 : 1);  // swizzle row mask
  static constexpr int NG = D / 64;
  static constexpr int VMETA = 32 * NG * 8;             // value (scale, low) of 32 tokens
  static constexpr int VSLOT = 32 * VROWB + VMETA;
  // Value lane mapping: lane r owns CPL channels in each of NCH chunks.
  static constexpr int CPL = BITS == 8 ? (D >= 128 ? 16 : 8) : D / 8;
  static constexpr int NCH = D / (8 * CPL);
  static constexpr int MTC = CPL / 2;                   // m-tiles per chunk
  static constexpr int MTV = D / 16;                    // m-tiles of the output
  // Residual slots (16 tokens of 16-bit values, padded pitch, cp.async).
  static constexpr int RKP = 2 * D + 32;
  static constexpr int RVP = CPL == 8 ? 2 * D + 32 : 2 * D + 16;
  static constexpr int RSLOT_K = 16 * RKP;
  static constexpr int RSLOT_V = 16 * RVP;
  static constexpr int SLOT_RAW = KSLOT > VSLOT ? KSLOT : VSLOT;
  static constexpr int SLOT_R = RSLOT_K > RSLOT_V ? RSLOT_K : RSLOT_V;
  // Slots start on 1024-byte boundaries (required by the 128-byte swizzle).
  static constexpr int SLOT = ((SLOT_RAW > SLOT_R ? SLOT_RAW : SLOT_R) + 1023) / 1024 * 1024;
  static constexpr int PBUF = 8 * NT * PPITCH;
  static constexpr int WARP_BYTES = (2 * SLOT + KMETA + PBUF + 1023) / 1024 * 1024;
  static constexpr int QFRAG = KSTEPS * NT * 32 * 8;    // one fragment set
  static constexpr int QFRAG_AL = (2 * QFRAG + 1023) / 1024 * 1024;
  static constexpr int SMEM = 1024 + QFRAG_AL + WARPS * WARP_BYTES;  // + alignment slack
  static constexpr int MERGE = WARPS * 8 * NT * (D + 2) * 4;
  static_assert(MERGE <= WARPS * WARP_BYTES, "merge scratch must fit the warp region");
  static_assert(2 * 16 * 256 * 4 + 16 * 2 * 4 <= WARPS * WARP_BYTES,
                "final-merge scratch (rows x CTAs per pair) must fit the warp region");
};

// Offset of byte `a` of a TMA box (rows of 128/64/32 bytes) after the hardware
// swizzle: 16-byte chunk bits [4,7) XOR row bits [7,10) (128 B), [4,6) with
// [7,9) (64 B), bit 4 with bit 7 (32 B).
template <int MASK>
__device__ __forceinline__ uint32_t swz(uint32_t a) {
  return a ^ (((a >> 7) & MASK) << 4);
}

// Residual PV token order: k-index (qd, e) -> token A[qd] + B[e].
template <int CPL>
__device__ __forceinline__ int resid_token(int qd, int e) {
  if constexpr (CPL == 16) {
    return ((qd & 1) | ((qd & 2) << 1)) + (((e & 1) << 1) | ((e & 2) << 2));
  } else {
    return qd + 4 * e;
  }
}
// Position of residual token t in the permuted P row.
template <int CPL>
__device__ __forceinline__ int resid_pos(int t) {
  if constexpr (CPL == 16) {
    int qd = (t & 1) | ((t >> 1) & 2);
    int e = ((t >> 1) & 1) | ((t >> 2) & 2);
    return 4 * qd + e;
  } else {
    return 4 * (t & 3) + (t >> 2);
  }
}
// Position of packed token t (0..63) in the permuted P row: within each
// 16-token k-step, lane qd's four tokens 2qd, 2qd+1, 2qd+8, 2qd+9 sit at
// 4qd..4qd+3 so its B fragment is one 8-byte load.
__device__ __forceinline__ int packed_pos(int t) {
  return (t & ~15) | (((t & 7) >> 1) << 2) | (((t >> 3) & 1) << 1) | (t & 1);
}

template <int BITS, int D, int NT, int DT>
struct Warp {
  using C = Cfg<BITS, D, NT>;
  using E = Elem<DT>;
  using T = typename E::T;

  // Per-lane state.
  float acc[C::MTV][NT][4];
  float m[NT][2], l[NT][2];
  float S[C::MTQ][NT][4];

  int lane, r, qd;
  uint32_t qfp, qfr;          // fragment sets (shared addresses)
  uint32_t ring, kmeta, pbuf; // per-warp shared regions
  float scale_log2;

  __device__ void init(int lane_, uint32_t qfp_, uint32_t qfr_, uint32_t base, float sl) {
    lane = lane_;
    r = lane >> 2;
    qd = lane & 3;
    qfp = qfp_;
    qfr = qfr_;
    ring = base;
    kmeta = base + 2 * C::SLOT;
    pbuf = kmeta + C::KMETA;
    scale_log2 = sl;
#pragma unroll
    for (int i = 0; i < C::MTV; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][nt][c] = 0.f;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        m[nt][j] = -INFINITY;
        l[nt][j] = 0.f;
      }
  }

  // ---------------------------------------------------------------------
  // Packed slot loads: lane 0 issues TMA tile copies (+ 1-D bulk copies of
  // the metadata) that complete on the slot's mbarrier.
  // ---------------------------------------------------------------------
  __device__ void load_packed_k(const SeqDev &sd, int head, int unit, int quarter, uint32_t slot,
                                bool with_meta, uint32_t bar) {
    if (lane == 0) {
      mbar_expect_tx(bar, C::KSLOT + (with_meta ? C::KMETA : 0));
      tma_load_4d(slot, &sd.tk, bar, quarter * 32, 0, unit, head);
      if (with_meta)
        bulk_load(kmeta, sd.km + head * sd.km_h + int64_t(unit) * sd.km_u, C::KMETA, bar);
    }
  }

  __device__ void load_packed_v(const SeqDev &sd, int head, int tok0, uint32_t slot, uint32_t bar) {
    if (lane == 0) {
      mbar_expect_tx(bar, C::VSLOT);
#pragma unroll
      for (int bx = 0; bx < C::NVB; ++bx)
        tma_load_3d(slot + bx * 32 * C::VBOX, &sd.tv, bar, bx * C::VBOX, tok0, head);
      bulk_load(slot + 32 * C::VROWB, sd.vm + head * sd.vm_h + int64_t(tok0) * sd.vm_t, C::VMETA, bar);
    }
  }

  // 16 residual tokens starting at window index t0 (rows >= re are zeroed).
  __device__ void load_resid(const void *base_, int64_t stride_t, int t0, int re, uint32_t slot,
                             int pitch) {
    const T *base = static_cast<const T *>(base_);
    constexpr int CH = D / 8;  // 16-byte chunks per row
#pragma unroll 4
    for (int x = lane; x < 16 * CH; x += 32) {
      const int t = x / CH, k = x % CH;
      const bool ok = t0 + t < re;
      const T *src = base + (ok ? int64_t(t0 + t) * stride_t : 0) + k * 8;
      cp_async16(slot + t * pitch + k * 16, src, ok ? 16 : 0);
    }
  }

  // ---------------------------------------------------------------------
  // QK^T over a packed K slot -> S (MTQ m-tiles of tokens x NT n-tiles)
  // ---------------------------------------------------------------------
  __device__ void qk_packed(uint32_t slot) {
#pragma unroll
    for (int mt = 0; mt < C::MTQ; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) S[mt][nt][c] = 0.f;
#pragma unroll 2
    for (int s = 0; s < C::KSTEPS; ++s) {
      float f[4][C::TPL];  // [channel e][token within lane]
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = 16 * s + qd + 4 * e;
        const uint32_t w = lds32(slot + c * 32 + 4 * r);
        const float2 sm = lds64f(kmeta + c * 8);
        const float2 sc = make_float2(sm.x, sm.x), lo = make_float2(sm.y, sm.y);
        if constexpr (BITS == 8) {
          float2 x0 = make_float2(byte_magic<0>(w), byte_magic<1>(w));
          float2 x1 = make_float2(byte_magic<2>(w), byte_magic<3>(w));
          x0 = __fadd2_rn(x0, make_float2(-kMagic, -kMagic));
          x1 = __fadd2_rn(x1, make_float2(-kMagic, -kMagic));
          x0 = __ffma2_rn(x0, sc, lo);
          x1 = __ffma2_rn(x1, sc, lo);
          f[e][0] = x0.x; f[e][1] = x0.y; f[e][2] = x1.x; f[e][3] = x1.y;
        } else {
          // byte b holds tokens 2b (low nibble) and 2b+1 (high nibble)
          const uint32_t lo4 = w & 0x0F0F0F0Fu, hi4 = (w >> 4) & 0x0F0F0F0Fu;
          float2 x0 = make_float2(byte_magic<0>(lo4), byte_magic<0>(hi4));
          float2 x1 = make_float2(byte_magic<1>(lo4), byte_magic<1>(hi4));
          float2 x2 = make_float2(byte_magic<2>(lo4), byte_magic<2>(hi4));
          float2 x3 = make_float2(byte_magic<3>(lo4), byte_magic<3>(hi4));
          const float2 mg = make_float2(-kMagic, -kMagic);
          x0 = __ffma2_rn(__fadd2_rn(x0, mg), sc, lo);
          x1 = __ffma2_rn(__fadd2_rn(x1, mg), sc, lo);
          x2 = __ffma2_rn(__fadd2_rn(x2, mg), sc, lo);
          x3 = __ffma2_rn(__fadd2_rn(x3, mg), sc, lo);
          f[e][0] = x0.x; f[e][1] = x0.y; f[e][2] = x1.x; f[e][3] = x1.y;
          f[e][4] = x2.x; f[e][5] = x2.y; f[e][6] = x3.x; f[e][7] = x3.y;
        }
      }
      uint2 b[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) b[nt] = lds64(qfp + ((s * NT + nt) * 32 + lane) * 8);
#pragma unroll
      for (int mt = 0; mt < C::MTQ; ++mt) {
        // m-tile mt: row r <-> lane token 2mt, row r+8 <-> lane token 2mt+1
        uint32_t a[4];
        a[0] = E::pack2(f[0][2 * mt], f[1][2 * mt]);
        a[1] = E::pack2(f[0][2 * mt + 1], f[1][2 * mt + 1]);
        a[2] = E::pack2(f[2][2 * mt], f[3][2 * mt]);
        a[3] = E::pack2(f[2][2 * mt + 1], f[3][2 * mt + 1]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<DT>(S[mt][nt], a, b[nt].x, b[nt].y);
      }
    }
  }

  // QK^T over a residual K slot (16 tokens, one m-tile) -> S[0]
  __device__ void qk_resid(uint32_t slot) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) S[0][nt][c] = 0.f;
#pragma unroll 4
    for (int s = 0; s < C::KSTEPS; ++s) {
      const uint2 w0 = lds64(slot + r * C::RKP + (16 * s + 4 * qd) * 2);
      const uint2 w1 = lds64(slot + (r + 8) * C::RKP + (16 * s + 4 * qd) * 2);
      uint32_t a[4] = {w0.x, w1.x, w0.y, w1.y};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b = lds64(qfr + ((s * NT + nt) * 32 + lane) * 8);
        mma16816<DT>(S[0][nt], a, b.x, b.y);
      }
    }
  }

  // ---------------------------------------------------------------------
  // Online softmax over the S tile; writes permuted P; rescales acc.
  //   MT       m-tiles in S
  //   tok(m,h) token (slot-local) of row r (h=0) / r+8 (h=1) of m-tile m
  //   valid(t, row) mask (true for packed tokens)
  //   pos(t)   column of token t in the permuted P row
  // ---------------------------------------------------------------------
  template <int MT, class Tok, class Valid, class Pos>
  __device__ void softmax(Tok tok, Valid valid, Pos pos) {
    float alpha[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int row = 8 * nt + 2 * qd + j;
        float v[2 * MT];
        float mx = -INFINITY;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float x = S[mt][nt][2 * h + j] * scale_log2;
            if (!valid(tok(mt, h), row)) x = -INFINITY;
            v[2 * mt + h] = x;
            mx = fmaxf(mx, x);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mnew = fmaxf(m[nt][j], mx);
        const float muse = mnew == -INFINITY ? 0.f : mnew;
        alpha[nt][j] = ex2(m[nt][j] - muse);
        m[nt][j] = mnew;
        float sum = 0.f;
        const uint32_t prow = pbuf + row * PPITCH;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float p = ex2(v[2 * mt + h] - muse);
            sum += p;
            const T ph = E::from_f32(p);
            const uint16_t bits = *reinterpret_cast<const uint16_t *>(&ph);
            asm volatile("st.shared.u16 [%0], %1;" ::"r"(prow + pos(tok(mt, h)) * 2), "h"(bits));
          }
        }
        l[nt][j] = l[nt][j] * alpha[nt][j] + sum;
      }
    }
    bool unit = true;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) unit = unit && alpha[nt][0] == 1.f && alpha[nt][1] == 1.f;
    if (!__all_sync(0xffffffffu, unit)) {
#pragma unroll
      for (int i = 0; i < C::MTV; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float2 al = make_float2(alpha[nt][0], alpha[nt][1]);
          float2 x0 = __fmul2_rn(make_float2(acc[i][nt][0], acc[i][nt][1]), al);
          float2 x1 = __fmul2_rn(make_float2(acc[i][nt][2], acc[i][nt][3]), al);
          acc[i][nt][0] = x0.x; acc[i][nt][1] = x0.y;
          acc[i][nt][2] = x1.x; acc[i][nt][3] = x1.y;
        }
    }
  }

  // ---------------------------------------------------------------------
  // P.V over a packed V slot of 32 tokens; kbase = first PV k-step of the
  // slot within the current K slot's P row.
  // ---------------------------------------------------------------------
  __device__ void pv_packed(uint32_t slot, int kbase) {
    const uint32_t meta = slot + 32 * C::VROWB;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint2 b[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        b[nt] = lds64(pbuf + (8 * nt + r) * PPITCH + (16 * (kbase + j) + 4 * qd) * 2);
#pragma unroll
      for (int ch = 0; ch < C::NCH; ++ch) {
        const int c0 = ch * 8 * C::CPL + C::CPL * r;   // lane's first channel in chunk
        const int grp = c0 / 64;
        constexpr int CB = C::CPL * BITS / 8;           // code bytes per token per chunk
        uint32_t w[4][CB / 4 > 0 ? CB / 4 : 1];
        float2 sc[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // k-index 2qd, 2qd+1, 2qd+8, 2qd+9 <-> slot token 16j + the same
          const int t = 16 * j + 2 * qd + (e & 1) + 8 * (e >> 1);
          const int off = c0 * BITS / 8;                 // byte of the lane's chunk in the row
          const uint32_t addr = slot + (off / C::VBOX) * 32 * C::VBOX +
                                swz<C::VSWZ>(t * C::VBOX + off % C::VBOX);
          if constexpr (CB == 16) {
            uint4 v = lds128(addr);
            w[e][0] = v.x; w[e][1] = v.y; w[e][2] = v.z; w[e][3] = v.w;
          } else if constexpr (CB == 8) {
            uint2 v = lds64(addr);
            w[e][0] = v.x; w[e][1] = v.y;
          } else {
            w[e][0] = lds32(addr);
          }
          const float2 sm = lds64f(meta + (t * C::NG + grp) * 8);
          sc[e] = make_float2(sm.x, sm.x);
          lo[e] = make_float2(sm.y, sm.y);
        }
#pragma unroll
        for (int i = 0; i < C::MTC; ++i) {
          // channels c0 + 2i (row r) and c0 + 2i + 1 (row r+8)
          float2 x[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if constexpr (BITS == 8) {
              const uint32_t word = w[e][i >> 1];
              x[e] = (i & 1) ? make_float2(byte_magic<2>(word), byte_magic<3>(word))
                             : make_float2(byte_magic<0>(word), byte_magic<1>(word));
            } else {
              const uint32_t word = w[e][i >> 2];
              const uint32_t lo4 = word & 0x0F0F0F0Fu, hi4 = (word >> 4) & 0x0F0F0F0Fu;
              const int bsel = i & 3;
              const uint32_t sel = 0x7440u | bsel;
              x[e] = make_float2(__uint_as_float(prmt(lo4, 0x4B000000u, sel)),
                                 __uint_as_float(prmt(hi4, 0x4B000000u, sel)));
            }
            x[e] = __ffma2_rn(__fadd2_rn(x[e], make_float2(-kMagic, -kMagic)), sc[e], lo[e]);
          }
          uint32_t a[4];
          a[0] = E::pack2(x[0].x, x[1].x);
          a[1] = E::pack2(x[0].y, x[1].y);
          a[2] = E::pack2(x[2].x, x[3].x);
          a[3] = E::pack2(x[2].y, x[3].y);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma16816<DT>(acc[ch * C::MTC + i][nt], a, b[nt].x, b[nt].y);
        }
      }
    }
  }

  // P.V over a residual V slot (16 tokens, exact values).
  __device__ void pv_resid(uint32_t slot) {
    uint2 b[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) b[nt] = lds64(pbuf + (8 * nt + r) * PPITCH + 4 * qd * 2);
#pragma unroll
    for (int ch = 0; ch < C::NCH; ++ch) {
      const int c0 = ch * 8 * C::CPL + C::CPL * r;
#pragma unroll
      for (int piece = 0; piece < C::CPL / 8; ++piece) {
        uint4 w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = resid_token<C::CPL>(qd, e);
          w[e] = lds128(slot + t * C::RVP + (c0 + 8 * piece) * 2);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t w0 = (&w[0].x)[k], w1 = (&w[1].x)[k], w2 = (&w[2].x)[k],
                         w3 = (&w[3].x)[k];
          uint32_t a[4];
          a[0] = prmt(w0, w1, 0x5410u);
          a[1] = prmt(w0, w1, 0x7632u);
          a[2] = prmt(w2, w3, 0x5410u);
          a[3] = prmt(w2, w3, 0x7632u);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma16816<DT>(acc[ch * C::MTC + piece * 4 + k][nt], a, b[nt].x, b[nt].y);
        }
      }
    }
  }

  // Channel of acc[i][*][c] for this lane (c = 0,1 -> row r; 2,3 -> row r+8).
  __device__ __forceinline__ int out_channel(int i, int c) const {
    return (i / C::MTC) * 8 * C::CPL + C::CPL * r + 2 * (i % C::MTC) + (c >> 1);
  }
};

}  // namespace attn
}  // namespace ckv
