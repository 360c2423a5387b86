// Split-KV GQA attention over the compressed KV cache (sm_100a).
//
// One launch covers every (sequence, KV head) pair of a call.  Each pair is
// split across `cph` CTAs.  A CTA holds NCW warps in groups of GW:
//   * packed blocks (128 tokens) go to groups; the GW warps of a group split
//     a block's tokens into columns of TPW = 128/GW tokens.  Key slots (KCH
//     channels x 128 tokens, one TMA box of 128-token rows) are shared by the
//     group: the group's first warp streams them through the group's RK-slot
//     ring (full/empty mbarriers), RK-1 slots ahead of its own consumption.
//     Each warp streams its own value slots (16 tokens x all channels) and
//     residual slots through a private RV-slot ring;
//   * residual items (16 exact tokens) go to single consumer warps;
//   * every consumer warp keeps its own online-softmax state; warps merge
//     inside the CTA, CTAs merge in the last CTA of the pair (atomic ticket),
//     all in one launch.
// Packed tiles arrive by TMA (cp.async.bulk.tensor from per-sequence tensor
// maps, metadata by 1-D bulk copies); the exact residual by 16-byte
// cp.async.  Every wait on a barrier is bounded (about a second) and flags an
// error instead of hanging.
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
// dequantized straight into A fragments in registers.  MMA k-index 2qd+b
// (+8) maps to channel / token 2qd+b (+8) of the k-step; the reduction order
// is free, so rows (M) are permuted instead:
//   * key slot rows are channels of 128 (Q8) or 64 (Q4) bytes, loaded with
//     the TMA 128/64-byte swizzle (16-byte chunk c of row y lands at c ^ f(y));
//     in its column, lane r owns tokens TPL*r .. TPL*r+TPL-1 (one 4-byte
//     load per channel); for Q8 the 32 lanes hit 32 different banks;
//   * value slot rows are tokens, loaded as 128-byte swizzled boxes; lane r
//     owns CPL channels per chunk;
//   * P is stored permuted so each lane's B fragment is one 8-byte load.
#pragma once

#include <cuda.h>

#include "ckv_common.cuh"

namespace ckv {
namespace attn {

constexpr int NCW = 8;               // consumer warps per CTA (one CTA per SM)
constexpr int WARPS = NCW;           // warps holding softmax state
constexpr int THREADS = NCW * 32;
constexpr int RKMAX = 4;             // key slots per group ring (at most)
constexpr int RV = 3;                // value / residual slots per consumer ring
constexpr int PPITCH = 160;          // bytes per P row (<= 64 tokens + pad), 40 words

struct alignas(64) SeqDev {
  CUtensorMap tk;   // key codes   [H][units][D][S] bytes; box S bytes x KC channels
  CUtensorMap tv;   // value codes [H][tokens][D*bits/8] bytes; box VBOX bytes x 16 tokens
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

// Kernel parameters: a single-sequence call passes a ~400-byte block, a
// batched call the full table (launch cost grows with parameter size).
template <int MAXS>
struct alignas(64) Params : ParamsHead {
  SeqDev seq[MAXS];
};

constexpr int kMaxCph = 256;  // CTAs per (sequence, KV head), bounded by the merge scratch

template <int BITS, int D, int NT>
struct Cfg {
  static constexpr int KSTEPS = D / 16;
  static constexpr int S = 128 * BITS / 8;              // key bytes per channel row (128 tokens)
  static constexpr int KC = BITS == 8 ? 32 : 64;         // channels per key slot
  static constexpr int KCH = D < KC ? D : KC;            // channels actually in a key slot
  static constexpr int KS = D / KCH;                     // key slots per block
  static constexpr int KSLOT = KCH * S;                  // key slot bytes
  static constexpr int KSWZ = S == 128 ? 7 : 3;          // key swizzle row mask (128 / 64 B)
  static constexpr int KMETA = D * 8;                    // key (scale, low) of one block
  static constexpr int GW = BITS == 8 ? 4 : 2;           // consumer warps per group
  static constexpr int RK = GW == 4 ? RKMAX : 3;         // key slots per group ring
  static constexpr int NGRP = NCW / GW;                  // groups per CTA
  static constexpr int TPW = 128 / GW;                   // tokens per warp column
  static constexpr int TPL = TPW / 8;                    // tokens per lane (4 B of codes)
  static constexpr int MTW = TPW / 16;                   // m-tiles per column
  static constexpr int VT = 16;                          // tokens per value slot
  static constexpr int VPW = TPW / VT;                   // value slots per column
  static constexpr int VROWB = D * BITS / 8;             // bytes of one token's value codes
  static constexpr int VBOX = VROWB < 128 ? VROWB : 128; // TMA box width (bytes)
  static constexpr int NVB = VROWB / VBOX;               // boxes per value slot
  static constexpr int VSWZ = VBOX == 128 ? 7 : (VBOX == 64 ? 3 : 1);
  static constexpr int NG = D / 64;
  static constexpr int VMETA = VT * NG * 8;              // value (scale, low) of VT tokens
  static constexpr int VSLOT = VT * VROWB + VMETA;
  // Value lane mapping: lane r owns CPL channels in each of NCH chunks.
  static constexpr int CPL = BITS == 8 ? (D >= 128 ? 16 : 8) : D / 8;
  static constexpr int NCH = D / (8 * CPL);
  static constexpr int MTC = CPL / 2;                    // output m-tiles per chunk
  static constexpr int MTV = D / 16;                     // output m-tiles
  // Residual slots: keys as 16 tokens x D/2 channels, values as 8 tokens x D.
  static constexpr int RKP = D + 32 > 160 ? D + 32 : 160;          // 8 words mod 32
  static constexpr int RVP = CPL == 8 ? 2 * D + 32 : 2 * D + 16;   // 8 / 4 words mod 32
  static constexpr int RSLOT_K = 16 * RKP;
  static constexpr int RSLOT_V = 8 * RVP;
  static constexpr int PRAW = VSLOT > RSLOT_K ? (VSLOT > RSLOT_V ? VSLOT : RSLOT_V)
                                              : (RSLOT_K > RSLOT_V ? RSLOT_K : RSLOT_V);
  // Slots start on 1024-byte boundaries (required by the 128-byte swizzle).
  static constexpr int VRSLOT = (PRAW + 1023) / 1024 * 1024;        // private slot
  static constexpr int KSLOT_AL = (KSLOT + 1023) / 1024 * 1024;
  static constexpr int PBUF = 8 * NT * PPITCH;
  static constexpr int GROUP_BYTES = (RK * KSLOT_AL + 2 * KMETA + 1023) / 1024 * 1024;
  static constexpr int WARP_BYTES = (RV * VRSLOT + PBUF + 1023) / 1024 * 1024;
  static constexpr int QFRAG = KSTEPS * NT * 32 * 8;
  static constexpr int QFRAG_AL = (QFRAG + 1023) / 1024 * 1024;
  static constexpr int BODY = NGRP * GROUP_BYTES + NCW * WARP_BYTES;
  static constexpr int SMEM = 1024 + QFRAG_AL + BODY;  // + alignment slack
  static constexpr int MERGE = NCW * 8 * NT * (D + 2) * 4;
  static_assert(MERGE <= BODY, "merge scratch must fit the group and warp regions");
  static_assert(2 * 16 * kMaxCph * 4 + 16 * 2 * 4 <= BODY,
                "final-merge scratch (rows x CTAs per pair) must fit");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Offset of byte `a` of a TMA box (rows of 128/64/32 bytes) after the hardware
// swizzle: 16-byte chunk bits [4,7) XOR row bits [7,10) (128 B), [4,6) with
// [7,9) (64 B), bit 4 with bit 7 (32 B).
template <int MASK>
__device__ __forceinline__ uint32_t swz(uint32_t a) {
  return a ^ (((a >> 7) & MASK) << 4);
}

// Residual P.V token order: k-index (qd, e) -> token A[qd] + B[e] of the
// 16-token item (e = 0, 1 in the first 8 tokens, e = 2, 3 in the last 8).
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
// Position of packed token t (0..127) in the permuted P row: within each
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
  float S[C::MTW][NT][4];     // column tokens: m-tile mt, rows r / r+8 <-> TPL*r+2mt (+1)

  int lane, r, qd;
  uint32_t qf;                // query fragments (shared address)
  uint32_t ring, pbuf;        // private slot ring and P buffer
  float scale_log2;

  __device__ void init(int lane_, uint32_t qf_, uint32_t base, float sl) {
    lane = lane_;
    r = lane >> 2;
    qd = lane & 3;
    qf = qf_;
    ring = base;
    pbuf = base + RV * C::VRSLOT;
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

  __device__ __forceinline__ void zero_s() {
#pragma unroll
    for (int mt = 0; mt < C::MTW; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) S[mt][nt][c] = 0.f;
  }

  // ---------------------------------------------------------------------
  // Packed slot loads: lane 0 issues TMA tile copies (+ 1-D bulk copies of
  // the metadata) that complete on the slot's mbarrier.
  // ---------------------------------------------------------------------
  __device__ void load_packed_v(const SeqDev &sd, int head, int tok0, uint32_t slot, uint32_t bar) {
    if (lane == 0) {
      mbar_expect_tx(bar, C::VSLOT);
#pragma unroll
      for (int bx = 0; bx < C::NVB; ++bx)
        tma_load_3d(slot + bx * C::VT * C::VBOX, &sd.tv, bar, bx * C::VBOX, tok0, head);
      bulk_load(slot + C::VT * C::VROWB, sd.vm + head * sd.vm_h + int64_t(tok0) * sd.vm_t, C::VMETA,
                bar);
    }
  }

  // Residual rows [t0, t0 + rows) x channels [c0, c0 + nch) into a padded
  // slot (rows at or past `re` are zero-filled).
  __device__ void load_resid(const T *base, int64_t stride_t, int t0, int re, int rows, int c0,
                             int nch, uint32_t slot, int pitch) {
    const int chunks = nch / 8;  // 16-byte chunks per row
    for (int x = lane; x < rows * chunks; x += 32) {
      const int t = x / chunks, k = x % chunks;
      const bool ok = t0 + t < re;
      const T *src = base + (ok ? int64_t(t0 + t) * stride_t : 0) + c0 + k * 8;
      cp_async16(slot + t * pitch + k * 16, src, ok ? 16 : 0);
    }
  }

  // ---------------------------------------------------------------------
  // QK^T of this warp's column (tokens wi*TPW ..) over shared key slot ks.
  // ---------------------------------------------------------------------
  __device__ void qk_packed(uint32_t slot, int ks, int wi, uint32_t kmeta) {
    constexpr int STEPS = C::KCH / 16;
#pragma unroll 1
    for (int sl = 0; sl < STEPS; ++sl) {
      const int s = ks * STEPS + sl;   // k-step (16 channels)
      // lane's channels: 2qd, 2qd+1, 2qd+8, 2qd+9 of the k-step
      float2 sc[4], lo[4];
      uint32_t w[4];              // 4 (Q8) or 8 (Q4) tokens of one channel
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int cl = 16 * sl + 2 * qd + (e & 1) + 8 * (e >> 1);   // row in the slot
        w[e] = lds32(slot + swz<C::KSWZ>(cl * C::S + wi * (C::S / C::GW) + 4 * r));
        const float2 sm = lds64f(kmeta + (16 * s + 2 * qd + (e & 1) + 8 * (e >> 1)) * 8);
        sc[e] = make_float2(sm.x, sm.x);
        lo[e] = make_float2(sm.y, sm.y);
      }
      uint2 b[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) b[nt] = lds64(qf + ((s * NT + nt) * 32 + lane) * 8);
#pragma unroll
      for (int mt = 0; mt < C::MTW; ++mt) {
        // m-tile mt: row r <-> token TPL*r+2mt, row r+8 <-> token TPL*r+2mt+1
        float2 x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (BITS == 8) {
            x[e] = mt ? make_float2(byte_magic<2>(w[e]), byte_magic<3>(w[e]))
                      : make_float2(byte_magic<0>(w[e]), byte_magic<1>(w[e]));
          } else {
            // byte mt holds token 2mt (low nibble) and 2mt+1 (high nibble)
            const uint32_t lo4 = w[e] & 0x0F0F0F0Fu, hi4 = (w[e] >> 4) & 0x0F0F0F0Fu;
            const uint32_t sel = 0x7440u | mt;
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
        for (int nt = 0; nt < NT; ++nt) mma16816<DT>(S[mt][nt], a, b[nt].x, b[nt].y);
      }
    }
  }

  // QK^T over residual key half h (16 tokens x D/2 channels) into S[0].
  __device__ void qk_resid(uint32_t slot, int h) {
    constexpr int STEPS = C::KSTEPS / 2;
#pragma unroll 2
    for (int sl = 0; sl < STEPS; ++sl) {
      const int s = h * STEPS + sl;
      const uint32_t col = (16 * sl + 2 * qd) * 2;
      uint32_t a[4];
      a[0] = lds32(slot + r * C::RKP + col);
      a[1] = lds32(slot + (r + 8) * C::RKP + col);
      a[2] = lds32(slot + r * C::RKP + col + 16);
      a[3] = lds32(slot + (r + 8) * C::RKP + col + 16);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b = lds64(qf + ((s * NT + nt) * 32 + lane) * 8);
        mma16816<DT>(S[0][nt], a, b.x, b.y);
      }
    }
  }

  // ---------------------------------------------------------------------
  // Online softmax over the S tile; writes permuted P; rescales acc.
  //   MT       m-tiles in S
  //   tok(m,h) token (item-local) of row r (h=0) / r+8 (h=1) of m-tile m
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
  // P.V over packed value slot v (block tokens 16v..16v+15).
  // ---------------------------------------------------------------------
  __device__ void pv_packed(uint32_t slot, int v) {
    const uint32_t meta = slot + C::VT * C::VROWB;
    uint2 b[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      b[nt] = lds64(pbuf + (8 * nt + r) * PPITCH + (16 * v + 4 * qd) * 2);
#pragma unroll
    for (int ch = 0; ch < C::NCH; ++ch) {
      const int c0 = ch * 8 * C::CPL + C::CPL * r;   // lane's first channel in chunk
      const int grp = c0 / 64;
      constexpr int CB = C::CPL * BITS / 8;          // code bytes per token per chunk
      uint32_t w[4][CB / 4 > 0 ? CB / 4 : 1];
      float2 sc[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // k-index 2qd, 2qd+1, 2qd+8, 2qd+9 <-> slot token of the same index
        const int t = 2 * qd + (e & 1) + 8 * (e >> 1);
        const int off = c0 * BITS / 8;                 // byte of the lane's chunk in the row
        const uint32_t addr =
            slot + (off / C::VBOX) * C::VT * C::VBOX + swz<C::VSWZ>(t * C::VBOX + off % C::VBOX);
        if constexpr (CB == 16) {
          const uint4 x = lds128(addr);
          w[e][0] = x.x; w[e][1] = x.y; w[e][2] = x.z; w[e][3] = x.w;
        } else if constexpr (CB == 8) {
          const uint2 x = lds64(addr);
          w[e][0] = x.x; w[e][1] = x.y;
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
            const uint32_t sel = 0x7440u | (i & 3);
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
        for (int nt = 0; nt < NT; ++nt) mma16816<DT>(acc[ch * C::MTC + i][nt], a, b[nt].x, b[nt].y);
      }
    }
  }

  // P.V over residual value half h (item tokens 8h..8h+7, exact values).
  __device__ void pv_resid(uint32_t slot, int h) {
    uint2 b[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) b[nt] = lds64(pbuf + (8 * nt + r) * PPITCH + 4 * qd * 2);
    const int t0 = resid_token<C::CPL>(qd, 2 * h) - 8 * h;
    const int t1 = resid_token<C::CPL>(qd, 2 * h + 1) - 8 * h;
#pragma unroll
    for (int ch = 0; ch < C::NCH; ++ch) {
      const int c0 = ch * 8 * C::CPL + C::CPL * r;
#pragma unroll
      for (int piece = 0; piece < C::CPL / 8; ++piece) {
        const uint4 w0 = lds128(slot + t0 * C::RVP + (c0 + 8 * piece) * 2);
        const uint4 w1 = lds128(slot + t1 * C::RVP + (c0 + 8 * piece) * 2);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t x0 = (&w0.x)[k], x1 = (&w1.x)[k];
          const uint32_t lo = prmt(x0, x1, 0x5410u), hi = prmt(x0, x1, 0x7632u);
          uint32_t a[4];
          a[0] = h ? 0u : lo;
          a[1] = h ? 0u : hi;
          a[2] = h ? lo : 0u;
          a[3] = h ? hi : 0u;
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
