// Split-KV GQA attention over the compressed KV cache (sm_100a).
//
// One launch covers every (sequence, KV head) pair of a call.  A pair's work
// items -- packed 128-token blocks, then 64-token chunks of the exact
// residual window -- are split into contiguous ranges, one per CTA; the CTAs
// of a pair merge their partial results in the last CTA to finish (atomic
// ticket), all in the same launch.
//
// Inside a CTA the roles are specialised.  Two teams take alternate items
// (team t owns items t, t+2, ...) with their own online-softmax state, so one
// team's synchronisation latency is covered by the other team's arithmetic;
// the two states merge once at the end.
//
//   2 producers    the K warp streams K stages (key codes by one TMA tile
//                  copy, [D channels][128 tokens] bytes, 128/64-byte swizzle,
//                  plus the block's (scale, low) by a 1-D bulk copy); the V
//                  warp streams V stages ([128 tokens][D*bits/8] bytes in
//                  boxes of up to 128 bytes, swizzled, plus per-token
//                  metadata).  Residual chunks arrive by 16-byte cp.async from
//                  all 32 lanes into padded rows.  Stages are rings of NK / NV
//                  buffers guarded by full/empty mbarriers, shared by the
//                  teams.
//   4 QK warps     per team; warp q owns token quarter q of a block (32
//                  tokens) over all channels: logits with mma.sync m16n8k16,
//                  then P = 2^(s - m_q) (query dtype) into the team's double
//                  buffer.  Each warp keeps its own running row maximum m_q,
//                  rounded up to an integer so that moving between the
//                  warps' scales is an exact power of two; the warps never
//                  wait for each other.
//   4 PV warps     per team; warp c owns channel quarter c (D/4 channels) over
//                  all tokens of the item.  It takes the item's common scale
//                  M = max(M, m_0..m_3), rescales its accumulator by 2^(M_old -
//                  M) and each QK warp's P fragments by 2^(m_q - M), then
//                  O += P.V.
//
// Numerics follow models/compressed_kv_kernels.py:_partial (:12-77): a code
// is dequantized as fma(code, scale, low) and rounded to the query dtype
// (:47,68); logits are the fp32 dot product times scale*log2(e) (:51); the
// softmax runs in the exp2 domain with a running max (:53-58); P is rounded
// to the query dtype before P.V (:72) while the denominator sums the fp32
// probabilities (:73); partials merge with 2^(m_s - max m) weights (:85-89).
//
// Tensor-core use is mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate) with
// tokens (QK) or channels (PV) on M and the query rows (position n, group
// member g) on N: the row count is at most 16, far too small for the
// shared-memory operands of the 5th-generation MMA, while the dequantized
// codes can go from registers straight into mma.sync fragments.
#pragma once

#include <cuda.h>

#include "ckv_common.cuh"

namespace ckv {
namespace attn {

constexpr int TEAMS = 2;
constexpr int TEAM_WARPS = 4;                    // QK warps (and PV warps) per team
constexpr int QK_WARPS = TEAMS * TEAM_WARPS;     // warps [0, 8): QK, team = w / 4
constexpr int PV_WARPS = TEAMS * TEAM_WARPS;     // warps [8, 16): PV, team = (w - 8) / 4
constexpr int PRODUCER = QK_WARPS + PV_WARPS;    // K producer warp; PRODUCER + 1: V
constexpr int WARPS = PRODUCER + 2;
constexpr int THREADS = WARPS * 32;
constexpr int TEAM_THREADS = TEAM_WARPS * 32;
constexpr int RCHUNK = 64;                       // residual tokens per work item
constexpr int NK = 3;                            // K stage ring depth
constexpr int PP = 288;                          // P row pitch: 128 tokens + 16-byte pad
constexpr int BAR_QFRAG = 1;                     // named barrier of the QK warps (query fragments)

struct alignas(64) SeqDev {
  CUtensorMap tk;   // key codes   [H][units][D][S] bytes, box S bytes x D channels
  CUtensorMap tv;   // value codes [H][tokens][D*bits/8] bytes, box VBOX bytes x 128 tokens
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
  float *rec_ml;        // [grid][ml_stride(rows)]: (m, l) per row
  unsigned *counters;   // [num_seqs * hkv]
  unsigned *error;      // set to 1 when a wait gives up
};

// Kernel parameters: a single-sequence call passes a ~300-byte block, a
// batched call the full table (launch cost grows with parameter size).
template <int MAXS>
struct alignas(64) Params : ParamsHead {
  SeqDev seq[MAXS];
};

constexpr int kMaxCph = 160;  // CTAs per (sequence, KV head): one wave of SMs, bounded by the merge scratch

constexpr int align1k(int x) { return (x + 1023) / 1024 * 1024; }
// Floats per CTA in the (m, l) record array: two per row, padded to 16 bytes
// so that the records of consecutive CTAs form one bulk copy.
__host__ __device__ constexpr int ml_stride(int rows) { return (rows * 2 + 3) & ~3; }
constexpr int cmax(int a, int b) { return a > b ? a : b; }

template <int BITS, int D, int NT>
struct Cfg {
  static constexpr int ROWS = 8 * NT;                   // query rows incl. padding
  // K stage: codes [D][SB] (one row per channel, 128 tokens) then (scale, low)[D].
  static constexpr int SB = 128 * BITS / 8;
  static constexpr int KCODE = D * SB;
  static constexpr int KMETA = D * 8;
  // Residual chunk: RCHUNK rows of D 16-bit values, padded pitch.
  static constexpr int RP = 2 * D + 16;
  static constexpr int RBYTES = RCHUNK * RP;
  static constexpr int KST = align1k(cmax(KCODE + KMETA, RBYTES));
  // V stage: codes [128][VROWB] in NVB boxes of VBOX bytes, then (scale, low)[128][NG].
  static constexpr int VROWB = D * BITS / 8;
  static constexpr int VBOX = VROWB < 128 ? VROWB : 128;
  static constexpr int NVB = VROWB / VBOX;
  static constexpr int VSWZ = VBOX == 128 ? 7 : (VBOX == 64 ? 3 : 1);  // swizzle row mask
  static constexpr int KSWZ = SB == 128 ? 7 : 3;
  static constexpr int NG = D / 64;
  static constexpr int VCODE = 128 * VROWB;
  static constexpr int VMETA = 128 * NG * 8;
  static constexpr int VST = align1k(cmax(VCODE + VMETA, RBYTES));
  static constexpr int NV = NT == 1 ? 3 : 2;            // V stage ring depth
  // QK: each warp covers all D channels in KQS k-steps of 16.
  static constexpr int KQS = D / 16;
  // PV: each warp covers D/4 channels, CPL per lane, MTV m-tiles.
  static constexpr int CPL = D / 32;
  static constexpr int MTV = CPL / 2;
  // Shared-memory map (offsets from a 1024-byte aligned base).
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + NK * KST;
  static constexpr int OFF_Q = OFF_V + NV * VST;                   // [KQS][NT][32] query B fragments
  static constexpr int OFF_P = OFF_Q + KQS * NT * 32 * 8;          // [TEAMS][2][ROWS][PP]
  static constexpr int OFF_XM = OFF_P + TEAMS * 2 * ROWS * PP;     // [TEAMS][2][4][ROWS] P scales m_q
  static constexpr int OFF_END = OFF_XM + TEAMS * 2 * TEAM_WARPS * ROWS * 4;
  static constexpr int SMEM = OFF_END + 1024;                      // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // End-of-CTA scratch (reuses the stage rings).
  static constexpr int RED = TEAMS * ROWS * D * 4;                 // [team][ROWS][D]
  static_assert(RED + 64 * ROWS * 4 <= NK * KST + NV * VST, "reduction scratch");
  // Merge scratch: (m, l) records, weights, the rows' (M, L), the partial
  // sums of the record parts, then at least one record.
  static_assert(kMaxCph * (ml_stride(ROWS) + ROWS) * 4 + 2 * ROWS * 4 + 16 + THREADS * 16 + 128 +
                        ROWS * D * 4 <=
                    NK * KST + NV * VST,
                "merge scratch");
};

// Offset of byte `a` of a TMA box (rows of 128/64/32 bytes) after the hardware
// swizzle: 16-byte chunk bits [4,7) XOR row bits [7,10) (128 B), [4,6) with
// [7,9) (64 B), bit 4 with bit 7 (32 B).
template <int MASK>
__device__ __forceinline__ uint32_t swz(uint32_t a) {
  return a ^ (((a >> 7) & MASK) << 4);
}

// Position of token t of an item in a P row: within each 16-token k-step,
// lane qd's four tokens 2qd, 2qd+1, 2qd+8, 2qd+9 sit at 4qd..4qd+3 so a PV
// lane reads its B fragment with one 8-byte load.
__device__ __forceinline__ int ppos(int t) {
  return (t & ~15) | (((t & 7) >> 1) << 2) | (((t >> 3) & 1) << 1) | (t & 1);
}

template <class T>
__device__ __forceinline__ T lds(const uint8_t *base, uint32_t off) {
  return *reinterpret_cast<const T *>(base + off);
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// 2^d for an integer-valued d <= 0; 0 below the normal range and for -inf
// or NaN (the difference of two -inf scales).
__device__ __forceinline__ float pow2i(float d) {
  return !(d >= -126.f) ? 0.f : __int_as_float((int(d) + 127) << 23);
}

// Nibble K (bits [4K, 4K + 4), K < 5) of w as the exact float 2^(23-4K) + code:
// the nibble lands in the mantissa bits whose weights are 2^0..2^3 under
// that exponent, so one and-or forms it.
template <int K>
__device__ __forceinline__ float nib_magic(uint32_t w) {
  static_assert(K >= 0 && K < 5, "nibble above the mantissa");
  return __uint_as_float((w & (0xFu << (4 * K))) | (uint32_t(127 + 23 - 4 * K) << 23));
}
// (-2^(23-4K), -2^(19-4K)): takes the offsets of nibbles K and K + 1 away.
template <int K>
__device__ __forceinline__ float2 nib_bias() {
  return make_float2(-__uint_as_float(uint32_t(127 + 23 - 4 * K) << 23),
                     -__uint_as_float(uint32_t(127 + 19 - 4 * K) << 23));
}

// Two codes held as 2^23 + code -> fma(code, scale, low) in fp32.
__device__ __forceinline__ float2 dq2(float2 magic, float sc, float lo) {
  const float2 c = __fadd2_rn(magic, make_float2(-kMagic, -kMagic));
  return make_float2(__fmaf_rn(c.x, sc, lo), __fmaf_rn(c.y, sc, lo));
}
// The same with (scale, scale) and (low, low) already paired.
__device__ __forceinline__ float2 dq2p(float2 magic, float2 sc, float2 lo) {
  return __ffma2_rn(__fadd2_rn(magic, make_float2(-kMagic, -kMagic)), sc, lo);
}

// The swizzle's XOR term for a row r of a 1024-byte swizzle atom depends only
// on r's low bits (r & 7 for 128-byte rows, (r >> 1) & 3 for 64-byte rows,
// (r >> 2) & 1 for 32-byte rows).  Rows that differ by a multiple of 8 share
// it, so a lane computes its swizzled column once per row residue and adds
// row * pitch for every other row.
template <int MASK, int PITCH>
__device__ __forceinline__ uint32_t swz_col(int row_rep, int col) {
  return swz<MASK>(row_rep * PITCH + col) - row_rep * PITCH;
}

// ---------------------------------------------------------------------------
// QK warp: partial logits of one item over half of the channels.
// ---------------------------------------------------------------------------
template <int BITS, int D, int NT, int DT>
struct QkWarp {
  using C = Cfg<BITS, D, NT>;
  using E = Elem<DT>;
  int lane, r, qd, q;
  const uint8_t *qfr;   // query B fragments [KQS][NT][32] (shared memory)

  __device__ __forceinline__ uint2 qfrag(int s, int nt) const {
    return lds<uint2>(qfr, ((s * NT + nt) * 32 + lane) * 8);
  }

  // S[mt][nt][c]: tokens 32q + 4r + 2mt (c = 0, 1) and 32q + 4r + 2mt + 1
  // (c = 2, 3), query rows 8nt + 2qd + (c & 1).
  __device__ void packed(const uint8_t *kst, float (&S)[2][NT][4]) const {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) S[mt][nt][c] = 0.f;
    const uint8_t *meta = kst + C::KCODE;
    // Channel rows 2qd + e_lo + 8 e_hi + 16 s share the swizzle term of
    // 2qd + e_lo.
    const int col = BITS == 8 ? 32 * q + 4 * r : 16 * q + 2 * r;
    const uint8_t *krow[2];
#pragma unroll
    for (int el = 0; el < 2; ++el)
      krow[el] = kst + (2 * qd + el) * C::SB + swz_col<C::KSWZ, C::SB>(2 * qd + el, col);
#pragma unroll 4
    for (int s = 0; s < C::KQS; ++s) {
      const int cb = 16 * s + 2 * qd;   // channels cb, cb+1, cb+8, cb+9
      const float4 m0 = lds<float4>(meta, cb * 8);
      const float4 m1 = lds<float4>(meta, (cb + 8) * 8);
      const float sc[4] = {m0.x, m0.z, m1.x, m1.z};
      const float lo[4] = {m0.y, m0.w, m1.y, m1.w};
      float f[4][4];  // [channel e][token j]
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint8_t *src = krow[e & 1] + (16 * s + 8 * (e >> 1)) * C::SB;
        float2 x0, x1;
        if constexpr (BITS == 8) {
          const uint32_t w = *reinterpret_cast<const uint32_t *>(src);
          x0 = make_float2(byte_magic<0>(w), byte_magic<1>(w));
          x1 = make_float2(byte_magic<2>(w), byte_magic<3>(w));
        } else {
          // two bytes: tokens 4r+0 (low nibble), +1 (high), +2, +3; nibble k
          // becomes 2^(23-4k) + code with one logic op (nib_magic).
          const uint32_t w = *reinterpret_cast<const uint16_t *>(src);
          x0 = make_float2(nib_magic<0>(w), nib_magic<1>(w));
          x1 = make_float2(nib_magic<2>(w), nib_magic<3>(w));
        }
        const float2 sc2 = make_float2(sc[e], sc[e]), lo2 = make_float2(lo[e], lo[e]);
        if constexpr (BITS == 8) {
          x0 = dq2p(x0, sc2, lo2);
          x1 = dq2p(x1, sc2, lo2);
        } else {
          x0 = __ffma2_rn(__fadd2_rn(x0, nib_bias<0>()), sc2, lo2);
          x1 = __ffma2_rn(__fadd2_rn(x1, nib_bias<2>()), sc2, lo2);
        }
        f[e][0] = x0.x; f[e][1] = x0.y; f[e][2] = x1.x; f[e][3] = x1.y;
      }
      uint2 b[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) b[nt] = qfrag(s, nt);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
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

  // Residual chunk: one m-tile of tokens 16q + r (c = 0, 1) and 16q + r + 8
  // (c = 2, 3).
  __device__ void resid(uint32_t kst, float (&S)[NT][4]) const {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) S[nt][c] = 0.f;
    const int row = 16 * q + (lane & 7) + 8 * ((lane >> 3) & 1);
    const uint32_t base = kst + row * C::RP + 8 * (lane >> 4) * 2;
#pragma unroll
    for (int s = 0; s < C::KQS; ++s) {
      uint32_t a[4];
      ldmatrix_x4(a, base + 32 * s);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b = qfrag(s, nt);
        mma16816<DT>(S[nt], a, b.x, b.y);
      }
    }
  }
};

// ---------------------------------------------------------------------------
// PV warp: O += P.V over one item's token half and channel quarter.
// O[i][nt][c]: channel (D/4)c + CPL r + 2i + (c >> 1), query row 8nt + 2qd + (c & 1).
// ---------------------------------------------------------------------------
template <int BITS, int D, int NT, int DT>
struct PvWarp {
  using C = Cfg<BITS, D, NT>;
  using E = Elem<DT>;
  int lane, r, qd, c;

  // fb[q][nt]: packed factor pair for the P fragments written by QK warp q
  // (applied when `scaled`).
  __device__ void packed(const uint8_t *vst, const uint8_t *pb, float (&O)[C::MTV][NT][4],
                         const uint32_t (&fb)[TEAM_WARPS][NT], bool scaled) const {
    constexpr int CB = C::CPL * BITS / 8;            // code bytes per lane per token
    const int off = ((D / 4) * c + C::CPL * r) * BITS / 8;   // lane's first byte in a row
    const uint8_t *box = vst + (off / C::VBOX) * 128 * C::VBOX;
    const int inb = off % C::VBOX;
    const int grp = ((D / 4) * c) / 64;
    // Token rows t = t0 + e_lo + 8 e_hi + 16 j with t0 = 2 qd share the
    // swizzle term of 2 qd + e_lo.
    const int t0 = 2 * qd;
    const uint8_t *vrow[2];
#pragma unroll
    for (int el = 0; el < 2; ++el)
      vrow[el] = box + (t0 + el) * C::VBOX + swz_col<C::VSWZ, C::VBOX>(2 * qd + el, inb);
    const uint8_t *meta = vst + C::VCODE + (t0 * C::NG + grp) * 8;
    const uint8_t *prow = pb + r * PP + 4 * qd * 2;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint2 b[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        b[nt] = lds<uint2>(prow, 8 * nt * PP + 32 * j);
        if (scaled) {
          b[nt].x = E::mul2(b[nt].x, fb[j >> 1][nt]);
          b[nt].y = E::mul2(b[nt].y, fb[j >> 1][nt]);
        }
      }
      uint32_t w[4][CB >= 4 ? CB / 4 : 1];
      float2 sc[4], lo[4];   // one token's (scale, low), paired for its CPL channels
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int dt = 16 * j + 8 * (e >> 1);       // token offset beyond t0 + e_lo
        const uint8_t *src = vrow[e & 1] + dt * C::VBOX;
        if constexpr (CB == 8) {
          const uint2 v = *reinterpret_cast<const uint2 *>(src);
          w[e][0] = v.x; w[e][1] = v.y;
        } else if constexpr (CB == 4) {
          w[e][0] = *reinterpret_cast<const uint32_t *>(src);
        } else if constexpr (CB == 2) {
          w[e][0] = *reinterpret_cast<const uint16_t *>(src);
        } else {
          w[e][0] = *src;
        }
        const float2 sm = lds<float2>(meta, ((dt + (e & 1)) * C::NG) * 8);
        sc[e] = make_float2(sm.x, sm.x);
        lo[e] = make_float2(sm.y, sm.y);
      }
#pragma unroll
      for (int i = 0; i < C::MTV; ++i) {
        // channels CPL r + 2i (row r) and CPL r + 2i + 1 (row r + 8)
        float2 x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (BITS == 8) {
            const uint32_t word = w[e][i >> 1];
            x[e] = (i & 1) ? make_float2(byte_magic<2>(word), byte_magic<3>(word))
                           : make_float2(byte_magic<0>(word), byte_magic<1>(word));
          } else {
            // byte i holds channel 2i (low nibble) and 2i + 1 (high nibble)
            const uint32_t word = w[e][i >> 2];
            const uint32_t lo4 = word & 0x0F0F0F0Fu, hi4 = (word >> 4) & 0x0F0F0F0Fu;
            const uint32_t sel = 0x7440u | (i & 3);
            x[e] = make_float2(__uint_as_float(prmt(lo4, 0x4B000000u, sel)),
                               __uint_as_float(prmt(hi4, 0x4B000000u, sel)));
          }
          x[e] = dq2p(x[e], sc[e], lo[e]);
        }
        uint32_t a[4];
        a[0] = E::pack2(x[0].x, x[1].x);
        a[1] = E::pack2(x[0].y, x[1].y);
        a[2] = E::pack2(x[2].x, x[3].x);
        a[3] = E::pack2(x[2].y, x[3].y);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<DT>(O[i][nt], a, b[nt].x, b[nt].y);
      }
    }
  }

  // Residual chunk: exact 16-bit values, tokens 16j + {2qd, 2qd+1, 2qd+8, 2qd+9}.
  __device__ void resid(const uint8_t *vst, const uint8_t *pb, float (&O)[C::MTV][NT][4],
                        const uint32_t (&fb)[TEAM_WARPS][NT], bool scaled) const {
    const uint32_t coff = ((D / 4) * c + C::CPL * r) * 2;
#pragma unroll
    for (int j = 0; j < RCHUNK / 16; ++j) {
      const int t0 = 16 * j + 2 * qd;
      uint2 b[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        b[nt] = lds<uint2>(pb, (8 * nt + r) * PP + (16 * j + 4 * qd) * 2);
        if (scaled) {
          b[nt].x = E::mul2(b[nt].x, fb[j][nt]);
          b[nt].y = E::mul2(b[nt].y, fb[j][nt]);
        }
      }
      uint32_t w[4][C::MTV];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = t0 + (e & 1) + 8 * (e >> 1);
        const uint32_t a = t * C::RP + coff;
        if constexpr (C::MTV == 4) {
          const uint4 v = lds<uint4>(vst, a);
          w[e][0] = v.x; w[e][1] = v.y; w[e][2] = v.z; w[e][3] = v.w;
        } else if constexpr (C::MTV == 2) {
          const uint2 v = lds<uint2>(vst, a);
          w[e][0] = v.x; w[e][1] = v.y;
        } else {
          w[e][0] = lds<uint32_t>(vst, a);
        }
      }
#pragma unroll
      for (int i = 0; i < C::MTV; ++i) {
        uint32_t a[4];
        a[0] = prmt(w[0][i], w[1][i], 0x5410u);
        a[1] = prmt(w[0][i], w[1][i], 0x7632u);
        a[2] = prmt(w[2][i], w[3][i], 0x5410u);
        a[3] = prmt(w[2][i], w[3][i], 0x7632u);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<DT>(O[i][nt], a, b[nt].x, b[nt].y);
      }
    }
  }
};

}  // namespace attn
}  // namespace ckv
