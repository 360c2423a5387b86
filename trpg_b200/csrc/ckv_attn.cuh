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

// FOLD selects the folded dequantization (see QkWarp::packed_fold and
// PvWarp::packed_fold); false is the exact per-element rule.
template <int BITS, int D, int NT, bool FOLD = false>
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
  // Query fragments per (k-step, n-tile, lane): two 16-bit pairs (8 bytes).
  static constexpr int QFRAG = 8;
  static constexpr int OFF_Q = OFF_V + NV * VST;                   // [KQS][NT][32] query fragments
  static constexpr int OFF_P = OFF_Q + KQS * NT * 32 * QFRAG;      // [TEAMS][2][ROWS][PP]
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

// Four 8x8 matrices of 16-bit elements, transposed on the way into registers
// (lane 4r + qd receives rows 2qd and 2qd + 1 of column r of each matrix).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// Two fp32 values -> fp16 pair (`lo` in the low half), rounded to nearest,
// saturating at the largest finite fp16 instead of overflowing to inf.
__device__ __forceinline__ uint32_t f16x2_sat(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// fp16 pair (1024, 1024): the constant operand that measures the offset of
// the exponent-bias conversion below.
constexpr uint32_t kF16Pair1024 = 0x64006400u;

// Bytes 0 and 2 (kLo) or 1 and 3 (kHi) of w as the fp16 pair (1024 + byte):
// the byte becomes the low mantissa bits under the exponent of 1024 (the
// exponent-bias conversion of Kim et al., "Who Says Elephants Can't Run",
// 2022).  One PRMT per two codes.
constexpr uint32_t kSelLo = 0x4240u, kSelHi = 0x4341u;
template <uint32_t SEL>
__device__ __forceinline__ uint32_t byte_pair_f16(uint32_t w) {
  return prmt(w, 0x64646464u, SEL);
}
// The same for 4-bit codes: nibble 0 (T = 0), 1, 2 or 3 of bytes 0 and 2
// as (1024 + code) for even T and (1024 + 16 code) for odd T.
template <int T>
__device__ __forceinline__ uint32_t nib_pair_f16(uint32_t w) {
  const uint32_t v = T >= 2 ? (w >> 8) : w;
  return (v & ((T & 1) ? 0x00F000F0u : 0x000F000Fu)) | kF16Pair1024;
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
template <int BITS, int D, int NT, int DT, bool FOLD = false>
struct QkWarp {
  using C = Cfg<BITS, D, NT, FOLD>;
  using E = Elem<DT>;
  int lane, r, qd, q;
  const uint8_t *qfr;   // query fragments [KQS][NT][32] (shared memory)

  // B fragment of the query (16-bit pairs): channels 16s + 2qd, +1 and
  // 16s + 2qd + 8, +9 of query row 8nt + r.
  __device__ __forceinline__ uint2 qfrag(int s, int nt) const {
    return lds<uint2>(qfr, ((s * NT + nt) * 32 + lane) * 8);
  }

  // Token (within the item) of logit S[mt][nt][2u + j] of a packed block.
  __device__ __forceinline__ int packed_token(int mt, int u) const {
    if constexpr (FOLD && BITS == 8) return 32 * q + 16 * mt + 2 * r + u;
    return 32 * q + 4 * r + 2 * mt + u;
  }

  // Folded dequantization of one packed block's logits, for this warp's 32
  // tokens.  With k = code * scale + low per (channel d, token t),
  //   q.k_t = sum_d w_d code_dt + sum_d q_d low_d,   w_d = q_d scale_d,
  // so the scales go into the query operand once per block instead of into
  // every code.  The codes reach the tensor cores as exact fp16 values
  // (1024 + code, or 1024 + 16 code for the odd 4-bit positions) straight
  // from an ldmatrix.trans of the channel-major stage and one PRMT / LOP3 per
  // two codes; w is rounded to fp16 (saturating); a second MMA with the
  // constant operand 1024 gives the offset sum_d 1024 w_d, which is
  // subtracted, and the low term is summed in fp32.  Same output layout as
  // packed(): S[mt][nt][2u + j], token packed_token(mt, u), row 8nt + 2qd + j.
  __device__ void packed_fold(uint32_t kst, const uint8_t *kst_ptr, float (&S)[2][NT][4]) const {
    float corr[NT][4];
    float2 clow[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        corr[nt][c] = 0.f;
        S[0][nt][c] = S[1][nt][c] = 0.f;
      }
      clow[nt] = make_float2(0.f, 0.f);
    }
    const uint8_t *meta = kst_ptr + C::KCODE;
    const uint32_t one[4] = {kF16Pair1024, kF16Pair1024, kF16Pair1024, kF16Pair1024};
    // ldmatrix row addresses: lane 8m + i gives row i of matrix m.
    const int m = lane >> 3, i = lane & 7;
    uint32_t base;
    if constexpr (BITS == 8) {
      // Matrix m: channels 8(m & 1) + 0..7 of the k-step, tokens 32q + 16(m >> 1)
      // + 0..15 (one 16-byte chunk of the 128-byte row, 128-byte swizzle).
      base = kst + (8 * (m & 1) + i) * 128 + (((2 * q + (m >> 1)) ^ i) << 4);
    } else {
      // Matrix m: channels 8m + 0..7 of a pair of k-steps, this warp's 32
      // tokens (chunk q of the 64-byte row, 64-byte swizzle: row bits [1, 3)).
      base = kst + (8 * m + i) * 64 + ((q ^ (i >> 1)) << 4);
    }
    uint32_t x[4];
#pragma unroll 4
    for (int s = 0; s < C::KQS; ++s) {
      const int cb = 16 * s + 2 * qd;   // channels cb, cb+1, cb+8, cb+9
      const float4 m0 = lds<float4>(meta, cb * 8);          // (scale, low) of cb, cb + 1
      const float4 m1 = lds<float4>(meta, (cb + 8) * 8);    // of cb + 8, cb + 9
      uint32_t b[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        // The query as stored (16-bit pairs), widened exactly to fp32.
        const uint2 qp = qfrag(s, nt);
        const float2 q01 = E::unpack2(qp.x), q89 = E::unpack2(qp.y);
        const float2 w01 = __fmul2_rn(q01, make_float2(m0.x, m0.z));
        const float2 w89 = __fmul2_rn(q89, make_float2(m1.x, m1.z));
        b[nt][0] = f16x2_sat(w01.x, w01.y);
        b[nt][1] = f16x2_sat(w89.x, w89.y);
        clow[nt] = __ffma2_rn(q01, make_float2(m0.y, m0.w), clow[nt]);
        clow[nt] = __ffma2_rn(q89, make_float2(m1.y, m1.w), clow[nt]);
        mma16816<CKV_F16>(corr[nt], one, b[nt][0], b[nt][1]);
      }
      uint32_t a[2][4];
      if constexpr (BITS == 8) {
        ldmatrix_x4_trans(x, base + s * 16 * 128);
        // x[2mt]: channels 2qd, 2qd+1 of the first 8, tokens 16mt + 2r, +1;
        // x[2mt + 1]: the same for channels 8..15.
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          a[mt][0] = byte_pair_f16<kSelLo>(x[2 * mt]);        // row r: token 16mt + 2r
          a[mt][1] = byte_pair_f16<kSelHi>(x[2 * mt]);        // row r + 8: token 16mt + 2r + 1
          a[mt][2] = byte_pair_f16<kSelLo>(x[2 * mt + 1]);
          a[mt][3] = byte_pair_f16<kSelHi>(x[2 * mt + 1]);
        }
      } else {
        if ((s & 1) == 0) ldmatrix_x4_trans(x, base + (s >> 1) * 32 * 64);
        // x[2(s & 1)]: channels 2qd, 2qd+1 of the first 8, tokens 4r..4r+3;
        // x[2(s & 1) + 1]: the same for channels 8..15.
        const uint32_t x0 = x[2 * (s & 1)], x1 = x[2 * (s & 1) + 1];
        a[0][0] = nib_pair_f16<0>(x0);   // row r: token 4r
        a[0][1] = nib_pair_f16<1>(x0);   // row r + 8: token 4r + 1 (x16)
        a[0][2] = nib_pair_f16<0>(x1);
        a[0][3] = nib_pair_f16<1>(x1);
        a[1][0] = nib_pair_f16<2>(x0);   // row r: token 4r + 2
        a[1][1] = nib_pair_f16<3>(x0);   // row r + 8: token 4r + 3 (x16)
        a[1][2] = nib_pair_f16<2>(x1);
        a[1][3] = nib_pair_f16<3>(x1);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<CKV_F16>(S[mt][nt], a[mt], b[nt][0], b[nt][1]);
    }
    // sum_d q_d low_d per row: this lane holds part of row 8nt + r's sum; the
    // logits of rows 8nt + 2qd + j need the whole sum of those rows.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float c = clow[nt].x + clow[nt].y;
      c += __shfl_xor_sync(0xffffffffu, c, 1);
      c += __shfl_xor_sync(0xffffffffu, c, 2);
      const float c0 = __shfl_sync(0xffffffffu, c, 8 * qd);
      const float c1 = __shfl_sync(0xffffffffu, c, 8 * qd + 4);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float f = (BITS == 4 && u == 1) ? 0.0625f : 1.f;
          S[mt][nt][2 * u] = (S[mt][nt][2 * u] - corr[nt][0]) * f + c0;
          S[mt][nt][2 * u + 1] = (S[mt][nt][2 * u + 1] - corr[nt][1]) * f + c1;
        }
    }
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
template <int BITS, int D, int NT, int DT, bool FOLD = false>
struct PvWarp {
  using C = Cfg<BITS, D, NT, FOLD>;
  using E = Elem<DT>;
  int lane, r, qd, c;

  // ---- folded dequantization ------------------------------------------------
  // With v = code * scale_t + low_t per (token t, 64-channel group),
  //   sum_t p_t v_t = sum_t (p_t scale_t) code_t + sum_t p_t low_t,
  // so the per-token scale goes into the probability operand: P'' = fp16(p f
  // scale_t), with f = 2^(m_q - M + E) (the softmax rescale of the QK warp
  // that wrote p, and this warp's range exponent E).  The codes reach the
  // tensor cores as exact fp16 values (1024 + code, 1024 + 16 code for odd
  // 4-bit channels) from an ldmatrix.trans of the token-major stage; a second
  // MMA with the constant 1024 measures the offset (Oc), and sum_t p_t f low_t
  // (Ls) is summed in fp32.  This warp's channels lie in one group.
  //
  // O[i][nt][cc]: channel fold_channel(i, cc), query row 8nt + 2qd + (cc & 1).
  static constexpr int CHUNKS = (D / 4) * BITS / 8 / 16;   // 16-byte chunks of this warp's channels

  __device__ __forceinline__ int fold_channel(int i, int cc) const {
    if constexpr (BITS == 8) return (D / 4) * c + 16 * i + 2 * r + (cc >> 1);
    return (D / 4) * c + 32 * (i >> 1) + 4 * r + 2 * (i & 1) + (cc >> 1);
  }
  // 1 / 16 for the odd 4-bit channels (their codes arrive as 1024 + 16 code).
  __device__ __forceinline__ static constexpr float fold_inv(int cc) {
    return (BITS == 4 && (cc >> 1)) ? 0.0625f : 1.f;
  }

  // Largest scale of this warp's group over the stage's 128 tokens (all lanes).
  __device__ float fold_scale_max(const uint8_t *vst) const {
    const int grp = ((D / 4) * c) / 64;
    const uint8_t *meta = vst + C::VCODE;
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) mx = fmaxf(mx, lds<float>(meta, ((lane + 32 * k) * C::NG + grp) * 8));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    return mx;
  }

  // ldmatrix row address of this lane in the stage for token row `row0`
  // (a multiple of 16) and 16-byte chunk `chunk` of this warp's bytes.
  __device__ __forceinline__ uint32_t fold_addr(uint32_t vst, int row, int chunk) const {
    const int off = ((D / 4) * c) * BITS / 8 + 16 * chunk;   // byte of the chunk in a token row
    const int box = off / C::VBOX, inb = off % C::VBOX;
    const uint32_t a = uint32_t(row * C::VBOX + inb);
    return vst + box * 128 * C::VBOX + swz<C::VSWZ>(a);
  }

  // Exact-window chunk in the folded accumulator layout: the same 16-bit MMA
  // as resid(), with m-tile i's rows on channels fold_channel(i, 0) and
  // fold_channel(i, 2) (= + 1), and the odd 4-bit channels' values times 16
  // (their packed accumulators are in that scale).
  __device__ void resid_fold(const uint8_t *vst, const uint8_t *pb, float (&O)[C::MTV][NT][4],
                             const uint32_t (&fb)[TEAM_WARPS][NT], bool scaled) const {
    const uint32_t sixteen = BITS == 4 ? E::pack2(16.f, 16.f) : 0u;
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
#pragma unroll
      for (int i = 0; i < C::MTV; ++i) {
        const uint32_t coff = uint32_t(fold_channel(i, 0)) * 2;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = lds<uint32_t>(vst, (t0 + (e & 1) + 8 * (e >> 1)) * C::RP + coff);
        uint32_t a[4];
        a[0] = prmt(w[0], w[1], 0x5410u);   // row r: channel fold_channel(i, 0), tokens t0, t0 + 1
        a[1] = prmt(w[0], w[1], 0x7632u);   // row r + 8: the next channel
        a[2] = prmt(w[2], w[3], 0x5410u);
        a[3] = prmt(w[2], w[3], 0x7632u);
        if constexpr (BITS == 4) {
          a[1] = E::mul2(a[1], sixteen);
          a[3] = E::mul2(a[3], sixteen);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<DT>(O[i][nt], a, b[nt].x, b[nt].y);
      }
    }
  }

  __device__ void packed_fold(uint32_t vst, const uint8_t *vst_ptr, const uint8_t *pb,
                              float (&O)[C::MTV][NT][4], float (&Oc)[NT][4], float2 (&Ls)[NT],
                              const float (&fs)[TEAM_WARPS][NT]) const {
    const int grp = ((D / 4) * c) / 64;
    const uint8_t *meta = vst_ptr + C::VCODE + grp * 8;
    const uint8_t *prow = pb + r * PP + 4 * qd * 2;
    const uint32_t one[4] = {kF16Pair1024, kF16Pair1024, kF16Pair1024, kF16Pair1024};
    const int m = lane >> 3, i = lane & 7;
    // Matrix m of the x4 loads: token rows 8(m & 1) + i of the k-step, chunk
    // (m >> 1) of the pair of chunks the load covers.
    uint32_t addr[C::MTV >= 2 ? 2 : 1];
    if constexpr (BITS == 8) {
#pragma unroll
      for (int k = 0; k < CHUNKS / 2; ++k) addr[k] = fold_addr(vst, 8 * (m & 1) + i, 2 * k + (m >> 1));
    } else if constexpr (CHUNKS == 2) {
      addr[0] = fold_addr(vst, 8 * (m & 1) + i, m >> 1);
    } else {
      // One chunk: the x4 load covers two k-steps (matrix m: k-step m >> 1).
      addr[0] = fold_addr(vst, 16 * (m >> 1) + 8 * (m & 1) + i, 0);
    }
    uint32_t x[CHUNKS / 2 > 0 ? 2 * CHUNKS : 4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t0 = 16 * j + 2 * qd;   // tokens t0, t0+1, t0+8, t0+9
      const float2 s0 = lds<float2>(meta, (t0 * C::NG) * 8);
      const float2 s1 = lds<float2>(meta, ((t0 + 1) * C::NG) * 8);
      const float2 s8 = lds<float2>(meta, ((t0 + 8) * C::NG) * 8);
      const float2 s9 = lds<float2>(meta, ((t0 + 9) * C::NG) * 8);
      uint32_t b[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 pv = lds<uint2>(prow, 8 * nt * PP + 32 * j);
        const float f = fs[j >> 1][nt];
        const float2 p01 = __fmul2_rn(E::unpack2(pv.x), make_float2(f, f));
        const float2 p89 = __fmul2_rn(E::unpack2(pv.y), make_float2(f, f));
        const float2 w01 = __fmul2_rn(p01, make_float2(s0.x, s1.x));
        const float2 w89 = __fmul2_rn(p89, make_float2(s8.x, s9.x));
        b[nt][0] = f16x2_sat(w01.x, w01.y);
        b[nt][1] = f16x2_sat(w89.x, w89.y);
        Ls[nt] = __ffma2_rn(p01, make_float2(s0.y, s1.y), Ls[nt]);
        Ls[nt] = __ffma2_rn(p89, make_float2(s8.y, s9.y), Ls[nt]);
        mma16816<CKV_F16>(Oc[nt], one, b[nt][0], b[nt][1]);
      }
      if constexpr (BITS == 8) {
#pragma unroll
        for (int k = 0; k < CHUNKS / 2; ++k) {
          uint32_t y[4];
          ldmatrix_x4_trans(y, addr[k] + j * 16 * C::VBOX);
          // y[2e]: chunk 2k + e, tokens t0, t0 + 1; y[2e + 1]: tokens t0 + 8, + 9.
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            uint32_t a[4];
            a[0] = byte_pair_f16<kSelLo>(y[2 * e]);       // row r: channel 2r of the chunk
            a[1] = byte_pair_f16<kSelHi>(y[2 * e]);       // row r + 8: channel 2r + 1
            a[2] = byte_pair_f16<kSelLo>(y[2 * e + 1]);
            a[3] = byte_pair_f16<kSelHi>(y[2 * e + 1]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816<CKV_F16>(O[2 * k + e][nt], a, b[nt][0], b[nt][1]);
          }
        }
      } else {
        uint32_t lo[CHUNKS], hi[CHUNKS];   // per chunk: tokens t0, t0+1 and t0+8, t0+9
        if constexpr (CHUNKS == 2) {
          ldmatrix_x4_trans(x, addr[0] + j * 16 * C::VBOX);
          lo[0] = x[0]; hi[0] = x[1]; lo[1] = x[2]; hi[1] = x[3];
        } else {
          if ((j & 1) == 0) ldmatrix_x4_trans(x, addr[0] + j * 16 * C::VBOX);
          lo[0] = x[2 * (j & 1)]; hi[0] = x[2 * (j & 1) + 1];
        }
#pragma unroll
        for (int k = 0; k < CHUNKS; ++k) {
          uint32_t a0[4], a1[4];
          a0[0] = nib_pair_f16<0>(lo[k]);   // row r: channel 4r
          a0[1] = nib_pair_f16<1>(lo[k]);   // row r + 8: channel 4r + 1 (x16)
          a0[2] = nib_pair_f16<0>(hi[k]);
          a0[3] = nib_pair_f16<1>(hi[k]);
          a1[0] = nib_pair_f16<2>(lo[k]);   // row r: channel 4r + 2
          a1[1] = nib_pair_f16<3>(lo[k]);   // row r + 8: channel 4r + 3 (x16)
          a1[2] = nib_pair_f16<2>(hi[k]);
          a1[3] = nib_pair_f16<3>(hi[k]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            mma16816<CKV_F16>(O[2 * k][nt], a0, b[nt][0], b[nt][1]);
            mma16816<CKV_F16>(O[2 * k + 1][nt], a1, b[nt][0], b[nt][1]);
          }
        }
      }
    }
  }

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


// Bounded wait on an mbarrier phase that also gives up as soon as another
// warp of the CTA has flagged an abort.  Returns false on either.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort || clock64() - start > (1ll << 31)) return false;
  }
  return true;
}

// 2^d for an integer-valued d <= 127 (either sign); 0 below the normal range
// and for -inf or NaN.
__device__ __forceinline__ float pow2s(float d) {
  return !(d >= -126.f) ? 0.f : __int_as_float((int(fminf(d, 127.f)) + 127) << 23);
}

// The last CTA of a (sequence, KV head) pair merges the pair's CTA records
// (m, l and the unnormalised output per row, in the workspace) into the
// output, or into the pair's partial record when p.partial.  `avail` bytes of
// shared memory at smem / sbase are free; s_mbar holds two mbarriers.
template <int D, int DT, int NTHREADS, int ROWSMAX, class P>
__device__ void merge_pair_records(const P &p, const SeqDev &sd, uint8_t *smem, uint32_t sbase,
                                   uint64_t *s_mbar, int avail, int seq, int head, int G, int nq,
                                   int rows, int tid, int warp, int lane) {
  const int mls = ml_stride(rows);
  // ---- last CTA of the pair: merge the pair's CTA records -------------------
  // The pair's records are consecutive in the workspace ([cph][rows][D] fp32,
  // then [cph][mls] (m, l) pairs), so bulk copies bring them into the freed
  // stage memory in a few large transfers (records in chunks of `mrec` when
  // they do not all fit).  The (m, l) pairs arrive first on their own
  // barrier, so the record weights are ready when the records land; every
  // output float4 is then summed by `parts` threads over disjoint record
  // ranges.
  const int c0 = sd.cta_begin + head * sd.cph;
  const int cph = sd.cph;
  constexpr int D4 = D / 4;
  const int AVAIL = avail;
  const int outs = rows * D4;
  const int parts = max(1, min(4, NTHREADS / outs));
  const uint32_t rec_bytes = uint32_t(rows) * D * 4;
  const uint32_t ml_bytes = uint32_t(cph) * mls * 4;                 // a multiple of 16
  const uint32_t w_off = ml_bytes;                                     // [rows][cph] weights
  const uint32_t row_off = w_off + uint32_t(rows) * cph * 4;           // [ROWS] (M, L)
  const uint32_t acc_off = (row_off + 2 * ROWSMAX * 4 + 15) & ~15u;    // [parts - 1][outs] float4
  const uint32_t rec_off = (acc_off + uint32_t(parts - 1) * outs * 16 + 127) & ~127u;
  const int mrec = max(1, min(cph, int((AVAIL - rec_off) / rec_bytes)));
  const float2 *s_ml = reinterpret_cast<const float2 *>(smem);        // [cph][mls / 2]
  float *s_w = reinterpret_cast<float *>(smem + w_off);
  float *s_row = reinterpret_cast<float *>(smem + row_off);
  float4 *s_acc = reinterpret_cast<float4 *>(smem + acc_off);
  const float4 *s_rec = reinterpret_cast<const float4 *>(smem + rec_off);   // [mrec][rows][D4]
  const uint32_t mbar_ml = smem_u32(&s_mbar[0]), mbar_rec = smem_u32(&s_mbar[1]);
  auto issue_rec = [&](int cb, int cnt) {
    mbar_expect_tx(mbar_rec, uint32_t(cnt) * rec_bytes);
    bulk_load(sbase + rec_off, p.rec + size_t(c0 + cb) * rows * D, uint32_t(cnt) * rec_bytes, mbar_rec);
  };
  if (tid == 0) {
    mbar_init(mbar_ml, 1);
    mbar_init(mbar_rec, 1);
    mbar_fence_init();
    // The CTA's earlier generic writes to this shared memory and the acquired
    // record stores of the other CTAs are ordered before the copies.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
    mbar_expect_tx(mbar_ml, ml_bytes);
    bulk_load(sbase, p.rec_ml + size_t(c0) * mls, ml_bytes, mbar_ml);
    issue_rec(0, min(mrec, cph));
  }
  __syncthreads();
  if (!mbar_wait(mbar_ml, 0)) atomicOr(p.error, 1u);
  // Row maxima, record weights and the merged denominator.
  for (int row = warp; row < rows; row += NTHREADS / 32) {
    float M = -INFINITY;
    for (int c = lane; c < cph; c += 32) M = fmaxf(M, s_ml[c * (mls / 2) + row].x);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int c = lane; c < cph; c += 32) {
      const float2 ml = s_ml[c * (mls / 2) + row];
      const float wt = (ml.x == -INFINITY) ? 0.f : ex2(ml.x - M);
      s_w[row * cph + c] = wt;
      L += wt * ml.y;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) {
      s_row[2 * row] = M;
      s_row[2 * row + 1] = L;
    }
  }
  __syncthreads();
  // Work unit u = tid + k * NTHREADS: output float4 o = u % outs, record part
  // u / outs (k < 2 covers the largest case, 16 rows x 64 float4s, parts 1).
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  for (int cb = 0, chunk = 0; cb < cph; cb += mrec, ++chunk) {
    const int cnt = min(mrec, cph - cb);
    if (chunk > 0) {
      __syncthreads();   // the previous chunk is consumed
      if (tid == 0) issue_rec(cb, cnt);
    }
    if (!mbar_wait(mbar_rec, chunk & 1)) atomicOr(p.error, 1u);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int u = tid + k * NTHREADS;
      if (u < outs * parts) {
        const int o = u % outs, part = u / outs;
        const int cl = part * cnt / parts, ce = (part + 1) * cnt / parts;
        const float *wr = s_w + (o / D4) * cph + cb;
        const float4 *src = s_rec + o;
        float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
        int c = cl;
        for (; c + 2 <= ce; c += 2) {
          const float w0 = wr[c], w1 = wr[c + 1];
          const float4 v0 = src[size_t(c) * outs], v1 = src[size_t(c + 1) * outs];
          a0.x += w0 * v0.x; a0.y += w0 * v0.y; a0.z += w0 * v0.z; a0.w += w0 * v0.w;
          a1.x += w1 * v1.x; a1.y += w1 * v1.y; a1.z += w1 * v1.z; a1.w += w1 * v1.w;
        }
        if (c < ce) {
          const float w0 = wr[c];
          const float4 v0 = src[size_t(c) * outs];
          a0.x += w0 * v0.x; a0.y += w0 * v0.y; a0.z += w0 * v0.z; a0.w += w0 * v0.w;
        }
        acc[k].x += a0.x + a1.x; acc[k].y += a0.y + a1.y; acc[k].z += a0.z + a1.z; acc[k].w += a0.w + a1.w;
      }
    }
  }
  if (parts > 1) {
    if (tid >= outs && tid < outs * parts) s_acc[tid - outs] = acc[0];
    __syncthreads();
    if (tid < outs)
      for (int pp = 1; pp < parts; ++pp) {
        const float4 v = s_acc[(pp - 1) * outs + tid];
        acc[0].x += v.x; acc[0].y += v.y; acc[0].z += v.z; acc[0].w += v.w;
      }
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int o = tid + k * NTHREADS;
    if (o >= outs || (parts > 1 && k > 0)) continue;
    const int row = o / D4, d4 = o % D4;
    const float M = s_row[2 * row], L = s_row[2 * row + 1];
    const int nn = row / G, g = row % G;
    const int64_t orow = int64_t(head * G + g) * nq + nn;
    if (p.partial) {
      float *out = static_cast<float *>(sd.out) + orow * (D + 2);
      out[4 * d4] = acc[k].x; out[4 * d4 + 1] = acc[k].y; out[4 * d4 + 2] = acc[k].z; out[4 * d4 + 3] = acc[k].w;
      if (d4 == 0) {
        out[D] = M;
        out[D + 1] = L;
      }
    } else {
      typename Elem<DT>::T *out = static_cast<typename Elem<DT>::T *>(sd.out) + orow * D + 4 * d4;
      const float inv = 1.f / L;
      out[0] = Elem<DT>::from_f32(acc[k].x * inv);
      out[1] = Elem<DT>::from_f32(acc[k].y * inv);
      out[2] = Elem<DT>::from_f32(acc[k].z * inv);
      out[3] = Elem<DT>::from_f32(acc[k].w * inv);
    }
  }
  if (tid == 0) p.counters[seq * p.hkv + head] = 0u;
}
}  // namespace attn
}  // namespace ckv
