// Decode attention with the folded dequantization rule, token-split warps
// (sm_100a).  8-bit codes, up to 8 query rows per KV head, head_dim 128/256.
//
// Same work split, workspace and cross-CTA merge as attn_kernel (ckv_attn.cu):
// a (sequence, KV head) pair's items -- packed 128-token blocks, then 64-token
// chunks of the exact window -- are cut into contiguous ranges, one per CTA,
// and the last CTA of the pair merges the CTA records.  Inside a CTA the
// roles differ:
//
//   K / V producer  one warp each: TMA of a block's codes (swizzled) plus its
//                   (scale, low) metadata, or 16-byte cp.async of a window
//                   chunk, into rings of NK / NV stages.
//   w warp          per block, the query operand with the key scales folded
//                   in, w[row][d] = fp16(q[row][d] * scale[d]), as MMA
//                   A-fragments, and per row the constant
//                   C = sum_d q low_d - 1024 sum_d w[row][d].
//   8 value warps   warp c owns tokens 16c..16c+15 of every block (window
//                   chunks: warps 0..3) over all channels, with its own
//                   online softmax state and output accumulator; no
//                   exchange between warps until the CTA's items are done.
//
// Logits are computed transposed, S^T[row][token] = w . code + C: the codes
// are the B operand, taken as exact fp16 values (1024 + code, one PRMT per
// two codes) from an ldmatrix.trans of the channel-major stage; the two
// 16-bit halves of one ldmatrix element are tokens 2n and 2n + 1, so one
// n-tile holds the block's even tokens and another its odd ones.  The
// logit accumulator of lane (r, qd) -- row r, tokens {4qd, 4qd + 2} (even
// tile) and {4qd + 1, 4qd + 3} (odd tile) -- is then exactly the lane's B
// fragment of the value MMA when the value tile's ldmatrix rows are
// addressed as the even, then the odd tokens: P never leaves registers.
//
// Values: O[channel][row] += sum_t code[t][channel] P''[t][row] with
// P'' = fp16(p f scale_t) per 64-channel group (f = 2^Ex, this warp's range
// exponent), the offset 1024 sum_t P'' measured by a second MMA with a
// constant operand, and sum_t p f low_t summed in fp32.  The exact window
// uses the 16-bit values directly.  Accumulators are fp32.
#pragma once

#include "ckv_attn.cuh"

namespace ckv {
namespace split {

using attn::align1k;
using attn::byte_pair_f16;
using attn::cmax;
using attn::f16x2_sat;
using attn::kF16Pair1024;
using attn::kSelHi;
using attn::kSelLo;
using attn::ldmatrix_x4_trans;
using attn::ml_stride;
using attn::Params;
using attn::pow2i;
using attn::SeqDev;
using attn::swz;

constexpr int CW = 8;                   // value warps
constexpr int WW = CW;                  // the w warp
constexpr int PKW = CW + 1;             // K producer warp
constexpr int PVW = CW + 2;             // V producer warp
constexpr int WARPS = CW + 3;
constexpr int THREADS = WARPS * 32;
constexpr int RCH = attn::RCHUNK;       // exact-window tokens per item (value warps 0..3)
constexpr int NK = 3, NV = 2;           // ring depths
constexpr int BAR_Q = 2;                // named barrier: query staged (value warps + w warp)

template <int D>
struct Cfg {
  static constexpr int SB = 128;                         // 8-bit: bytes per key channel row
  static constexpr int KCODE = D * SB, KMETA = D * 8;
  static constexpr int RP = 2 * D + 16;                  // window row pitch (16-bit values)
  static constexpr int RBYTES = RCH * RP;
  static constexpr int KST = align1k(cmax(KCODE + KMETA, RBYTES));
  static constexpr int VROWB = D;
  static constexpr int VBOX = VROWB < 128 ? VROWB : 128;
  static constexpr int NVB = VROWB / VBOX;
  static constexpr int VSWZ = VBOX == 128 ? 7 : 3;
  static constexpr int NG = D / 64;
  static constexpr int VCODE = 128 * VROWB, VMETA = 128 * NG * 8;
  static constexpr int VST = align1k(cmax(VCODE + VMETA, RBYTES));
  static constexpr int KQS = D / 16;                     // channel k-steps of the logits
  static constexpr int MT = D / 16;                      // value m-tiles (16 channels each)
  // Per K stage: w fragments [KQS][32 lanes] (a0, a2) then C[8] (fp32).
  static constexpr int WFR = KQS * 32 * 8;
  static constexpr int WST = WFR + 64;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + NK * KST;
  static constexpr int OFF_W = OFF_V + NV * VST;
  static constexpr int OFF_QF = OFF_W + NK * WST;         // [8][D] fp32 query (w warp)
  static constexpr int OFF_QB = OFF_QF + 8 * D * 6;       // [KQS][32] 16-bit query A-fragments
                                                          // (after the fp32 rows, 16-bit staging)
  static constexpr int OFF_END = OFF_QB + KQS * 32 * 8;
  static constexpr int SMEM = OFF_END + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // End of the items: per value warp (m, l) per row and the output rows.
  static constexpr int RED_O = 0;                          // [CW][8][D] fp32
  static constexpr int RED_M = CW * 8 * D * 4;             // [CW][8]
  static constexpr int RED_L = RED_M + CW * 8 * 4;         // [CW][8]
  static_assert(RED_L + CW * 8 * 4 <= NK * KST + NV * VST, "reduction scratch");
};

template <int D, int DT, int MAXS>
__global__ void __launch_bounds__(THREADS, 1) split_kernel(const __grid_constant__ Params<MAXS> p) {
  using C = Cfg<D>;
  using E = Elem<DT>;
  using T = typename E::T;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int s_seq, s_last;
  __shared__ volatile int s_abort;
  // kfull[NK] kempty[NK] wfull[NK] vfull[NV] vempty[NV]
  __shared__ __align__(8) uint64_t s_bar[3 * NK + 2 * NV];
  __shared__ __align__(8) uint64_t s_mbar[2];   // bulk copies of the merge
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return smem_u32(&s_bar[i]); };
  constexpr int KFULL = 0, KEMPTY = NK, WFULL = 2 * NK, VFULL = 3 * NK, VEMPTY = 3 * NK + NV;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  if (tid == 0) {
    int lo = 0, hi = p.num_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.seq[mid].cta_begin <= cta) lo = mid; else hi = mid - 1;
    }
    s_seq = lo;
    s_abort = 0;
    for (int i = 0; i < NK; ++i) {
      mbar_init(bar(KFULL + i), 1);
      mbar_init(bar(KEMPTY + i), CW + 1);   // one arrival per value warp and the w warp
      mbar_init(bar(WFULL + i), 1);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(bar(VFULL + i), 1);
      mbar_init(bar(VEMPTY + i), CW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();
  const int seq = s_seq;
  const SeqDev &sd = p.seq[seq];
  const int local = cta - sd.cta_begin;
  const int head = local / sd.cph, split = local % sd.cph;
  const int rsplit = sd.cph - 1 - split;   // see attn_kernel: the first split starts last
  const int G = p.group, rows = p.rows, nq = p.nq;

  // Items: packed units [ub, ue) then window chunks of RCH tokens.  Local
  // order: as many packed blocks as the K ring holds (all issued before the
  // wait on the previous kernel), the window chunks, the other blocks.
  const int np = sd.ue - sd.ub;
  const int nr = (sd.re - sd.rb + RCH - 1) / RCH;
  const int ni = np + nr;
  const int ib = int(int64_t(rsplit) * ni / sd.cph);
  const int n = int(int64_t(rsplit + 1) * ni / sd.cph) - ib;
  const int npk = max(0, min(n, np - ib));
  const int nrs = n - npk;
  const int pre = min(npk, NK);
  auto item = [&](int i) {
    if (nrs == 0 || i < pre) return ib + i;
    return i < pre + nrs ? ib + npk + (i - pre) : ib + (i - nrs);
  };

  auto fail = [&]() {
    atomicOr(p.error, 1u);
    s_abort = 1;
  };
  auto wait = [&](int b, int parity) {
    if (s_abort) return false;
    const bool ok = attn::wait_or_abort(bar(b), parity, &s_abort);
    if (!ok && !s_abort) fail();
    return ok;
  };

  auto issue_packed = [&](bool kchain, int i, int st) {
    const int unit = sd.ub + item(i);
    if (kchain) {
      const uint32_t dst = sbase + C::OFF_K + st * C::KST, fb = bar(KFULL + st);
      mbar_expect_tx(fb, C::KCODE + C::KMETA);
      tma_load_4d(dst, &sd.tk, fb, 0, 0, unit, head);
      bulk_load(dst + C::KCODE, sd.km + head * sd.km_h + int64_t(unit) * sd.km_u, C::KMETA, fb);
    } else {
      const uint32_t dst = sbase + C::OFF_V + st * C::VST, fb = bar(VFULL + st);
      mbar_expect_tx(fb, C::VCODE + C::VMETA);
#pragma unroll
      for (int bx = 0; bx < C::NVB; ++bx)
        tma_load_3d(dst + bx * 128 * C::VBOX, &sd.tv, fb, bx * C::VBOX, unit * 128, head);
      bulk_load(dst + C::VCODE, sd.vm + head * sd.vm_h + int64_t(unit) * 128 * sd.vm_t, C::VMETA, fb);
    }
  };

  // Before the wait on the previous kernel: fill both rings with packed
  // blocks (the banks are never written by a kernel of this library that
  // lets its successor start early).
  int preissued = 0;
  if (warp == PKW || warp == PVW) {
    const bool kchain = warp == PKW;
    const int ahead = min(pre, kchain ? NK : NV);
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(kchain ? &sd.tk : &sd.tv) : "memory");
      for (int i = 0; i < ahead; ++i) issue_packed(kchain, i, i);
    }
    preissued = ahead;
  }
  pdl_wait();

  // Query: fp32 rows for the w warp and 16-bit A-fragments (rows r, channels
  // 16s + 2qd.. and + 8..) for the exact window.  Each thread takes 8
  // consecutive channels of one row with one 16-byte load (q rows are dense
  // and 16-byte aligned), so the whole query arrives in one round trip.
  if (warp <= WW) {
    const T *qb = static_cast<const T *>(sd.q);
    float *qf = reinterpret_cast<float *>(smem + C::OFF_QF);
    uint16_t *qh = reinterpret_cast<uint16_t *>(smem + C::OFF_QF + 8 * D * 4);   // staging [8][D]
    for (int x = tid; x < D; x += (CW + 1) * 32) {   // x: 8-channel group of row x / (D / 8)
      const int row = x / (D / 8), d0 = (x % (D / 8)) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row < rows)
        v = *reinterpret_cast<const uint4 *>(qb + (head * G + row % G) * sd.q_h + (row / G) * sd.q_n + d0);
      *reinterpret_cast<uint4 *>(qh + row * D + d0) = v;
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = E::unpack2(w[k]);
        qf[row * D + d0 + 2 * k] = f.x;
        qf[row * D + d0 + 2 * k + 1] = f.y;
      }
    }
    named_sync(BAR_Q, (CW + 1) * 32);
    for (int x = tid; x < C::KQS * 32; x += (CW + 1) * 32) {
      const int ln = x & 31, s = x >> 5, row = ln >> 2, cb = 16 * s + 2 * (ln & 3);
      const uint16_t *qr = qh + row * D;
      *reinterpret_cast<uint2 *>(smem + C::OFF_QB + x * 8) =
          make_uint2(qr[cb] | (uint32_t(qr[cb + 1]) << 16), qr[cb + 8] | (uint32_t(qr[cb + 9]) << 16));
    }
    named_sync(BAR_Q, (CW + 1) * 32);
  }

  const int r = lane >> 2, qd = lane & 3;
  // Value-warp state (row r of this lane for m / l / Ls; rows 2qd, 2qd + 1
  // for the accumulators).
  float O[C::MT][4];
  float Oc[C::NG][4];
  float2 Ls[C::NG];
  float m_run = -INFINITY, l_run = 0.f;
  int Ex = 0;

  if (warp == PKW || warp == PVW) {
    // ---- producers ------------------------------------------------------------
    const bool kchain = warp == PKW;
    const int depth = kchain ? NK : NV;
    const int full0 = kchain ? KFULL : VFULL, empty0 = kchain ? KEMPTY : VEMPTY;
    const int stage_bytes = kchain ? C::KST : C::VST;
    const uint32_t ring = sbase + (kchain ? C::OFF_K : C::OFF_V);
    const T *res = static_cast<const T *>(kchain ? sd.rk : sd.rv);
    const int64_t res_h = kchain ? sd.rk_h : sd.rv_h, res_t = kchain ? sd.rk_t : sd.rv_t;
    int issued = preissued;
    for (int i = preissued; i < n; ++i) {
      const int st = i % depth;
      int go = 0;
      if (lane == 0) {
        go = !s_abort;
        if (go && i >= depth && !attn::wait_or_abort(bar(empty0 + st), ((i / depth) & 1) ^ 1, &s_abort)) {
          fail();
          go = 0;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      const uint32_t dst = ring + st * stage_bytes, fb = bar(full0 + st);
      const int it = item(i);
      if (it < np) {
        if (lane == 0) issue_packed(kchain, i, st);
      } else {
        const int t0 = sd.rb + (it - np) * RCH;
        const int cnt = min(RCH, sd.re - t0);
        const T *src = res + head * res_h;
        constexpr int CH = 2 * D / 16;
        for (int x = lane; x < RCH * CH; x += 32) {
          const int t = x / CH, k = x % CH;
          const int ts = t < cnt ? t : cnt - 1;
          cp_async16(dst + t * C::RP + k * 16, src + int64_t(t0 + ts) * res_t + k * 8);
        }
        cp_async_mbar_arrive(fb);
        __syncwarp();
        if (lane == 0) mbar_arrive(fb);
      }
      __syncwarp();
      issued = i + 1;
    }
    cp_async_commit();
    cp_async_wait<0>();
    if (lane == 0) {
      for (int st = 0; st < depth && st < issued; ++st) {
        const int last = st + (issued - 1 - st) / depth * depth;
        mbar_wait(bar(full0 + st), (last / depth) & 1);
      }
    }
    __syncwarp();
  } else if (warp == WW) {
    // ---- w warp: the folded query operand of each block ------------------------
    const float *qf = reinterpret_cast<const float *>(smem + C::OFF_QF);
    const uint32_t one2 = kF16Pair1024;
    for (int i = 0; i < n; ++i) {
      const int sk = i % NK;
      const bool ok = wait(KFULL + sk, (i / NK) & 1);
      uint8_t *wst = smem + C::OFF_W + sk * C::WST;
      if (ok && item(i) < np) {
        const uint8_t *meta = smem + C::OFF_K + sk * C::KST + C::KCODE;
        float corr[4][4] = {};   // four chains (k-steps s mod 4)
        float2 cl = make_float2(0.f, 0.f);
#pragma unroll 4
        for (int s = 0; s < C::KQS; ++s) {
          const int cb = 16 * s + 2 * qd;
          const float4 m0 = attn::lds<float4>(meta, cb * 8);
          const float4 m1 = attn::lds<float4>(meta, (cb + 8) * 8);
          const float2 q01 = *reinterpret_cast<const float2 *>(qf + r * D + cb);
          const float2 q89 = *reinterpret_cast<const float2 *>(qf + r * D + cb + 8);
          const float2 w01 = __fmul2_rn(q01, make_float2(m0.x, m0.z));
          const float2 w89 = __fmul2_rn(q89, make_float2(m1.x, m1.z));
          uint32_t a[4];
          a[0] = f16x2_sat(w01.x, w01.y);
          a[1] = 0u;
          a[2] = f16x2_sat(w89.x, w89.y);
          a[3] = 0u;
          *reinterpret_cast<uint2 *>(wst + (s * 32 + lane) * 8) = make_uint2(a[0], a[2]);
          cl = __ffma2_rn(q01, make_float2(m0.y, m0.w), cl);
          cl = __ffma2_rn(q89, make_float2(m1.y, m1.w), cl);
          mma16816<CKV_F16>(corr[s & 3], a, one2, one2);   // 1024 sum_d w[row r][d] (any column)
        }
        float c = cl.x + cl.y;
        c += __shfl_xor_sync(0xffffffffu, c, 1);
        c += __shfl_xor_sync(0xffffffffu, c, 2);
        if (qd == 0)
          reinterpret_cast<float *>(wst + C::WFR)[r] = c - ((corr[0][0] + corr[1][0]) + (corr[2][0] + corr[3][0]));
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar(WFULL + sk));
        mbar_arrive(bar(KEMPTY + sk));
      }
    }
  } else {
    // ---- value warps --------------------------------------------------------------
    const int c = warp;   // token slice 16c..16c+15 of a block, 0..3 of a window chunk
#pragma unroll
    for (int i = 0; i < C::MT; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) O[i][k] = 0.f;
#pragma unroll
    for (int g = 0; g < C::NG; ++g) {
#pragma unroll
      for (int k = 0; k < 4; ++k) Oc[g][k] = 0.f;
      Ls[g] = make_float2(0.f, 0.f);
    }
    const float sl = p.scale_log2;
    const uint32_t one[4] = {kF16Pair1024, kF16Pair1024, kF16Pair1024, kF16Pair1024};
    // ldmatrix row of this lane: matrix m = lane >> 3, row i = lane & 7.
    const int mm = lane >> 3, mi = lane & 7;
    // Keys of a block: matrix m covers channel rows 8m + i of a pair of
    // k-steps, this warp's 16-byte chunk (tokens 16c..16c+15), 128-byte swizzle.
    const uint32_t kaddr = uint32_t((8 * mm + mi) * 128 + ((c ^ mi) << 4));
    for (int i = 0; i < n; ++i) {
      const int sk = i % NK, sv = i % NV;
      const int it = item(i);
      const bool pk = it < np;
      const bool mine = pk || c < RCH / 16;
      bool ok = wait(KFULL + sk, (i / NK) & 1);
      ok = wait(WFULL + sk, (i / NK) & 1) && ok;
      // ---- logits S^T: row r, tokens {4qd, 4qd + 2} (Se) and {4qd + 1, 4qd + 3} (So)
      float Se[4] = {0.f, 0.f, 0.f, 0.f}, So[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok && mine) {
        const uint32_t kst = sbase + C::OFF_K + sk * C::KST;
        if (pk) {
          const uint8_t *wst = smem + C::OFF_W + sk * C::WST;
          // Four independent accumulator chains per tile (k-steps s mod 4):
          // the MMAs of one chain wait for each other, the chains do not.
          float ce[4][4], co[4][4];
#pragma unroll
          for (int h = 0; h < 4; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k) ce[h][k] = co[h][k] = 0.f;
#pragma unroll
          for (int s = 0; s < C::KQS; s += 2) {
            uint32_t x[4];
            ldmatrix_x4_trans(x, kst + kaddr + (s >> 1) * 32 * 128);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint2 wv = attn::lds<uint2>(wst, ((s + u) * 32 + lane) * 8);
              const uint32_t a[4] = {wv.x, 0u, wv.y, 0u};
              const uint32_t xa = x[2 * u], xb = x[2 * u + 1];
              mma16816<CKV_F16>(ce[(s + u) & 3], a, byte_pair_f16<kSelLo>(xa), byte_pair_f16<kSelLo>(xb));
              mma16816<CKV_F16>(co[(s + u) & 3], a, byte_pair_f16<kSelHi>(xa), byte_pair_f16<kSelHi>(xb));
            }
          }
          const float cr = reinterpret_cast<const float *>(wst + C::WFR)[r];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            Se[k] = (ce[0][k] + ce[1][k]) + (ce[2][k] + ce[3][k]) + cr;
            So[k] = (co[0][k] + co[1][k]) + (co[2][k] + co[3][k]) + cr;
          }
        } else {
          // Exact window: matrix m = (class m >> 1: even / odd tokens,
          // channels 8(m & 1)..+7 of the k-step); rows are tokens.
          const uint32_t raddr = kst + uint32_t((16 * c + 2 * mi + (mm >> 1)) * C::RP + 16 * (mm & 1));
          const uint8_t *qbf = smem + C::OFF_QB;
#pragma unroll 4
          for (int s = 0; s < C::KQS; ++s) {
            uint32_t x[4];
            attn::ldmatrix_x4(x, raddr + 32 * s);
            const uint2 qv = attn::lds<uint2>(qbf, (s * 32 + lane) * 8);
            const uint32_t a[4] = {qv.x, 0u, qv.y, 0u};
            mma16816<DT>(Se, a, x[0], x[1]);
            mma16816<DT>(So, a, x[2], x[3]);
          }
        }
      }
      if (lane == 0) mbar_arrive(bar(KEMPTY + sk));
      // ---- online softmax of row r over this warp's tokens -------------------------
      float pv[4] = {0.f, 0.f, 0.f, 0.f};   // tokens 4qd, 4qd + 2, 4qd + 1, 4qd + 3
      if (ok && mine) {
        float sv4[4] = {Se[0] * sl, Se[1] * sl, So[0] * sl, So[1] * sl};
        if (!pk) {
          const int rb = sd.rb + (it - np) * RCH + 16 * c;
          const int toks[4] = {4 * qd, 4 * qd + 2, 4 * qd + 1, 4 * qd + 3};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int ri = rb + toks[k];
            const bool vis = ri < sd.re && (nq == 1 || sd.packed + ri <= sd.length - nq + r / G);
            if (!vis) sv4[k] = -INFINITY;
          }
        }
        float mx = fmaxf(fmaxf(sv4[0], sv4[1]), fmaxf(sv4[2], sv4[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = mx > m_run ? ceilf(mx) : m_run;
        const bool grow = mnew != m_run;
        if (__any_sync(0xffffffffu, grow)) {
          // Rescale by the exact power of two 2^(m_old - m_new): rows 2qd + j of
          // the accumulators take the factor of lane 4(2qd + j).
          const float f = pow2i(m_run - mnew);
          const float f0 = __shfl_sync(0xffffffffu, f, 8 * qd), f1 = __shfl_sync(0xffffffffu, f, 8 * qd + 4);
#pragma unroll
          for (int t = 0; t < C::MT; ++t) {
            O[t][0] *= f0; O[t][1] *= f1; O[t][2] *= f0; O[t][3] *= f1;
          }
#pragma unroll
          for (int g = 0; g < C::NG; ++g) {
            Oc[g][0] *= f0; Oc[g][1] *= f1; Oc[g][2] *= f0; Oc[g][3] *= f1;
            Ls[g] = __fmul2_rn(Ls[g], make_float2(f, f));
          }
          l_run *= f;
          m_run = mnew;
        }
        const float mu = m_run == -INFINITY ? 0.f : m_run;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          pv[k] = ex2(sv4[k] - mu);
          l_run += pv[k];
        }
      }
      // ---- values ------------------------------------------------------------------
      bool vok = wait(VFULL + sv, (i / NV) & 1);
      if (vok && ok && mine) {
        const uint32_t vst = sbase + C::OFF_V + sv * C::VST;
        const uint8_t *vsp = smem + C::OFF_V + sv * C::VST;
        if (pk) {
          const uint8_t *meta = vsp + C::VCODE + (16 * c + 4 * qd) * C::NG * 8;   // tokens 4qd..4qd+3
          // (scale, low) of every group for this lane's tokens 4qd + 0..3.
          float2 tm[4][C::NG];
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int g = 0; g < C::NG; g += 2) {
              const float4 v = attn::lds<float4>(meta, (k * C::NG + g) * 8);
              tm[k][g] = make_float2(v.x, v.y);
              tm[k][g + 1] = make_float2(v.z, v.w);
            }
          // Range exponent of this warp: the largest scale among its tokens
          // times 2^Ex stays at 2^12 (P'' <= 2^12); it moves down whenever a
          // block needs it and up only by more than 8 (precision), and the
          // accumulators follow by the exact power of two.
          {
            float smax = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
              for (int g = 0; g < C::NG; ++g) smax = fmaxf(smax, tm[k][g].x);
            smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 1));
            smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 2));
            const int eb = ((__float_as_int(smax) >> 23) & 0xff) - 127 + ((__float_as_int(smax) & 0x7fffff) != 0);
            const int need = smax > 0.f ? max(-60, min(60, 12 - eb)) : Ex;
            if (need < Ex || need > Ex + 8) {
              const float f0 = attn::pow2s(float(need - Ex));
#pragma unroll
              for (int t = 0; t < C::MT; ++t)
#pragma unroll
                for (int k = 0; k < 4; ++k) O[t][k] *= f0;
#pragma unroll
              for (int g = 0; g < C::NG; ++g) {
#pragma unroll
                for (int k = 0; k < 4; ++k) Oc[g][k] *= f0;
                Ls[g] = __fmul2_rn(Ls[g], make_float2(f0, f0));
              }
              Ex = need;
            }
          }
          const float fx = attn::pow2s(float(Ex));
          const float2 pe = __fmul2_rn(make_float2(pv[0], pv[1]), make_float2(fx, fx));   // tokens 4qd, 4qd + 2
          const float2 po = __fmul2_rn(make_float2(pv[2], pv[3]), make_float2(fx, fx));   // 4qd + 1, 4qd + 3
          uint32_t b[C::NG][2];
#pragma unroll
          for (int g = 0; g < C::NG; ++g) {
            const float2 we = __fmul2_rn(pe, make_float2(tm[0][g].x, tm[2][g].x));
            const float2 wo = __fmul2_rn(po, make_float2(tm[1][g].x, tm[3][g].x));
            b[g][0] = f16x2_sat(we.x, we.y);
            b[g][1] = f16x2_sat(wo.x, wo.y);
            Ls[g] = __ffma2_rn(pe, make_float2(tm[0][g].y, tm[2][g].y), Ls[g]);
            Ls[g] = __ffma2_rn(po, make_float2(tm[1][g].y, tm[3][g].y), Ls[g]);
            mma16816<CKV_F16>(Oc[g], one, b[g][0], b[g][1]);
          }
          // Value codes: x4 load k covers channel chunks 2k, 2k + 1, each as the
          // even-token matrix (rows 16c + 2i) and the odd-token matrix.
#pragma unroll
          for (int k = 0; k < C::MT / 2; ++k) {
            const int chunk = 2 * k + (mm >> 1);
            const int row = 16 * c + 2 * mi + (mm & 1);
            const int off = 16 * chunk;
            const uint32_t a = vst + (off / C::VBOX) * 128 * C::VBOX + swz<C::VSWZ>(uint32_t(row * C::VBOX + off % C::VBOX));
            uint32_t y[4];
            ldmatrix_x4_trans(y, a);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int t = 2 * k + e;
              uint32_t av[4];
              av[0] = byte_pair_f16<kSelLo>(y[2 * e]);       // row r: channel 16t + 2r
              av[1] = byte_pair_f16<kSelHi>(y[2 * e]);       // row r + 8: channel 16t + 2r + 1
              av[2] = byte_pair_f16<kSelLo>(y[2 * e + 1]);
              av[3] = byte_pair_f16<kSelHi>(y[2 * e + 1]);
              mma16816<CKV_F16>(O[t], av, b[t / 4][0], b[t / 4][1]);
            }
          }
        } else {
          // Exact window: the accumulators at scale 1 around 16-bit MMAs
          // (P <= 1 stays in range for fp16 queries).
          const float down = attn::pow2s(float(-Ex)), up = attn::pow2s(float(Ex));
#pragma unroll
          for (int t = 0; t < C::MT; ++t)
#pragma unroll
            for (int k = 0; k < 4; ++k) O[t][k] *= down;
          const uint32_t b0 = E::pack2(pv[0], pv[1]), b1 = E::pack2(pv[2], pv[3]);
          const int ta = 16 * c + 4 * qd;   // tokens ta, ta + 2 (even), ta + 1, ta + 3 (odd)
#pragma unroll
          for (int t = 0; t < C::MT; ++t) {
            const uint32_t col = uint32_t(16 * t + 2 * r) * 2;
            const uint32_t w0 = attn::lds<uint32_t>(vsp, (ta + 0) * C::RP + col);
            const uint32_t w2 = attn::lds<uint32_t>(vsp, (ta + 2) * C::RP + col);
            const uint32_t w1 = attn::lds<uint32_t>(vsp, (ta + 1) * C::RP + col);
            const uint32_t w3 = attn::lds<uint32_t>(vsp, (ta + 3) * C::RP + col);
            uint32_t av[4];
            av[0] = prmt(w0, w2, 0x5410u);   // row r: channel 16t + 2r, tokens ta, ta + 2
            av[1] = prmt(w0, w2, 0x7632u);   // row r + 8: channel 16t + 2r + 1
            av[2] = prmt(w1, w3, 0x5410u);
            av[3] = prmt(w1, w3, 0x7632u);
            mma16816<DT>(O[t], av, b0, b1);
          }
#pragma unroll
          for (int t = 0; t < C::MT; ++t)
#pragma unroll
            for (int k = 0; k < 4; ++k) O[t][k] *= up;
        }
      }
      if (lane == 0) mbar_arrive(bar(VEMPTY + sv));
    }
  }
  __syncthreads();

  // ---- CTA record: merge the value warps' states ------------------------------
  float *rO = reinterpret_cast<float *>(smem + C::RED_O);
  float *rM = reinterpret_cast<float *>(smem + C::RED_M);
  float *rL = reinterpret_cast<float *>(smem + C::RED_L);
  if (warp < CW) {
    // O = (accumulator - offset + sum p f low) / 2^Ex per (channel, row).
    float L = l_run;
    L += __shfl_xor_sync(0xffffffffu, L, 1);
    L += __shfl_xor_sync(0xffffffffu, L, 2);
    if (qd == 0) {
      rM[warp * 8 + r] = m_run;
      rL[warp * 8 + r] = L;
    }
    const float down = attn::pow2s(float(-Ex));
    float Lg0[C::NG], Lg1[C::NG];
#pragma unroll
    for (int g = 0; g < C::NG; ++g) {
      float v = Ls[g].x + Ls[g].y;
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      Lg0[g] = __shfl_sync(0xffffffffu, v, 8 * qd);
      Lg1[g] = __shfl_sync(0xffffffffu, v, 8 * qd + 4);
    }
    float *wo = rO + warp * 8 * D;
#pragma unroll
    for (int t = 0; t < C::MT; ++t) {
      const int g = t / 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int row = 2 * qd + (k & 1);
        const int ch = 16 * t + 2 * r + (k >> 1);
        wo[row * D + ch] = (O[t][k] - Oc[g][k & 1] + ((k & 1) ? Lg1[g] : Lg0[g])) * down;
      }
    }
  }
  __syncthreads();
  float *rec = p.rec + size_t(cta) * rows * D;
  const int mls = ml_stride(rows);
  float *recml = p.rec_ml + size_t(cta) * mls;
  for (int idx = tid; idx < rows * D; idx += THREADS) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < CW; ++w) M = fmaxf(M, rM[w * 8 + row]);
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) {
      const float mw = rM[w * 8 + row];
      const float wt = mw == -INFINITY ? 0.f : ex2(mw - M);
      acc += rO[(w * 8 + row) * D + d] * wt;
      L += rL[w * 8 + row] * wt;
    }
    rec[idx] = acc;
    if (d == 0) {
      recml[row * 2] = M;
      recml[row * 2 + 1] = L;
    }
  }
  __syncthreads();
  if (tid == 0) {
    unsigned prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(&p.counters[seq * p.hkv + head])
                 : "memory");
    s_last = prev == unsigned(sd.cph - 1);
  }
  __syncthreads();
  if (!s_last) return;
  attn::merge_pair_records<D, DT, THREADS, 8>(p, sd, smem, sbase, s_mbar, NK * C::KST + NV * C::VST,
                                              seq, head, G, nq, rows, tid, warp, lane);
}

}  // namespace split
}  // namespace ckv
