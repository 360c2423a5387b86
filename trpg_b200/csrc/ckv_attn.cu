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


// Wait until the producer has issued `item` into a ring stage (its index is
// published in `slot`), then for that item's data.  A parity wait only tells
// the current phase from the one before it, and the two teams use a ring
// stage alternately, so a team can reach its item while the other team's
// previous item of the stage is still in flight: waiting on the parity alone
// would then match that older phase.  Once the item is known to be issued,
// the stage's barrier is at most one phase behind it and the parity is exact.
__device__ __forceinline__ bool wait_stage(uint32_t bar, volatile int *slot, int item, int ph,
                                           volatile int *abort) {
  if (*slot < item) {
    const long long start = clock64();
    while (*slot < item) {
      if (*abort || clock64() - start > (1ll << 31)) return false;
      __nanosleep(64);   // the producer publishes within a few hundred ns
    }
  }
  return wait_or_abort(bar, ph & 1, abort);
}



template <int BITS, int D, int NT, int DT, int MAXS, bool FOLD>
__global__ void __launch_bounds__(THREADS, 1) attn_kernel(const __grid_constant__ Params<MAXS> p) {
  using C = Cfg<BITS, D, NT, FOLD>;
  using T = typename Elem<DT>::T;
  constexpr int NV = C::NV;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int s_seq, s_last;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_issued[NK + NV];   // last item issued into each K, then V, stage
  // kfull[NK] kempty[NK] vfull[NV] vempty[NV] pfull[TEAMS][2] pempty[TEAMS][2]
  __shared__ __align__(8) uint64_t s_bar[2 * NK + 2 * NV + 4 * TEAMS];
  __shared__ __align__(8) uint64_t s_mbar[2];   // bulk copies of the merge: (m, l), records
  // 1024-byte aligned base: the TMA swizzle patterns repeat every 1024 bytes.
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return smem_u32(&s_bar[i]); };
  constexpr int KFULL = 0, KEMPTY = NK, VFULL = 2 * NK, VEMPTY = 2 * NK + NV,
                PFULL = 2 * NK + 2 * NV, PEMPTY = PFULL + 2 * TEAMS;

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
    for (int i = 0; i < NK + NV; ++i) s_issued[i] = -1;
    for (int i = 0; i < NK; ++i) {
      mbar_init(bar(KFULL + i), 1);
      mbar_init(bar(KEMPTY + i), TEAM_THREADS);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(bar(VFULL + i), 1);
      mbar_init(bar(VEMPTY + i), TEAM_THREADS);
    }
    for (int i = 0; i < 2 * TEAMS; ++i) {
      mbar_init(bar(PFULL + i), TEAM_THREADS);
      mbar_init(bar(PEMPTY + i), TEAM_THREADS);
    }
    mbar_fence_init();
  }
  __syncthreads();
  // The next kernel in the stream may launch now; its CTAs start as this
  // grid's CTAs exit.
  pdl_trigger();
  const int seq = s_seq;
  const SeqDev &sd = p.seq[seq];
  const int local = cta - sd.cta_begin;
  const int head = local / sd.cph, split = local % sd.cph;
  // Item ranges go to the splits in reverse order: the highest CTA indices
  // start last (their SMs are the last ones the previous kernel frees), so
  // they take the first, shortest range of packed blocks, and split 0, which
  // starts first, takes the range that ends with the exact-window chunks.
  const int rsplit = sd.cph - 1 - split;
  const int G = p.group, rows = p.rows, nq = p.nq;

  // This CTA's items: packed units [ub, ue) then residual chunks of RCHUNK tokens.
  const int np = sd.ue - sd.ub;
  const int nr = (sd.re - sd.rb + RCHUNK - 1) / RCHUNK;
  const int ni = np + nr;
  const int ib = int(int64_t(rsplit) * ni / sd.cph);
  const int n = int(int64_t(rsplit + 1) * ni / sd.cph) - ib;
  // Local order of the range: its first packed block (issued before the
  // wait on the previous kernel), then its exact-window chunks (loaded only
  // after that wait, so they get the whole pipeline to arrive), then the
  // other packed blocks.  item(i) is the range's item at local position i.
  // (Filling the whole ring before the wait did not help this kernel: its
  // items are bound by arithmetic, not by the loads.)
  const int npk = max(0, min(n, np - ib));       // packed blocks in the range
  const int nrs = n - npk;                       // window chunks in the range
  auto item = [&](int i) {
    if (npk == 0 || nrs == 0 || i == 0) return ib + i;
    return i <= nrs ? ib + npk + (i - 1) : ib + (i - nrs);
  };

  // Producer side of one packed item: stage st of the K (kchain) or V ring.
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

  // Before waiting for the previous kernel, each producer starts the first
  // packed block: the banks are never written by a kernel of this library
  // that lets its successor start early, so they are complete already.
  // Everything else (query, exact window, workspace, output) comes after the
  // wait.
  int preissued = 0;
  if (warp >= PRODUCER) {
    const bool kchain = warp == PRODUCER;
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(kchain ? &sd.tk : &sd.tv) : "memory");
      if (n > 0 && ib < np) {
        issue_packed(kchain, 0, 0);
        s_issued[kchain ? 0 : NK] = 0;
      }
    }
    preissued = (n > 0 && ib < np) ? 1 : 0;
  }
  pdl_wait();

  // Query B fragments (channel order of the MMA k index) as 16-bit pairs,
  // filled by the QK warps while the producers start streaming.
  if (warp < QK_WARPS) {
    const T *qb = static_cast<const T *>(sd.q);
    for (int x = tid; x < C::KQS * NT * 32; x += QK_WARPS * 32) {
      const int ln = x & 31, nt = (x >> 5) % NT, s = (x >> 5) / NT;
      const int row = 8 * nt + (ln >> 2), cb = 16 * s + 2 * (ln & 3);
      const T *qrow = qb + (head * G + row % G) * sd.q_h + (row / G) * sd.q_n;
      uint2 v = make_uint2(0, 0);
      if (row < rows) {
        const uint16_t *qr = reinterpret_cast<const uint16_t *>(qrow);
        v.x = qr[cb] | (uint32_t(qr[cb + 1]) << 16);
        v.y = qr[cb + 8] | (uint32_t(qr[cb + 9]) << 16);
      }
      *reinterpret_cast<uint2 *>(smem + C::OFF_Q + x * 8) = v;
    }
    named_sync(BAR_QFRAG, QK_WARPS * 32);
  }

  auto fail = [&]() {
    atomicOr(p.error, 1u);
    s_abort = 1;
  };

  const int r = lane >> 2, qd = lane & 3;
  const int team = warp < QK_WARPS ? warp / TEAM_WARPS : (warp - QK_WARPS) / TEAM_WARPS;
  float m_run[NT][2], l_run[NT][2];
  float O[C::MTV][NT][4];
  float Oc[NT][4];     // folded rule: the 1024-offset sum of the value MMAs
  float2 Ls[NT];       // folded rule: sum of p f low for row 8nt + r (this lane's tokens)
  int Ex = 0;          // folded rule: this PV warp's range exponent

  if (warp >= PRODUCER) {
    // ---- producers: warp PRODUCER streams K stages, PRODUCER + 1 V stages -------
    const bool kchain = warp == PRODUCER;
    const int depth = kchain ? NK : NV;
    const int full0 = kchain ? KFULL : VFULL, empty0 = kchain ? KEMPTY : VEMPTY;
    const int stage_bytes = kchain ? C::KST : C::VST;
    const uint32_t ring = sbase + (kchain ? C::OFF_K : C::OFF_V);
    const T *res = static_cast<const T *>(kchain ? sd.rk : sd.rv);
    const int64_t res_h = kchain ? sd.rk_h : sd.rv_h, res_t = kchain ? sd.rk_t : sd.rv_t;
    int issued = preissued;
    for (int i = preissued; i < n; ++i) {
      const int st = i % depth;
      // One lane decides for the warp so that all lanes take the same path.
      int go = 0;
      if (lane == 0) {
        go = !s_abort;
        if (go && i >= depth && !wait_or_abort(bar(empty0 + st), ((i / depth) & 1) ^ 1, &s_abort)) {
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
        // Residual chunk: 16-byte cp.async by every lane into rows of pitch
        // RP.  Rows past the window's end repeat its last token (finite
        // values, masked out of the softmax).
        const int t0 = sd.rb + (it - np) * RCHUNK;
        const int cnt = min(RCHUNK, sd.re - t0);
        const T *src = res + head * res_h;
        constexpr int CH = 2 * D / 16;   // 16-byte pieces per row
        for (int x = lane; x < RCHUNK * CH; x += 32) {
          const int t = x / CH, k = x % CH;
          const int ts = t < cnt ? t : cnt - 1;
          cp_async16(dst + t * C::RP + k * 16, src + int64_t(t0 + ts) * res_t + k * 8);
        }
        cp_async_mbar_arrive(fb);
        __syncwarp();
        if (lane == 0) mbar_arrive(fb);
      }
      __syncwarp();
      if (lane == 0) s_issued[(kchain ? 0 : NK) + st] = i;
      issued = i + 1;
    }
    // Let every issued copy land before the stage memory is reused.
    cp_async_commit();
    cp_async_wait<0>();
    if (lane == 0) {
      for (int st = 0; st < depth && st < issued; ++st) {
        const int last = st + (issued - 1 - st) / depth * depth;
        mbar_wait(bar(full0 + st), (last / depth) & 1);
      }
    }
    __syncwarp();
  } else if (warp < QK_WARPS) {
    // ---- QK warps: team `team`, token quarter q ------------------------------------
    QkWarp<BITS, D, NT, DT, FOLD> qw;
    qw.lane = lane; qw.r = r; qw.qd = qd; qw.q = warp % TEAM_WARPS;
    qw.qfr = smem + C::OFF_Q;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        m_run[nt][j] = -INFINITY;   // this warp's P scale m_q (integer valued)
        l_run[nt][j] = 0.f;
      }
    const float sl = p.scale_log2;
    for (int i = team; i < n; i += TEAMS) {
      const int k = i >> 1, par = k & 1;
      const int st = i % NK;
      const int it = item(i);
      const bool pk = it < np;
      float S[2][NT][4];
      const bool have = !s_abort && wait_stage(bar(KFULL + st), &s_issued[st], i, i / NK, &s_abort);
      if (!have && !s_abort) fail();
      if (have) {
        if (pk) {
          if constexpr (FOLD) qw.packed_fold(sbase + C::OFF_K + st * C::KST, smem + C::OFF_K + st * C::KST, S);
          else qw.packed(smem + C::OFF_K + st * C::KST, S);
        } else {
          qw.resid(sbase + C::OFF_K + st * C::KST, S[0]);
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) S[mt][nt][c] = 0.f;
      }
      mbar_arrive(bar(KEMPTY + st));

      // Scale and mask; S[mt][nt][2u + j] is token tok(mt, u), query row 8nt + 2qd + j.
      const int rbase = sd.rb + (it - np) * RCHUNK;   // residual window index of chunk token 0
      float muse[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int row = 8 * nt + 2 * qd + j;
          float m = -INFINITY;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              float x = S[mt][nt][2 * u + j] * sl;
              if (!pk) {
                const int ri = rbase + 16 * qw.q + r + 8 * u;
                const bool ok = mt == 0 && ri < sd.re &&
                                (nq == 1 || sd.packed + ri <= sd.length - nq + row / G);
                if (!ok) x = -INFINITY;
              }
              S[mt][nt][2 * u + j] = x;
              m = fmaxf(m, x);
            }
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
          // Raise this warp's scale to the next integer above the new maximum.
          const float mold = m_run[nt][j];
          const float mnew = m > mold ? ceilf(m) : mold;
          l_run[nt][j] *= pow2i(mold - mnew);
          m_run[nt][j] = mnew;
          muse[nt][j] = mnew == -INFINITY ? 0.f : mnew;
        }
      if (k >= 2 && !s_abort &&
          !wait_or_abort(bar(PEMPTY + team * 2 + par), ((k >> 1) & 1) ^ 1, &s_abort))
        fail();
      uint8_t *pb = smem + C::OFF_P + (team * 2 + par) * C::ROWS * PP;
      float *ms = reinterpret_cast<float *>(smem + C::OFF_XM) + ((team * 2 + par) * TEAM_WARPS + qw.q) * C::ROWS;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int row = 8 * nt + 2 * qd + j;
          float sum = 0.f;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (!pk && mt == 1) continue;
              const float pv = ex2(S[mt][nt][2 * u + j] - muse[nt][j]);
              sum += pv;
              const int t = pk ? qw.packed_token(mt, u) : 16 * qw.q + r + 8 * u;
              *reinterpret_cast<T *>(pb + row * PP + ppos(t) * 2) = Elem<DT>::from_f32(pv);
            }
          l_run[nt][j] += sum;
          if (r == 0) ms[row] = m_run[nt][j];
        }
      mbar_arrive(bar(PFULL + team * 2 + par));
    }
  } else {
    // ---- PV warps: team `team`, channel quarter c ----------------------------------
    PvWarp<BITS, D, NT, DT, FOLD> pw;
    pw.lane = lane; pw.r = r; pw.qd = qd; pw.c = (warp - QK_WARPS) % TEAM_WARPS;
#pragma unroll
    for (int i = 0; i < C::MTV; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) O[i][nt][c] = 0.f;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int c = 0; c < 4; ++c) Oc[nt][c] = 0.f;
      Ls[nt] = make_float2(0.f, 0.f);
    }
    // Common scale of this team's accumulator: rows 8nt + 2qd + j (the
    // accumulator columns) and rows 8nt + r (the P fragment columns).
    float Mc[NT][2], Mb[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      Mc[nt][0] = Mc[nt][1] = Mb[nt] = -INFINITY;
    }
    for (int i = team; i < n; i += TEAMS) {
      const int k = i >> 1, par = k & 1;
      const int sv = i % NV;
      const bool pk = item(i) < np;
      bool ok = !s_abort && wait_stage(bar(VFULL + sv), &s_issued[NK + sv], i, i / NV, &s_abort);
      ok = ok && wait_or_abort(bar(PFULL + team * 2 + par), (k >> 1) & 1, &s_abort);
      if (!ok && !s_abort) fail();
      if (ok) {
        const float *ms = reinterpret_cast<const float *>(smem + C::OFF_XM) + (team * 2 + par) * TEAM_WARPS * C::ROWS;
        const uint8_t *vst = smem + C::OFF_V + sv * C::VST;
        // Folded rule: the range exponent of this warp's group, so that the
        // block's largest scale times 2^Ex is 2^12 (P'' <= 2^12 < fp16 max).
        // It moves down whenever a block needs it and up only by more than 8
        // (precision); the accumulators are rescaled by the exact power of two.
        int dE = 0;
        if constexpr (FOLD) {
          if (pk) {
            const float smax = pw.fold_scale_max(vst);
            const int eb = ((__float_as_int(smax) >> 23) & 0xff) - 127 + ((__float_as_int(smax) & 0x7fffff) != 0);
            const int need = smax > 0.f ? max(-60, min(60, 12 - eb)) : Ex;
            if (need < Ex || need > Ex + 8) {
              dE = need - Ex;
              Ex = need;
            }
          }
        }
        // Accumulator rescale: new common scale per accumulator column.
        bool unit = dE == 0;
        float2 a2[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float mx0 = Mc[nt][0], mx1 = Mc[nt][1];
#pragma unroll
          for (int w = 0; w < TEAM_WARPS; ++w) {
            const float2 v = *reinterpret_cast<const float2 *>(ms + w * C::ROWS + 8 * nt + 2 * qd);
            mx0 = fmaxf(mx0, v.x);
            mx1 = fmaxf(mx1, v.y);
          }
          if constexpr (FOLD)
            a2[nt] = make_float2(pow2s(Mc[nt][0] - mx0 + dE), pow2s(Mc[nt][1] - mx1 + dE));
          else
            a2[nt] = make_float2(pow2i(Mc[nt][0] - mx0), pow2i(Mc[nt][1] - mx1));
          unit = unit && (mx0 == Mc[nt][0]) && (mx1 == Mc[nt][1]);
          Mc[nt][0] = mx0;
          Mc[nt][1] = mx1;
        }
        if (!__all_sync(0xffffffffu, unit)) {
#pragma unroll
          for (int m = 0; m < C::MTV; ++m)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              float2 x0 = __fmul2_rn(make_float2(O[m][nt][0], O[m][nt][1]), a2[nt]);
              float2 x1 = __fmul2_rn(make_float2(O[m][nt][2], O[m][nt][3]), a2[nt]);
              O[m][nt][0] = x0.x; O[m][nt][1] = x0.y; O[m][nt][2] = x1.x; O[m][nt][3] = x1.y;
            }
          if constexpr (FOLD) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              Oc[nt][0] *= a2[nt].x; Oc[nt][1] *= a2[nt].y;
              Oc[nt][2] *= a2[nt].x; Oc[nt][3] *= a2[nt].y;
            }
          }
        }
        // P fragment factors 2^(m_q - M) for the fragment column row 8nt + r
        // (times 2^Ex for the folded rule's packed blocks).
        uint32_t fb[TEAM_WARPS][NT];
        float fs[TEAM_WARPS][NT];
        bool same = true;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float mq[TEAM_WARPS];
          float mx = Mb[nt];
#pragma unroll
          for (int w = 0; w < TEAM_WARPS; ++w) {
            mq[w] = ms[w * C::ROWS + 8 * nt + r];
            mx = fmaxf(mx, mq[w]);
          }
          if constexpr (FOLD) Ls[nt] = __fmul2_rn(Ls[nt], make_float2(pow2s(Mb[nt] - mx + dE), pow2s(Mb[nt] - mx + dE)));
          Mb[nt] = mx;
#pragma unroll
          for (int w = 0; w < TEAM_WARPS; ++w) {
            const float f = pow2i(mq[w] - mx);
            same = same && mq[w] == mx;
            fb[w][nt] = Elem<DT>::pack2(f, f);
            if constexpr (FOLD) fs[w][nt] = pow2s(mq[w] - mx + Ex);
          }
        }
        const bool scaled = !__all_sync(0xffffffffu, same);
        const uint8_t *pb = smem + C::OFF_P + (team * 2 + par) * C::ROWS * PP;
        if (pk) {
          if constexpr (FOLD) pw.packed_fold(sbase + C::OFF_V + sv * C::VST, vst, pb, O, Oc, Ls, fs);
          else pw.packed(vst, pb, O, fb, scaled);
        } else if constexpr (FOLD) {
          // The exact window at the accumulator's scale 2^Ex: bring the
          // accumulator to scale 1 around the 16-bit MMAs (fb <= 1 keeps P
          // in range for fp16 queries).
          const float down = pow2s(float(-Ex)), up = pow2s(float(Ex));
#pragma unroll
          for (int m = 0; m < C::MTV; ++m)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int c = 0; c < 4; ++c) O[m][nt][c] *= down;
          pw.resid_fold(vst, pb, O, fb, scaled);
#pragma unroll
          for (int m = 0; m < C::MTV; ++m)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int c = 0; c < 4; ++c) O[m][nt][c] *= up;
        } else {
          pw.resid(vst, pb, O, fb, scaled);
        }
      }
      mbar_arrive(bar(VEMPTY + sv));
      mbar_arrive(bar(PEMPTY + team * 2 + par));
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = Mc[nt][0];
      m_run[nt][1] = Mc[nt][1];
    }
  }
  __syncthreads();

  // ---- CTA record: merge the two teams' states ----------------------------------
  // Stage memory is free now.  red[t][row][d]: team t's accumulator at its
  // common scale M_t; lred[t][q][row] / lms[t][q][row]: QK warp q's row sum
  // and its scale m_q; mrow[t][row] = M_t.
  float *red = reinterpret_cast<float *>(smem);          // [TEAMS][ROWS][D]
  float *lred = red + TEAMS * C::ROWS * D;               // [TEAMS][4][ROWS]
  float *lms = lred + TEAMS * TEAM_WARPS * C::ROWS;      // [TEAMS][4][ROWS]
  float *mrow = lms + TEAMS * TEAM_WARPS * C::ROWS;      // [TEAMS][ROWS]
  if (warp < QK_WARPS) {
    const int q = warp % TEAM_WARPS;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float v = l_run[nt][j];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (r == 0) {
          const int row = 8 * nt + 2 * qd + j;
          lred[(team * TEAM_WARPS + q) * C::ROWS + row] = v;
          lms[(team * TEAM_WARPS + q) * C::ROWS + row] = m_run[nt][j];
        }
      }
  } else if (warp < PRODUCER) {
    const int c = (warp - QK_WARPS) % TEAM_WARPS;
    float *rt = red + team * C::ROWS * D;
    if constexpr (FOLD) {
      // O = ((accumulator - offset) / (1 or 16) + sum p f low) / 2^Ex, in the
      // team's common softmax scale.
      PvWarp<BITS, D, NT, DT, FOLD> pw;
      pw.lane = lane; pw.r = r; pw.qd = qd; pw.c = c;
      const float down = pow2s(float(-Ex));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float L = Ls[nt].x + Ls[nt].y;
        L += __shfl_xor_sync(0xffffffffu, L, 1);
        L += __shfl_xor_sync(0xffffffffu, L, 2);
        const float L0 = __shfl_sync(0xffffffffu, L, 8 * qd);
        const float L1 = __shfl_sync(0xffffffffu, L, 8 * qd + 4);
#pragma unroll
        for (int m = 0; m < C::MTV; ++m)
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int row = 8 * nt + 2 * qd + (cc & 1);
            const float v = (O[m][nt][cc] - Oc[nt][cc & 1]) * pw.fold_inv(cc) + ((cc & 1) ? L1 : L0);
            rt[row * D + pw.fold_channel(m, cc)] = v * down;
          }
      }
    } else {
#pragma unroll
      for (int m = 0; m < C::MTV; ++m)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int row = 8 * nt + 2 * qd + (cc & 1);
            const int ch = (D / 4) * c + C::CPL * r + 2 * m + (cc >> 1);
            rt[row * D + ch] = O[m][nt][cc];
          }
    }
    if (c == 0 && r == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) mrow[team * C::ROWS + 8 * nt + 2 * qd + j] = m_run[nt][j];
    }
  }
  __syncthreads();
  float *rec = p.rec + size_t(cta) * rows * D;
  const int mls = ml_stride(rows);
  float *recml = p.rec_ml + size_t(cta) * mls;
  for (int idx = tid; idx < rows * D; idx += THREADS) {
    const int row = idx / D, d = idx % D;
    const float m0 = mrow[row], m1 = mrow[C::ROWS + row];
    const float M = fmaxf(m0, m1);
    const float w0 = m0 == -INFINITY ? 0.f : ex2(m0 - M);
    const float w1 = m1 == -INFINITY ? 0.f : ex2(m1 - M);
    rec[idx] = red[row * D + d] * w0 + red[(C::ROWS + row) * D + d] * w1;
    if (d == 0) {
      float L[TEAMS] = {0.f, 0.f};
#pragma unroll
      for (int t = 0; t < TEAMS; ++t)
#pragma unroll
        for (int w = 0; w < TEAM_WARPS; ++w) {
          const int x = (t * TEAM_WARPS + w) * C::ROWS + row;
          L[t] += lred[x] * pow2i(lms[x] - mrow[t * C::ROWS + row]);
        }
      recml[row * 2] = M;
      recml[row * 2 + 1] = L[0] * w0 + L[1] * w1;
    }
  }
  __syncthreads();
  if (tid == 0) {
    // Release: the whole CTA's record stores (ordered before this thread by
    // the barrier) become visible with the ticket.  Acquire: for the last
    // CTA, the other CTAs' records are visible to every thread ordered after
    // the next barrier.
    unsigned prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(&p.counters[seq * p.hkv + head])
                 : "memory");
    s_last = prev == unsigned(sd.cph - 1);
  }
  __syncthreads();
  if (!s_last) return;

  merge_pair_records<D, DT, THREADS, C::ROWS>(p, sd, smem, sbase, s_mbar, NK * C::KST + NV * C::VST, seq,
                                              head, G, nq, rows, tid, warp, lane);
}

template <int DT>
__global__ void combine_kernel(const float *__restrict__ parts, int nparts, int64_t rows, int D,
                               int tpr, typename Elem<DT>::T *__restrict__ out) {
  // `tpr` threads per row (32 or the whole block), lanes over the channels
  // (coalesced): many rows take a warp each, few rows a block each.
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / tpr) + threadIdx.x / tpr;
  if (row >= rows) return;
  const int lane = threadIdx.x % tpr;
  const size_t stride = size_t(rows) * (D + 2);
  const float *base = parts + row * (D + 2);
  float M = -INFINITY;
  for (int k = 0; k < nparts; ++k) M = fmaxf(M, base[k * stride + D]);
  for (int d = lane; d < D; d += tpr) {
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
      for (int k = 0; k < nparts; ++k) {
        const float *pr = base + k * stride;
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
  return (s.unit_end - s.unit_begin) + (s.resid_end - s.resid_begin + RCHUNK - 1) / RCHUNK;
}

// Items (blocks / residual chunks) a CTA of a many-pair launch takes on:
// each CTA pays a fixed start-up and a record + merge tail, the tail four
// times larger with 16 query rows than with 4, so the 16-row variant takes
// longer ranges.  Measured on B200 (kernel time from graph replay):
//   64 ragged sequences (1024..8192), 4 rows: 8 items 189 us, 16 items 169 us,
//     24 items 164 us, 32 items 183 us;
//   16 sequences x 4 queries at 16K, 16 rows: 8 items 223 us, 16 items 187 us,
//     24 items 186 us, 32 items 173 us, 44 items 173 us.
int items_per_cta(int rows) { return rows > 8 ? 32 : 24; }

// CTAs per (sequence, KV head): a whole number of waves of one CTA per SM,
// shared out in proportion to each pair's items.
int make_plan(const ckv_attn_args &a, int D, Plan &pl) {
  const int sms = sm_count();
  int64_t total = 0;
  for (int i = 0; i < a.num_seqs; ++i) total += int64_t(seq_items(a.seqs[i])) * a.heads_kv;
  const int64_t per_wave = int64_t(sms) * items_per_cta(a.nq * (a.heads_q / a.heads_kv));
  // Few pairs (each gets at least 8 CTAs of one wave): one wave, however long
  // the ranges -- no wave tails and fewer records to merge.  Many pairs:
  // whole waves of about items_per_cta items, which the block scheduler
  // balances across ragged pairs.
  const int64_t pairs = int64_t(a.num_seqs) * a.heads_kv;
  const int64_t waves =
      pairs * 8 <= sms ? 1 : std::max<int64_t>(1, (total + per_wave - 1) / per_wave);
  const int64_t target = int64_t(sms) * waves;
  // Largest remainders: the pairs' CTA counts add up to the target grid
  // exactly (whole waves), each count within [1, min(items, kMaxCph)].
  int64_t rem[CKV_MAX_SEQS];
  int64_t used = 0;
  for (int i = 0; i < a.num_seqs; ++i) {
    const int items = seq_items(a.seqs[i]);
    const int64_t cap = std::min<int64_t>(std::max(items, 1), kMaxCph);
    const int64_t num = total > 0 ? target * items : 0;
    int64_t c = total > 0 ? num / total : 1;
    rem[i] = total > 0 ? num % total : 0;
    c = std::max<int64_t>(1, std::min<int64_t>(c, cap));
    if (c == cap) rem[i] = -1;
    pl.cph[i] = int(c);
    used += c * a.heads_kv;
  }
  // Hand out whole CTA-per-pair increments (heads_kv CTAs each) by remainder.
  while (used + a.heads_kv <= target) {
    int best = -1;
    for (int i = 0; i < a.num_seqs; ++i)
      if (rem[i] >= 0 && (best < 0 || rem[i] > rem[best])) best = i;
    if (best < 0) break;
    ++pl.cph[best];
    used += a.heads_kv;
    const int items = seq_items(a.seqs[best]);
    rem[best] = pl.cph[best] >= std::min<int64_t>(std::max(items, 1), kMaxCph) ? -1 : 0;
  }
  int grid = 0;
  for (int i = 0; i < a.num_seqs; ++i) {
    pl.cta_begin[i] = grid;
    grid += pl.cph[i] * a.heads_kv;
  }
  pl.grid = grid;
  pl.rows = a.nq * (a.heads_q / a.heads_kv);
  pl.rec_off = kCounterBytes;
  pl.ml_off = pl.rec_off + (size_t(grid) * pl.rows * D * 4 + 255) / 256 * 256;
  pl.bytes = pl.ml_off + (size_t(grid) * ml_stride(pl.rows) * 4 + 255) / 256 * 256;
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
  const cuuint32_t kbox[4] = {cuuint32_t(S), cuuint32_t(D), 1, 1};
  const cuuint32_t one[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle kswz = S == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = enc(&d.tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(s.key_data), kdims,
                   kstr, kbox, one, CU_TENSOR_MAP_INTERLEAVE_NONE, kswz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("key tensor map rejected (bank strides)");
    return CKV_ERR_INVALID;
  }
  const cuuint64_t vdims[3] = {cuuint64_t(C::VROWB), cuuint64_t(s.unit_end) * 128, cuuint64_t(hkv)};
  const cuuint64_t vstr[2] = {cuuint64_t(s.vd_stride_token), cuuint64_t(s.vd_stride_head)};
  const cuuint32_t vbox[3] = {cuuint32_t(C::VBOX), 128, 1};
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

// Encoded tensor maps of recent calls, per host thread: a decode loop passes
// the same banks call after call (they change only when a slab grows or a
// block is compacted), and encoding costs more than a lookup.
struct MapKey {
  const void *kd, *vd;
  int64_t kd_u, kd_h, vd_t, vd_h;
  int32_t unit_end, hkv, bits, d;
  bool operator==(const MapKey &o) const {
    return kd == o.kd && vd == o.vd && kd_u == o.kd_u && kd_h == o.kd_h && vd_t == o.vd_t &&
           vd_h == o.vd_h && unit_end == o.unit_end && hkv == o.hkv && bits == o.bits && d == o.d;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap tk, tv;
  bool used = false;
};

template <int BITS, int D>
int cached_maps(const ckv_seq &s, int hkv, SeqDev &d) {
  constexpr int N = 16;
  thread_local MapEntry cache[N];
  thread_local int next = 0;
  const MapKey key{s.key_data, s.value_data, s.kd_stride_unit, s.kd_stride_head, s.vd_stride_token,
                   s.vd_stride_head, s.unit_end, hkv, BITS, D};
  for (int i = 0; i < N; ++i)
    if (cache[i].used && cache[i].key == key) {
      d.tk = cache[i].tk;
      d.tv = cache[i].tv;
      return CKV_OK;
    }
  const int st = encode_maps<BITS, D>(s, hkv, d);
  if (st != CKV_OK) return st;
  MapEntry &e = cache[next];
  next = (next + 1) % N;
  e.key = key;
  e.tk = d.tk;
  e.tv = d.tv;
  e.used = true;
  return CKV_OK;
}

// Kernel parameters of one call (tensor maps from the per-thread cache).
template <int BITS, int D, int MAXS>
int fill_params(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, Params<MAXS> &p) {
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
      const int st = cached_maps<BITS, D>(s, a.heads_kv, d);
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
  return CKV_OK;
}

// Launch with programmatic stream serialization: this grid may start while
// the previous kernel in the stream finishes (the kernel waits for it before
// touching anything that kernel could have written).  The dynamic shared
// memory attribute belongs to the device's context: set once per context (a
// cudaDeviceReset gives the device a new one).
template <class K, class P>
int launch_kernel(K kern, int smem_bytes, int threads, const Plan &pl, const P &p, cudaStream_t st,
                  std::atomic<unsigned long long> (&configured)[64]) {
  int dev = 0;
  CKV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CKV_ERR_INVALID;
  const unsigned long long ctx = context_id();
  if (ctx == 0 || configured[dev].load(std::memory_order_acquire) != ctx) {
    CKV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
    configured[dev].store(context_id(), std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
  return CKV_OK;
}

template <int BITS, int D, int NT, int DT, int MAXS, bool FOLD>
int launch(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  using C = Cfg<BITS, D, NT, FOLD>;
  static std::atomic<unsigned long long> configured[64];
  Params<MAXS> &p = params_scratch<MAXS>();
  const int fs = fill_params<BITS, D, MAXS>(a, pl, ws, p);
  if (fs != CKV_OK) return fs;
  return launch_kernel(attn_kernel<BITS, D, NT, DT, MAXS, FOLD>, C::SMEM, THREADS, pl, p, st, configured);
}

template <int BITS, int D, int NT, int DT, bool FOLD>
int dispatch_seqs(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  return a.num_seqs == 1 ? launch<BITS, D, NT, DT, 1, FOLD>(a, pl, ws, st)
                         : launch<BITS, D, NT, DT, CKV_MAX_SEQS, FOLD>(a, pl, ws, st);
}
// The folded rule covers D = 128 and 256 (each value warp's channels fill
// whole 16-byte chunks of the stage rows).
template <int BITS, int D, int NT, int DT>
int dispatch_fold(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  if constexpr (D >= 128) {
    if (a.flags & CKV_DEQUANT_FOLDED) return dispatch_seqs<BITS, D, NT, DT, true>(a, pl, ws, st);
  }
  return dispatch_seqs<BITS, D, NT, DT, false>(a, pl, ws, st);
}
template <int BITS, int D, int NT>
int dispatch_dt(const ckv_attn_args &a, const Plan &pl, uint8_t *ws, cudaStream_t st) {
  return a.dtype == CKV_BF16 ? dispatch_fold<BITS, D, NT, CKV_BF16>(a, pl, ws, st)
                             : dispatch_fold<BITS, D, NT, CKV_F16>(a, pl, ws, st);
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
    CKV_CUDA_TRY(cudaMemsetAsync(ws, 0, kCounterBytes, st));
  return args->bits == 8 ? dispatch_d<8>(*args, pl, ws, st) : dispatch_d<4>(*args, pl, ws, st);
}

int static_scratch_error(int *flag, ckv_stream_t stream);   // ckv_static.cu

extern "C" int ckv_attention_error(const void *workspace, int *flag, ckv_stream_t stream) {
  if (!flag) return CKV_ERR_INVALID;
  if (!workspace) return static_scratch_error(flag, stream);
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
  // Enough rows for 16 blocks of 8 warp-rows per SM: a warp per row;
  // otherwise a 256-thread block per row.
  const int tpr = rows >= int64_t(sm_count()) * 128 ? 32 : 256;
  const int64_t per_block = 256 / tpr;
  const unsigned blocks = unsigned((rows + per_block - 1) / per_block);
  if (dtype == CKV_BF16)
    combine_kernel<CKV_BF16><<<blocks, 256, 0, st>>>(partials, parts, rows, head_dim, tpr,
                                                     static_cast<__nv_bfloat16 *>(out));
  else
    combine_kernel<CKV_F16><<<blocks, 256, 0, st>>>(partials, parts, rows, head_dim, tpr,
                                                    static_cast<__half *>(out));
  return cuda_status(cudaGetLastError());
}
