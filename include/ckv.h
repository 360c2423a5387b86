/*
 * ckv.h -- C ABI of the B200 compressed-KV library (libtrpg_ckv.so).
 *
 * Plain pointers, sizes and strides only; every entry point returns a
 * ckv_status and never allocates device memory.  All device pointers must be
 * resident on the current CUDA device; work is enqueued on `stream` and the
 * functions return without synchronising.
 *
 * Cache layout (unchanged from the reference, models/quantized_kv.py:43-66):
 *   key codes   uint8 [B,H,Ucap,D,128/(8/bits)]  one row = one channel over
 *               a 128-token block; Q4 keeps token 2j in the low nibble of
 *               byte j, token 2j+1 in the high nibble
 *   key meta    fp32  [B,H,Ucap,D,2]              (scale, low) per row
 *   value codes uint8 [B,H,Tcap,D/64,64/(8/bits)] one row = one token over a
 *               64-channel group; Q4 keeps channel 2j low, 2j+1 high
 *   value meta  fp32  [B,H,Tcap,D/64,2]
 *   residual    bf16|fp16 [B,H,R,D]               exact recent window
 * Inner dimensions (the last two of every bank) must be dense; head and
 * unit/token strides are free (slab capacity).  All strides are in elements
 * of their own tensor.
 */
#ifndef TRPG_CKV_H
#define TRPG_CKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ckv_stream_t; /* identical to cudaStream_t */

typedef enum {
  CKV_OK = 0,
  CKV_ERR_INVALID = 1,     /* bad pointer, size, stride or alignment */
  CKV_ERR_UNSUPPORTED = 2, /* valid request this build has no kernel for */
  CKV_ERR_WORKSPACE = 3,   /* workspace missing or too small */
  CKV_ERR_CUDA = 4         /* a CUDA call or launch failed */
} ckv_status;

typedef enum { CKV_BF16 = 0, CKV_F16 = 1 } ckv_dtype;
typedef enum { CKV_ROUND_HALF_EVEN = 0, CKV_ROUND_HALF_UP = 1 } ckv_rounding;

/* Human-readable text for a status code (static storage). */
const char *ckv_status_string(int status);
/* Last CUDA error string recorded by this thread, or "" (static storage). */
const char *ckv_last_error(void);
/* ABI version: (major << 16) | minor. */
int ckv_version(void);

/* ---------------------------------------------------------------------- */
/* Quantizer                                                               */
/* ---------------------------------------------------------------------- */

/*
 * Affine-quantize `rows` dense rows of `group` (64 or 128) elements each.
 * Per row: low = min, scale = max((max - low) / (2^bits - 1), 1e-8),
 * code = clamp(round((x - low) / scale), 0, 2^bits - 1) with IEEE fp32
 * arithmetic; `rounding` selects half-to-even (the reference CPU quantizer,
 * models/quantized_kv.py:19-25) or half-up (the reference Triton kernel,
 * models/quantized_kv_kernels.py:7-22).  Q4 packs code 2j | code 2j+1 << 4.
 * Replaces models/quantized_kv_kernels.py:39 `pack(rows, bits)`.
 * codes: rows*group*bits/8 bytes; meta: rows*2 floats (scale, low).
 */
int ckv_pack_rows(const void *x, int dtype, int64_t rows, int group, int bits,
                  int rounding, uint8_t *codes, float *meta, ckv_stream_t stream);

/*
 * Dequantize: out = round_to_dtype(fma(code, scale, low)), one rounding of
 * the fused multiply-add, as the reference CUDA path does.
 * Replaces models/quantized_kv_kernels.py:50 `unpack(data, meta, bits, dtype)`.
 */
int ckv_unpack_rows(const uint8_t *codes, const float *meta, int64_t rows, int group,
                    int bits, int dtype, void *out, ckv_stream_t stream);

/* Direct-to-slab bank append: quantize `count` (a multiple of 128) tokens of
 * one sequence's residual window straight into the key and value banks at
 * unit `unit_offset` (token unit_offset*128).  Same arithmetic as
 * ckv_pack_rows; replaces the pack + copy_ pair of
 * models/quantized_kv.py:43-66 (`_PackedBank.append`). */
typedef struct {
  const void *keys;    /* residual [H,R,D]: strides below, last dim dense */
  const void *values;
  int64_t k_stride_head, k_stride_token;
  int64_t v_stride_head, v_stride_token;
  uint8_t *key_data;   /* bank base pointers (batch index 0) */
  float *key_meta;
  uint8_t *value_data;
  float *value_meta;
  int64_t kd_stride_head, kd_stride_unit;   /* key codes: dims 1 and 2 */
  int64_t km_stride_head, km_stride_unit;
  int64_t vd_stride_head, vd_stride_token;
  int64_t vm_stride_head, vm_stride_token;
  int32_t heads, head_dim, bits, dtype, rounding;
  int32_t count;        /* tokens to quantize, multiple of 128 */
  int32_t unit_offset;  /* first destination unit */
} ckv_append_args;

int ckv_pack_append(const ckv_append_args *args, ckv_stream_t stream);

/* Append `tokens` new rows per head to the exact (residual) window, in place:
 * keys[h][offset + t] = keys_new[h][t], the same for values, one launch for
 * both.  Replaces the torch.cat pair of models/quantized_kv.py:109-110
 * (`append_for_attention`) when the window lives in a buffer with spare
 * capacity.  16-bit elements; rows must be dense and 16-byte aligned
 * (strides in elements, multiples of 8). */
typedef struct {
  const void *keys_new;   /* [H][tokens][D] */
  const void *values_new;
  int64_t kn_stride_head, kn_stride_token;
  int64_t vn_stride_head, vn_stride_token;
  void *keys;             /* window buffers [H][capacity][D] */
  void *values;
  int64_t k_stride_head, k_stride_token;
  int64_t v_stride_head, v_stride_token;
  int32_t heads, tokens, head_dim, offset;
} ckv_residual_args;

int ckv_residual_append(const ckv_residual_args *args, ckv_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Attention over a compressed view                                         */
/* ---------------------------------------------------------------------- */

/*
 * One sequence.  Queries attend to packed tokens [unit_begin*128,
 * unit_end*128) and residual tokens [resid_begin, resid_end) (indices into
 * the residual window; absolute position packed_tokens + index).  A full view
 * uses unit_begin = 0, unit_end = packed_tokens/128, resid_begin = 0,
 * resid_end = R.  A split-KV shard narrows the ranges.
 * Query row (n, g) of KV head h is query head h*G + g, query position n
 * (0..nq-1, the last nq positions of the sequence).  With nq > 1 the mask is
 * lower-right causal: query n sees absolute position p iff
 * p <= length - nq + n (models/compressed_prefill_kernels.py:81,90).
 */
typedef struct {
  const void *query;            /* [Hq,nq,D] dtype, last dim dense */
  int64_t q_stride_head, q_stride_pos;
  const uint8_t *key_data;  int64_t kd_stride_head, kd_stride_unit;
  const float *key_meta;    int64_t km_stride_head, km_stride_unit;
  const uint8_t *value_data; int64_t vd_stride_head, vd_stride_token;
  const float *value_meta;  int64_t vm_stride_head, vm_stride_token;
  const void *keys;         int64_t rk_stride_head, rk_stride_token;
  const void *values;       int64_t rv_stride_head, rv_stride_token;
  int64_t packed_tokens;        /* P, a multiple of 128 */
  int64_t length;               /* L = P + R */
  int32_t unit_begin, unit_end;
  int32_t resid_begin, resid_end;
  void *out;                    /* normalized: [Hq,nq,D] dtype, dense
                                   partial:    see ckv_attn_args.partial */
} ckv_seq;

typedef struct {
  const ckv_seq *seqs;          /* host array of `num_seqs` descriptors */
  int32_t num_seqs;
  int32_t heads_q, heads_kv, head_dim, nq, bits, dtype;
  float scale;                  /* softmax scale applied to q.k */
  /* partial = 0: write normalized outputs to seqs[i].out.
   * partial = 1: write unnormalized split-KV partials, fp32, to
   *   seqs[i].out laid out as [Hq*nq rows] x (D + 2): row (h*G+g)*nq... see
   *   ckv_partial_row(); o[0..D) = sum 2^(s - m) v, then m (log2 domain,
   *   -inf if the shard saw no token) and l = sum 2^(s - m). */
  int32_t partial;
  int32_t flags;                /* CKV_WS_COUNTERS_ZERO, ... */
} ckv_attn_args;

#define CKV_WS_COUNTERS_ZERO 1  /* caller guarantees the workspace header and
                                   ticket region are zero; the call leaves the
                                   tickets at zero */
#define CKV_DEQUANT_FOLDED 2    /* folded dequantization (head_dim 128 or 256;
                                   other sizes use the exact rule): the scales
                                   go into the query and probability operands
                                   and the codes reach the tensor cores as
                                   exact fp16 values; results agree with the
                                   exact rule to fp16 rounding of q*scale and
                                   p*scale instead of bf16 rounding of every
                                   dequantized value */

/* Maximum sequences in one ckv_attention call (the per-sequence descriptors,
 * TMA tensor maps included, travel as kernel parameters). */
#define CKV_MAX_SEQS 64

/* Bytes of workspace ckv_attention needs for `args` (host only: reads the
 * current device's SM count, launches nothing). */
int ckv_attention_workspace(const ckv_attn_args *args, size_t *bytes);

/* Copy the workspace's error word to *flag and wait for the stream: 0, or 1
 * when a kernel gave up waiting for an asynchronous copy (about a second)
 * instead of hanging.  The word stays set until the caller clears it.
 * workspace == NULL reads the word of the current device's static scratch
 * array instead (see ckv_attention_static; every static call clears it
 * before its kernel runs, so it reports the latest static call). */
int ckv_attention_error(const void *workspace, int *flag, ckv_stream_t stream);

/*
 * Split-KV GQA attention over compressed views (decode when nq == 1,
 * multi-query verify when nq > 1).  Dequantizes in registers with the
 * reference's rounding (fma then round to the query dtype,
 * models/compressed_kv_kernels.py:47,68), online softmax in the log2 domain
 * (:51-58), fp32 accumulation, and merges split partials with the
 * log-sum-exp rule of :85-89 inside the same launch.  Replaces
 * models/compressed_kv_kernels.py:93 `decode(query, view, scale)` and, for
 * nq > 1, the dequantize + SDPA(causal_lower_right) verify path
 * (models/quantized_kv.py:126-134 then scaled_dot_product_attention).
 * workspace: ckv_attention_workspace() bytes, 256-byte aligned.
 */
int ckv_attention(const ckv_attn_args *args, void *workspace, size_t workspace_bytes,
                  ckv_stream_t stream);

/* Size of the library's own scratch buffer used by ckv_attention_static. */
#define CKV_STATIC_SCRATCH_BYTES (4u << 20)

/*
 * ckv_attention without a caller workspace, for callers that may not
 * allocate device memory where they call it: a host function enqueued on a
 * stream, an allocator or memory-pool hook (allocating there re-enters the
 * allocator), or an embedding runtime that owns every device allocation and
 * hands out none for scratch.  Same arguments and results as ckv_attention;
 * the split records and merge tickets go to a CKV_STATIC_SCRATCH_BYTES
 * (4 MiB) array inside the library instead, so the call allocates nothing.
 * Each device that loads the library holds its own copy of that array until
 * the process exits.  A request whose ckv_attention_workspace() exceeds
 * CKV_STATIC_SCRATCH_BYTES returns CKV_ERR_WORKSPACE before any GPU work.
 * The ticket area is cleared on the stream at every call.  The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.
 * Every call on one device uses the same array: two calls whose kernels can
 * overlap on the GPU (different streams without ordering between them) race
 * and give wrong results, so the caller must serialise them.  A bounded wait
 * that gave up inside the kernel is reported by
 * ckv_attention_error(NULL, &flag, stream) for this array.  The array's
 * address is cached per device and CUDA context, so a cudaDeviceReset is
 * followed by a fresh lookup on the next call.
 * No counterpart in the reference.
 */
int ckv_attention_static(const ckv_attn_args *args, ckv_stream_t stream);

/* Row index of (query head hq, position n) in a partial buffer. */
static inline int64_t ckv_partial_row(int hq, int n, int nq) { return (int64_t)hq * nq + n; }

/*
 * Merge `parts` split-KV partials (each rows x (D+2) fp32 as written by
 * ckv_attention with partial = 1, stored back to back in `partials`) into
 * normalized outputs [rows, D] of `dtype`.  Same rule as
 * models/compressed_kv_kernels.py:85-89; shards that saw no token (m = -inf)
 * get weight 0.
 */
int ckv_combine_partials(const float *partials, int parts, int64_t rows, int head_dim,
                         int dtype, void *out, ckv_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Packed prefill                                                          */
/* ---------------------------------------------------------------------- */

/*
 * Lower-right causal attention of a query chunk over the whole quantized
 * history plus the exact residual window, which already holds the chunk
 * (the caller appends before and compacts after).  Replaces the kernel
 * behind models/compressed_prefill_attention.py:6-52
 * (models/compressed_prefill_kernels.py:29-111).
 *
 * seq:   query [Hq,qlen,D] (q_stride_head, q_stride_pos multiples of 8, base
 *        16-byte aligned), the banks as for ckv_attention, the residual
 *        [Hkv,R,D] (strides multiples of 8, bases 16-byte aligned) and out
 *        [Hq,qlen,D] dense.  The ranges must cover the whole history:
 *        unit_begin = 0, unit_end = P/128, resid_begin = 0, resid_end = R.
 * Needs P >= 128 and R >= qlen.  Residual token t is visible to query
 * position n iff t <= R - qlen + n; every packed token is visible.
 *
 * One CTA per (KV head, 128 query rows).  When that grid would leave SMs
 * idle (short of one wave, or a part-empty last wave), each CTA's history is
 * split across more CTAs; they write (o, m, l) partial records to the
 * workspace and a ckv_combine_partials launch writes `out`.
 */
typedef struct {
  ckv_seq seq;
  int32_t heads_q, heads_kv, head_dim, qlen, bits, dtype;
  float scale;                  /* softmax scale applied to q.k */
} ckv_prefill_args;

/* Workspace bytes ckv_prefill needs for `args` (0 when the history is not
 * split; host only: reads the current device's SM count, launches nothing). */
int ckv_prefill_workspace(const ckv_prefill_args *args, size_t *bytes);

/* workspace: ckv_prefill_workspace() bytes, 16-byte aligned (may be NULL
 * when that is 0). */
int ckv_prefill(const ckv_prefill_args *args, void *workspace, size_t workspace_bytes,
                ckv_stream_t stream);
/* 1 if a ckv_prefill launch on the current device gave up a bounded wait on
 * its tensor-core products since the last call (its outputs are then not
 * valid); read and cleared on `stream`, which it synchronises. */
int ckv_prefill_error(int *flag, ckv_stream_t stream);
/* Selects the prefill kernel for head_dim 128 / 256 (process-wide): 2 (the
 * default) the pipelined tcgen05 kernel (operands in shared memory,
 * accumulators in tensor memory; producer warps dequantize the next tile
 * while the products and the softmax of this one run), 1 the tcgen05 kernel
 * with its phases in order, 0 the mma.sync kernel.  Same results up to fp32
 * summation order.  Returns CKV_ERR_INVALID for another value. */
int ckv_prefill_set_tensor_cores(int on);

/* ---------------------------------------------------------------------- */
/* Split-KV partials exchanged over peer memory (one process per GPU)     */
/* ---------------------------------------------------------------------- */

/*
 * The cross-GPU half of sequence-split-KV decode without a collective
 * library: every rank owns one exchange buffer, maps every other rank's
 * buffer into its address space (CUDA IPC over NVLink, plain peer mappings,
 * no multicast), and one launch per rank and step
 *   1. writes this rank's partial (rows x (D+2) fp32, as ckv_attention with
 *      partial = 1 leaves it) into every rank's buffer, each value as one
 *      8-byte word together with the step number that wrote it;
 *   2. merges the world partials into `out` [rows, D] of `dtype`, with the
 *      rule of ckv_combine_partials (models/compressed_kv_kernels.py:85-89),
 *      reading each word once its step field shows this step (an aligned
 *      8-byte store is seen whole, so no fence or separate flag is needed);
 *      the wait is bounded: after `spin_limit` clock cycles (2^31 when 0) it
 *      sets the buffer's error word and leaves the output unwritten.
 * The step number is a counter in the buffer that each launch advances, so
 * the launch can be captured in a CUDA graph and replayed. Partials
 * alternate between two slots by step parity: a rank's step s + 1 waits for
 * every rank's step s + 1 partial, which each rank publishes only after its
 * own step s, so no rank overwrites a slot that another rank is still
 * reading. Every rank must make the same sequence of calls.
 *
 * Buffer: ckv_exchange_bytes(world, rows, head_dim) bytes, zeroed, from
 * ckv_exchange_alloc; world <= CKV_EXCHANGE_MAX_WORLD.
 */
#define CKV_EXCHANGE_MAX_WORLD 8
size_t ckv_exchange_bytes(int world, int64_t rows, int head_dim);
/* cudaMalloc + clear of one exchange buffer on the current device, and its
 * CUDA IPC handle (64 bytes) for the other ranks. */
int ckv_exchange_alloc(int world, int64_t rows, int head_dim, void **buffer,
                       unsigned char handle[64]);
/* Map another rank's buffer (from its handle) into this process. */
int ckv_exchange_open(const unsigned char handle[64], void **peer_buffer);
/* Unmap a buffer from ckv_exchange_open / free one from ckv_exchange_alloc.
 * No launch that uses it may still be in flight on any rank. */
int ckv_exchange_close(void *peer_buffer);
int ckv_exchange_free(void *buffer);
/* buffers[r]: rank r's buffer as seen by this process (buffers[rank] is this
 * rank's own).  phases: 3 for both phases in one launch (one rank per GPU);
 * 1 (publish only) and 2 (wait and merge only) let one process drive several
 * ranks' buffers on one GPU without launches that wait on each other. */
int ckv_exchange_combine(const float *partial, int64_t rows, int head_dim, void *const *buffers,
                         int world, int rank, int phases, long long spin_limit, int dtype,
                         void *out, ckv_stream_t stream);
/* The buffer's error word (1 after a wait gave up), read and cleared on
 * `stream` (synchronises the stream). */
int ckv_exchange_error(void *buffer, int *flag, ckv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TRPG_CKV_H */
