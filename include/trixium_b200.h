/*
 * trixium_b200.h -- C ABI of the B200 ternary decode path (libtrixium_b200.so).
 *
 * The library replaces the TriXium engine's matvec and the vector-unit operations that wrap it
 * on the decode path.  Every entry point:
 *   - takes device pointers (caller-owned) and a cudaStream_t, and only enqueues work;
 *   - returns a trx_status (0 = ok, < 0 = error); arguments are checked on the host before
 *     anything is enqueued, and nothing aborts the process;
 *   - reports conditions found on the device (int48/int32 overflow, invalid trit5 bytes,
 *     a bounded wait that ran out) in the context's error word, read with trx_get_error().
 *
 * Packed tensors are the converter's row packets byte for byte: per output row
 * [ceil(G/16) x 32 bytes of fp16 group scales][codes: 2-bit (kind 0) or 5 trits per byte,
 * 26 bytes per 128-group (kind 5), padded to 32 bytes], rows back to back
 * (reference: model/layout.py:17-30, :184-217; model/bons.py:115-175).  The device pointer of a
 * packed tensor must be 16-byte aligned.
 */
#ifndef TRIXIUM_B200_H
#define TRIXIUM_B200_H

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int trx_status;

#define TRX_OK               0
#define TRX_ERR_ARG         -1   /* bad pointer, size, alignment or parameter */
#define TRX_ERR_LAYOUT      -2   /* kind/cols not a ternary row-packet layout; invalid trit5 byte */
#define TRX_ERR_OVERFLOW    -3   /* |acc| >= 2^47 or |result| >= 2^31 (model/bitexact.py:116,118) */
#define TRX_ERR_CUDA        -4   /* a CUDA runtime call failed */
#define TRX_ERR_TIMEOUT     -5   /* a bounded device-side wait ran out */
#define TRX_ERR_UNSUPPORTED -6

/* Error-word bits (trx_get_error). */
#define TRX_DEV_OVERFLOW   0x1u
#define TRX_DEV_BADBYTE    0x2u
#define TRX_DEV_TIMEOUT    0x4u
#define TRX_DEV_INTERNAL   0x8u   /* a launch found shared memory laid out unlike its plan */
#define TRX_DEV_RANGE      0x10u  /* an index read from device memory (a position) was out of range */

#define TRX_KIND_TERNARY   0    /* KIND_TERNARY,  model/layout.py:46 */
#define TRX_KIND_Q8        1    /* KIND_Q8,       model/layout.py:47 (int8 weights, group 32) */
#define TRX_KIND_TERNARY5  5    /* KIND_TERNARY5, model/layout.py:50 */

/* The fields of a BONS tensor-table entry a matvec needs (model/layout.py:311-333). */
typedef struct trx_entry {
    uint32_t rows;      /* output rows (this device's shard)       */
    uint32_t cols;      /* K, a multiple of 128                     */
    int32_t  kind;      /* TRX_KIND_TERNARY or TRX_KIND_TERNARY5   */
    int32_t  bias;      /* B: the tensor's scale bias  (entry byte 36) */
    int32_t  rshift;    /* R: the tensor's result shift (entry byte 37) */
} trx_entry;

/* Per-device context: the device error word and the library's scratch. */
typedef struct trx_ctx trx_ctx;

/* Create a context on `device` (allocates its scratch; call outside stream capture). */
trx_status trx_create(trx_ctx **ctx, int device);
trx_status trx_destroy(trx_ctx *ctx);

/* Synchronise `stream`, return the accumulated device error bits in *bits and clear them. */
trx_status trx_get_error(trx_ctx *ctx, cudaStream_t stream, uint32_t *bits);

/* The message of the CUDA error behind the last TRX_ERR_CUDA returned on this thread. */
const char *trx_last_cuda_error(void);

/* Bytes of one row packet (model/layout.py:215-217): ternary kinds (cols % 128 == 0) and
 * TRX_KIND_Q8 (cols % 32 == 0); 0 for any other kind or width. */
uint64_t trx_row_bytes(uint32_t cols, int32_t kind);

/*
 * Integer engine matvec: out[n] = (sum_g (gs[n,g]*m11[n,g]) <<or>> (e16[n,g]+B)) >> R as int32,
 * gs the exact sum over the group of (code-1)*x8.  Bit-exact with model/bitexact.py:101-119
 * (matvec_ternary).  x8: K int8.
 */
trx_status trx_matvec_i8(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                         const int8_t *d_x8, int32_t *d_out, cudaStream_t stream);

/*
 * Q8 row-dot engine matvec over KIND_Q8 row packets (e->kind == TRX_KIND_Q8; cols a multiple of
 * 32, at most 32768): out[n] = (sum_g (gs[n,g]*m11[n,g]) <<or>> (e16[n,g]+B)) >> R as int32, gs the
 * exact sum over the 32-weight group of q8w*x8.  Bit-exact with model/bitexact.py:127-144
 * (matvec_q8), the mode of Q8 tensors in the engine's matvec (model/mirror.py:672-675) and of the
 * K-cache scores (model/mirror.py:243-253).  Where the reference asserts (int48 accumulator,
 * int32 result; :141, :143) TRX_DEV_OVERFLOW is set in the error word.  x8: K int8.
 */
trx_status trx_matvec_q8(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                         const int8_t *d_x8, int32_t *d_out, cudaStream_t stream);

/*
 * Float projection of a KIND_Q8 tensor in the engine's arithmetic (model/mirror.py:664-678 with
 * its Q8 branch :672-675, one K-segment): x8, e8 = the power-of-two quantisation of x (as
 * trx_quantize_pow2), then y = float(trx_matvec_q8 result) * 2^(e8 + R - B).  Two launches on
 * `stream`; the quantised x lives in the context's scratch, so calls on one context are
 * serialised by the caller (one stream at a time).  x: K floats, y: rows floats.
 */
trx_status trx_matvec_q8_f(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                           const float *d_x, float *d_y, cudaStream_t stream);

/*
 * Multi-row engine matvec: nb independent rows of x8 ([nb, K] int8) against one weight pass,
 * out [nb, rows] int32 (model/bitexact.py:121-125, matvec_ternary_rows).  nb <= 32: up to 8 rows
 * on the integer dot-product path, 9..32 on the tensor cores (tcgen05 kind::i8, decoded codes times
 * the rows, exact int32 group sums, the engine's int64 scale epilogue).  The tensor-core form uses
 * the context's scratch: calls on one context must not overlap.
 */
trx_status trx_matvec_i8_rows(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                              const int8_t *d_x8, int nb, int32_t *d_out, cudaStream_t stream);

/*
 * Batched float projection: nb <= 32 independent fp32 rows x [nb, K] (a decode batch), each
 * quantised with its own power-of-two exponent (model/mirror.py:45-51), against one weight pass on
 * the tensor cores, y [nb, rows] = float(int32 result) * 2^(e8_row + R - B) (model/mirror.py:664-678
 * per row), plus d_resid [nb, rows] when not NULL.  Two launches (the rows' quantisation, the
 * tensor-core matvec) on the context's scratch.
 */
trx_status trx_matvec_f_rows(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                             int nb, const float *d_resid, float *d_y, cudaStream_t stream);

/*
 * The batched form of trx_matvec_f_multi: nseg <= 4 tensors of the same cols and kind, their row
 * packets back to back in d_packed, on the same nb <= 32 activation rows d_x [nb][cols] (each row
 * optionally RMS-normalised with d_norm_w first, the canonical sum of squares of
 * model/mirror.py:576-591,697-700, then quantised with its own exponent); segment i's rows go to
 * d_y[i] [nb][rows_i] (device pointers in a host array), plus d_resid[i] when d_resid (a host array
 * of device pointers or NULLs) is given.  One tensor-core launch (model/bitexact.py:121-125 per
 * tensor, model/mirror.py:648-678 per row).
 */
trx_status trx_matvec_f_rows_multi(trx_ctx *ctx, const trx_entry *entries, int nseg, const void *d_packed,
                                   const float *d_x, int nb, const float *d_norm_w, float eps, float *const *d_y,
                                   const float *const *d_resid, cudaStream_t stream);

/* The per-row steps around the batched projections of a decode batch (nrows independent sequences;
 * model/mirror.py:1002-1034 per sequence):
 *   trx_embed_lookup_rows: x[r] = table[tokens[r]] (as trx_embed_lookup, fp16 or fp32 table);
 *   trx_rmsnorm_rows: y[r] = RMSNorm(x[r]) * w (as trx_rmsnorm), rows of n floats;
 *   trx_silu_mul: act = silu(g) * u elementwise over n floats (model/mirror.py:713,1020);
 *   trx_argmax_rows: tokens[r] = the largest of logits[r][0..V), ties to the smallest index;
 *   trx_advance_positions: pos[i] += n for i < count. */
trx_status trx_embed_lookup_rows(trx_ctx *ctx, const void *d_table, uint32_t vocab, uint32_t dim, int32_t f16,
                                 const int32_t *d_tokens, int32_t nrows, float *d_x, cudaStream_t stream);
trx_status trx_rmsnorm_rows(trx_ctx *ctx, const float *d_x, const float *d_w, uint32_t n, int32_t nrows, float eps,
                            float *d_y, cudaStream_t stream);
trx_status trx_silu_mul(trx_ctx *ctx, const float *d_g, const float *d_u, uint64_t n, float *d_act,
                        cudaStream_t stream);
trx_status trx_argmax_rows(trx_ctx *ctx, const float *d_logits, uint32_t V, int32_t nrows, int32_t *d_tokens,
                           cudaStream_t stream);
trx_status trx_advance_positions(trx_ctx *ctx, int32_t *d_pos, int32_t count, int32_t n, cudaStream_t stream);

/*
 * Power-of-two int8 activation quantisation: e8 = frexp(max|x|) - 7,
 * x8 = clamp(lround(x * 2^-e8), -127, 127) with the mirror's rounding (floor(x+0.5) in fp32).
 * model/mirror.py:45-51; firmware/infer_internal.h:60-124 (f32_quant_e8, f32_pack_q8x4).
 * d_e8: one int32 on the device.
 */
trx_status trx_quantize_pow2(trx_ctx *ctx, const float *d_x, uint32_t n, int8_t *d_x8,
                             int32_t *d_e8, cudaStream_t stream);

/*
 * Float projection in the engine's arithmetic (the firmware's infer_matvec_f,
 * firmware/infer_float.c:398; model/mirror.py:648-678): quantise x (the whole vector, one
 * exponent), the integer matvec, y = float(int32) * 2^(e8 + R - B).  Fused in one launch.
 * If d_norm_w is not NULL, x is first RMS-normalised with the canonical 64-partial sum of
 * squares: x <- (x * 1/sqrt(ss/K + eps)) * w  (model/mirror.py:697-700, :576-591).
 * If d_resid is not NULL, y = resid + projection (the residual add, model/mirror.py:1013,1024).
 */
trx_status trx_matvec_f(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                        const float *d_x, const float *d_norm_w, float eps,
                        const float *d_resid, float *d_y, cudaStream_t stream);

/*
 * fp-mode projection: y[n] = sum_g scale[n,g] * sum_{j in g} (code-1) * x_j in fp32
 * (model/fastref.py:103-125, HybridRef.matmul for one row of X).
 */
trx_status trx_matvec_fp(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                         const float *d_x, float *d_y, cudaStream_t stream);

/*
 * fp-mode projection of nrows rows (model/fastref.py:119-125, HybridRef.matmul(entry, X)):
 * d_y [nrows][rows] = d_x [nrows][cols] . W^T in fp32, W = (code - 1) * scale; d_resid (or NULL),
 * [nrows][rows], is added (the K-segments of one entry accumulate this way).
 */
trx_status trx_matvec_fp_rows(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                              int32_t nrows, const float *d_resid, float *d_y, cudaStream_t stream);

/*
 * Gate/up projection with the SwiGLU epilogue (model/mirror.py:1016-1020;
 * model/fastref.py:253-255): act[i] = silu(gate(x)[i]) * up(x)[i], both projections in the
 * engine's arithmetic on the same quantised (optionally RMS-normalised) x.
 */
trx_status trx_matvec_swiglu(trx_ctx *ctx, const trx_entry *gate, const void *d_gate,
                             const trx_entry *up, const void *d_up,
                             const float *d_x, const float *d_norm_w, float eps,
                             float *d_act, cudaStream_t stream);

/* Check a packed trit5 tensor for bytes above 242 (gateware/core/trit5.py:37-39).  Sets
 * TRX_DEV_BADBYTE in the error word when one is found. */
trx_status trx_validate_packed(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                               cudaStream_t stream);

/*
 * Batched benchmark/driver form: njobs independent float projections (one launch), job j
 * reading x + j*x_stride and packed + j*w_stride, writing y + j*y_stride.  Same arithmetic as
 * trx_matvec_f without norm or residual.
 */
trx_status trx_matvec_f_batch(trx_ctx *ctx, const trx_entry *e, const void *d_packed,
                              uint64_t w_stride, const float *d_x, uint64_t x_stride,
                              float *d_y, uint64_t y_stride, int njobs, cudaStream_t stream);

/*
 * Several tensors on one input in one launch (q/k/v of an attention layer, qkv/z/beta/alpha of a
 * DeltaNet layer): nseg <= 4 entries with the same cols and kind, their row packets back to back
 * in d_packed (segment i after the rows of segments 0..i-1).  Each segment is trx_matvec_f of its
 * entry on the same (optionally RMS-normalised) x (mirror.py proj(): every projection quantises the
 * same input, so the quantisation is shared exactly); d_y[i] (device pointers, given in a host
 * array) receives segment i's rows; d_resid, if not NULL, is a host array of nseg device pointers
 * or NULLs added to the results.
 */
trx_status trx_matvec_f_multi(trx_ctx *ctx, const trx_entry *entries, int nseg, const void *d_packed,
                              const float *d_x, const float *d_norm_w, float eps, float *const *d_y,
                              const float *const *d_resid, cudaStream_t stream);

/* x = table[*d_token] as fp32 (table [vocab][dim], fp16 when f16 != 0, else fp32); a token
 * outside [0, vocab) sets TRX_DEV_RANGE and writes zeros (model/mirror.py:1003 embed_row). */
trx_status trx_embed_lookup(trx_ctx *ctx, const void *d_table, uint32_t vocab, uint32_t dim, int32_t f16,
                            const int32_t *d_token, float *d_x, cudaStream_t stream);

/* x = mant[*d_token] * 2^exp[*d_token] as fp32: the int16 embedding table of a BONS image
 * (ROLE_TOK_EMB16 rows [vocab][dim] and ROLE_TOK_EMB16_EXP exponents; model/mirror.py:777-783,
 * firmware embed_row_bfp).  A token outside [0, vocab) sets TRX_DEV_RANGE and writes zeros. */
trx_status trx_embed_lookup_bfp16(trx_ctx *ctx, const int16_t *d_mant, const int32_t *d_exp, uint32_t vocab,
                                  uint32_t dim, const int32_t *d_token, float *d_x, cudaStream_t stream);

/* y = (x * r) * w with r = 1/sqrt(ss/n + eps), ss the canonical 64-partial sum of squares
 * (model/mirror.py:576-591, :697-700 rmsnorm).  One launch; y may not alias x. */
trx_status trx_rmsnorm(trx_ctx *ctx, const float *d_x, const float *d_w, uint32_t n, float eps, float *d_y,
                       cudaStream_t stream);

/*
 * Float projection of a K-segmented tensor (FLAG_KSEG: a matvec wider than one engine op stored as
 * nseg tensors over consecutive column ranges, model/bons.py:83-113 split_wide), in the engine's
 * arithmetic (model/mirror.py:664-678, firmware/infer_float.c:183-186): x quantised once (one
 * exponent for the whole input), each segment's int32 engine result (>> R per segment), their
 * int64 sum wrapped to int32, times 2^(e8 + R - B), plus d_resid when not NULL.  segs: the
 * segments' entries in order (same rows, the tensor's B and R in every one; ternary kinds or
 * TRX_KIND_Q8); d_packed: a host array of their device pointers.  x: the sum of the segments' cols
 * floats (at most 32768).  Uses the context's scratch: calls on one context must not overlap.
 */
trx_status trx_matvec_f_kseg(trx_ctx *ctx, const trx_entry *segs, int nseg, const void *const *d_packed,
                             const float *d_x, const float *d_resid, float *d_y, cudaStream_t stream);

/* *d_pos += n on the device (the decode loop's position, read by the attention and DeltaNet steps). */
trx_status trx_advance_position(trx_ctx *ctx, int32_t *d_pos, int32_t n, cudaStream_t stream);

/*
 * LM head + greedy token (model/mirror.py:1027-1034; doc/units.md:148-149): the float projection of
 * trx_matvec_f (with the final RMSNorm fused when d_norm_w is set), and the index of its largest
 * value, ties to the smallest row, written to *d_token (one int32 on the device) by the same
 * launch.  d_logits may be NULL (the logits are then not stored).
 */
trx_status trx_lmhead_argmax(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                             const float *d_norm_w, float eps, float *d_logits, int32_t *d_token,
                             cudaStream_t stream);

/*
 * One shard of a row-sharded LM head (tensor parallelism): as trx_lmhead_argmax, but writes the
 * shard's argmax key to *d_key (one uint64 on the device: the orderable float bits of the largest
 * logit in the high word, ~(row + row_offset) in the low word, so the largest key over all shards
 * is the global greedy token with ties to the smallest row).  row_offset: the shard's first row.
 */
trx_status trx_lmhead_argmax_key(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                                 const float *d_norm_w, float eps, uint32_t row_offset, float *d_logits,
                                 uint64_t *d_key, cudaStream_t stream);

/* *d_token = the row of the largest of the n keys at d_keys (gathered shard keys). */
trx_status trx_argmax_token(trx_ctx *ctx, const uint64_t *d_keys, int32_t n, int32_t *d_token, cudaStream_t stream);

/* Shape of one attention layer (model/configs.py head counts; mirror.py:945-996). */
typedef struct trx_attn_shape {
    uint32_t n_head;     /* query heads H                                              */
    uint32_t n_kv;       /* kv heads (H % n_kv == 0; query head h reads kv head h/(H/n_kv)) */
    uint32_t head_dim;   /* hd, a multiple of 8, <= 512                                 */
    uint32_t rope_dims;  /* rotated dims per head (even, <= hd; neox pairs inside them)  */
    uint32_t max_pos;    /* cache capacity in positions                                 */
    int32_t  gated;      /* q holds [q | gate] per head (2*hd floats): out *= sigmoid(gate) */
    float    eps;        /* epsilon of the q/k RMSNorms                                 */
} trx_attn_shape;

/*
 * One decode step of GQA attention over an fp16 KV cache (model/mirror.py:945-996,
 * model/golden.py:361-398), in one launch:
 *   q[h] = RoPE(RMSNorm(q[h]) * qnorm_w), k = RoPE(RMSNorm(k) * knorm_w) (neox pairs over the
 *   first rope_dims, angle fp32(pos * rope_freq[i])); k and v (rounded to fp16) are written to
 *   the caches at position *d_pos; out[h] = softmax(q[h].K^T / sqrt(hd)) V over positions
 *   0..pos, times sigmoid(gate[h]) when gated.
 * d_q: H * (gated ? 2 : 1) * hd floats; d_k, d_v: n_kv * hd; d_qnorm_w, d_knorm_w: hd;
 * d_rope_freq: rope_dims/2 floats; caches: [max_pos][n_kv][hd] fp16 (16-byte aligned);
 * d_pos: one int32 on the device (read by the kernel, so a captured graph replays every step);
 * d_out: H * hd floats.  A position outside [0, max_pos) sets TRX_DEV_RANGE and does nothing.
 * Launches on the context's scratch: calls on one context must not overlap.
 */
trx_status trx_attn_decode(trx_ctx *ctx, const trx_attn_shape *shape, const float *d_q, const float *d_k,
                           const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                           const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                           float *d_out, cudaStream_t stream);

/*
 * trx_attn_decode for a batch of nseq independent sequences in one launch: q [nseq][H*(1+gated)*hd],
 * k/v [nseq][n_kv*hd], caches [nseq][max_pos][n_kv][hd] fp16, d_pos [nseq] (each sequence's own
 * position), out [nseq][H*hd]; the scratch-merge kernel with a sequence grid dimension.
 */
trx_status trx_attn_decode_rows(trx_ctx *ctx, const trx_attn_shape *shape, int32_t nseq, const float *d_q,
                                const float *d_k, const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                                const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                                float *d_out, cudaStream_t stream);

/*
 * trx_attn_decode over an fp32 KV cache (caches [max_pos][n_kv][head_dim] float, 16-byte aligned):
 * the reference mirror keeps its cache in fp32 (model/mirror.py:966, kc[l].append(k)), so a run
 * that must follow the mirror's values to fp32 rounding (token parity in the engine's int8
 * arithmetic, where an fp16-rounded cache moves activations across int8 rounding boundaries)
 * takes this form.  Same arguments and computation otherwise; one launch of the scratch-merge
 * kernel on the context's scratch (calls on one context must not overlap).
 */
trx_status trx_attn_decode_f32cache(trx_ctx *ctx, const trx_attn_shape *shape, const float *d_q, const float *d_k,
                                    const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                                    const float *d_rope_freq, float *d_kcache, float *d_vcache,
                                    const int32_t *d_pos, float *d_out, cudaStream_t stream);

/*
 * trx_attn_decode without a context, for callers that cannot allocate device memory while they
 * run (a serving loop that reserved the device's memory up front, a host runtime whose allocator
 * belongs to another framework).  No counterpart in the reference.  Same computation and
 * arguments as trx_attn_decode; the partials and arrival counts live in the library's static
 * device arrays (limits: n_kv <= 64 and n_kv * splits * (H/n_kv) * (head_dim + 2) floats <= 2^20,
 * splits = ceil(max_pos / chunk) with chunk the smallest of 64, 128, 256 (128 when head_dim >
 * 128) giving at most 16 splits; larger shapes return TRX_ERR_UNSUPPORTED), so the library
 * allocates nothing.  Device error bits are OR'd into *d_err (a caller-owned device word).  The
 * arrays are zero when the library's module loads on a device and every launch leaves the arrival
 * counts at zero again; each call looks the arrays' device addresses up on the host (no device
 * work, no allocation).  Calls that overlap on the GPU race on the arrays.
 */
trx_status trx_attn_decode_static(const trx_attn_shape *shape, const float *d_q, const float *d_k,
                                  const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                                  const float *d_rope_freq, void *d_kcache, void *d_vcache,
                                  const int32_t *d_pos, float *d_out, uint32_t *d_err, cudaStream_t stream);

/* Shape of one gated-DeltaNet layer (model/configs.py dn_* fields). */
typedef struct trx_deltanet_shape {
    uint32_t n_k_heads;    /* nk                                                    */
    uint32_t k_head_dim;   /* hk: 32, 64, 128 or 256                                 */
    uint32_t n_v_heads;    /* nv, a multiple of nk (value head h uses key head h % nk) */
    uint32_t v_head_dim;   /* hv <= 1024                                             */
    uint32_t conv_kernel;  /* K taps of the causal conv, 2..8                        */
    float    eps;          /* epsilon of the L2 norms and the output RMSNorm         */
} trx_deltanet_shape;

/*
 * One decode step of a gated-DeltaNet layer after its projections (model/mirror.py:892-943,
 * mathematical profile), in one launch:
 *   causal conv over the last K inputs of each of the C = 2*nk*hk + nv*hv qkv channels, SiLU;
 *   q, k L2-normalised per key head; per value head h (key head h % nk):
 *   M *= exp(softplus(alpha+dt_bias)*a); delta = (v - M k)*sigmoid(beta); M += delta k^T;
 *   o = M q / sqrt(hk); out[grouped position of h] = RMSNorm(o)*norm_w*silu(z_h).
 * d_qkv: C floats; d_z: nv*hv; d_beta, d_alpha (pre-activation), d_dt_bias, d_ssm_a: nv;
 * d_conv_w: [C][K]; d_norm_w: hv; d_conv_ring: [K][C] floats, zero before the first step, slot
 * pos % K receives this step's qkv; d_state: [nv][hv][hk] fp32, updated in place; d_pos: one int32
 * on the device, the step's position (0 for the first token); d_out: nv*hv floats, value head h
 * at (h % nk)*(nv/nk) + h/nk (mirror.py:941-942).  Uses the context's scratch: calls on one
 * context must not overlap.
 */
trx_status trx_deltanet_step(trx_ctx *ctx, const trx_deltanet_shape *shape, const float *d_qkv, const float *d_z,
                             const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                             const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                             float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                             cudaStream_t stream);

/*
 * The integer gated-DeltaNet head step (model/deltanet.py:99-147, head_step; the vector unit's
 * bit-exact fast path): nheads independent heads, each an int16 state hv x hk (d_state
 * [nheads][hv][hk], value = m * 2^exp) at exponent d_exp[h] with d_maxabs[h] its max |m| as the
 * previous step left it (negative: computed from the state, the reference's maxM=None); fp32 key
 * and query d_k, d_q [nheads][hk], value d_v [nheads][hv], decay and beta d_decay, d_beta [nheads].
 * The state, exponent and max are updated in place; d_out [nheads][hv] receives o (fp32).  hv <= 256,
 * hk <= 128.  A value outside the reference's asserted ranges sets TRX_DEV_OVERFLOW.
 */
trx_status trx_deltanet_int_step(trx_ctx *ctx, uint32_t nheads, uint32_t hv, uint32_t hk, int16_t *d_state,
                                 int32_t *d_exp, int32_t *d_maxabs, const float *d_k, const float *d_q,
                                 const float *d_v, const float *d_decay, const float *d_beta, float *d_out,
                                 cudaStream_t stream);

/*
 * trx_deltanet_step for a batch of nseq independent sequences in one launch: every per-sequence
 * argument (qkv, z, beta, alpha, conv ring, state, position, output) is nseq consecutive copies of
 * the single-sequence layout; the weights (dt_bias, ssm_a, conv_w, norm_w) are shared.
 */
trx_status trx_deltanet_step_rows(trx_ctx *ctx, const trx_deltanet_shape *shape, int32_t nseq, const float *d_qkv,
                                  const float *d_z, const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                                  const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                                  float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                                  cudaStream_t stream);

/*
 * Tensor-parallel exchange over peer memory (no counterpart in the reference, which runs on one
 * device; the reference's multi-device plan shards output rows and all-gathers the hidden vector,
 * which these calls do without a collective library).  Every rank holds the same buffers at
 * addresses its peers can store to (peer-mapped device memory).  A producing launch stores each
 * result into dst[r] + offset for every rank r other than its own (its own result goes to the
 * launch's usual output) and, when every CTA is done, adds 1 to *signal[r] on every rank r
 * (its own included).  A consuming launch first waits, bounded, until its own counter *wait
 * holds (*step + 1) * world, the completions of this step's producers on every rank; on timeout
 * it records TRX_DEV_TIMEOUT and goes on.  *step is this rank's step counter (advanced once per
 * step, e.g. with trx_advance_position), *arrive a launch arrival count, zero between launches.
 * Every rank must run the same sequence of exchanging launches.  NULL dst entries get no copy;
 * signal[0] == NULL: the launch signals nothing; wait == NULL: it waits for nothing.
 */
#define TRX_TP_MAX 8
typedef struct trx_tp_xfer {
    uint32_t world, rank;            /* world <= TRX_TP_MAX, rank < world                  */
    void *dst[TRX_TP_MAX];           /* each rank's destination base (device addresses)   */
    uint32_t offset;                 /* elements: this rank's first element in dst[*]     */
    uint32_t *signal[TRX_TP_MAX];    /* each rank's counter of the completed gather point */
    const uint32_t *wait;            /* this rank's counter to wait on, or NULL           */
    const int32_t *step;             /* this rank's step counter                          */
    uint32_t *arrive;                /* arrival count of the signalling launch            */
    /* Tagged words (tag_points > 0).  Each element of an exchanged vector is one 64-bit word, the
     * value's bits | tag << 32, written by one single-copy-atomic store; the tag of gather point p
     * at step s is s * tag_points + p + 1.  tag_out >= 0: the output goes to dst[r] of EVERY rank
     * (this rank's included) as tagged words, and signal/arrive are not used.  tag_in >= 0: d_x
     * points to tagged words, and the kernel reads each one once it carries point tag_in's tag
     * of this step (bounded wait, TRX_DEV_TIMEOUT); wait is not used.  All zero: counters only. */
    uint32_t tag_points;
    int32_t tag_out;                 /* gather point of the output, or -1                */
    int32_t tag_in;                  /* gather point of the tagged input, or -1          */
} trx_tp_xfer;

/* trx_matvec_f with an exchange: float results copied to dst (offset + row), input waited on. */
trx_status trx_matvec_f_tp(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                           const float *d_norm_w, float eps, const float *d_resid, float *d_y,
                           const trx_tp_xfer *tp, cudaStream_t stream);

/* trx_matvec_f_multi with an exchange (wait only: its outputs stay on this rank). */
trx_status trx_matvec_f_multi_tp(trx_ctx *ctx, const trx_entry *entries, int nseg, const void *d_packed,
                                 const float *d_x, const float *d_norm_w, float eps, float *const *d_y,
                                 const float *const *d_resid, const trx_tp_xfer *tp, cudaStream_t stream);

/* trx_matvec_swiglu with an exchange: silu(g)*u copied to dst (offset + row), input waited on. */
trx_status trx_matvec_swiglu_tp(trx_ctx *ctx, const trx_entry *gate, const void *d_gate, const trx_entry *up,
                                const void *d_up, const float *d_x, const float *d_norm_w, float eps,
                                float *d_act, const trx_tp_xfer *tp, cudaStream_t stream);

/* trx_lmhead_argmax_key with an exchange: the key copied to dst (offset, uint64), input waited on. */
trx_status trx_lmhead_argmax_key_tp(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                                    const float *d_norm_w, float eps, uint32_t row_offset, float *d_logits,
                                    uint64_t *d_key, const trx_tp_xfer *tp, cudaStream_t stream);

/* trx_deltanet_step with an exchange: the grouped output copied to dst (offset + index) of every rank
 * as tagged words (tag_points > 0 and tag_out >= 0 required). */
trx_status trx_deltanet_step_tp(trx_ctx *ctx, const trx_deltanet_shape *shape, const float *d_qkv, const float *d_z,
                                const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                                const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                                float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                                const trx_tp_xfer *tp, cudaStream_t stream);

/* trx_matvec_f_kseg with an exchange (tagged words only): the input read as tagged words when
 * tag_in >= 0, the float results copied to dst (offset + row) of every rank when tag_out >= 0. */
trx_status trx_matvec_f_kseg_tp(trx_ctx *ctx, const trx_entry *segs, int nseg, const void *const *d_packed,
                                const float *d_x, const float *d_resid, float *d_y, const trx_tp_xfer *tp,
                                cudaStream_t stream);

/* trx_matvec_f_kseg for a batch of nb <= 32 rows on the tensor cores (model/mirror.py:648-678 per row):
 * d_x [nb][K] with K the segments' total width, each row quantised with one exponent over all K,
 * d_y [nb][rows] (plus d_resid [nb][rows] when given).  Two ternary segments of one kind only
 * (TRX_ERR_UNSUPPORTED otherwise). */
trx_status trx_matvec_f_rows_kseg(trx_ctx *ctx, const trx_entry *segs, int nseg, const void *const *d_packed,
                                  const float *d_x, int nb, const float *d_resid, float *d_y, cudaStream_t stream);

/* trx_argmax_token after waiting for the exchange of the keys. */
trx_status trx_argmax_token_tp(trx_ctx *ctx, const uint64_t *d_keys, int32_t n, int32_t *d_token,
                               const trx_tp_xfer *tp, cudaStream_t stream);

/* trx_attn_decode with an exchange: out[h][d] copied to dst (offset + h*hd + d).  Tagged words: any
 * shape.  Plain words with completion counters: head dims 64 and 128 with at most 8 query heads per
 * kv head only (TRX_ERR_UNSUPPORTED otherwise). */
trx_status trx_attn_decode_tp(trx_ctx *ctx, const trx_attn_shape *shape, const float *d_q, const float *d_k,
                              const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                              const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                              float *d_out, const trx_tp_xfer *tp, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TRIXIUM_B200_H */
