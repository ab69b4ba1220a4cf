// C ABI of libtrixium_b200.so (declarations and contracts in include/trixium_b200.h).
#include <cstdint>
#include <cstdlib>
#include <new>
#include <cuda_runtime.h>

#include "../../include/trixium_b200.h"
#include "trx_internal.h"

struct trx_ctx {
    int device;
    uint32_t *err;    // device error word
    uint32_t *lut;    // replicated trit5 byte LUT (64 KiB), copied into each CTA's shared memory
    // Decode-attention partials and per-kv-head arrival counts (zero between launches).
    float *attn_part;
    unsigned *attn_cnt;
    // Greedy-argmax keys (one per job) and the matvec's arrival count (zero between launches).
    unsigned long long *amax_key;
    unsigned *amax_cnt;
    // The quantised activation of trx_matvec_q8_f and trx_matvec_f_kseg: 32 KiB of x8, then its
    // exponent e8.
    int8_t *q8x;
    // trx_matvec_f_kseg: the segments' int32 engine results, [nseg][rows].
    int32_t *kseg_part;
    // Batched rows on the tensor cores: the permuted activation rows, their group sums and
    // exponents; the K-split partial sums and per-row arrival counts (zero between launches).
    int8_t *rows_x8p;
    int *rows_xsum;
    int *rows_e8;
    unsigned long long *rows_acc;
    unsigned *rows_cnt;
};

static const uint64_t kAttnPartFloats = 1ull << 24;  // 64 MiB of attention partials (batches of sequences)
static const uint32_t kAttnMaxKv = 4096;  // arrival counts: kv heads (or value heads) x sequences
static const int kMaxArgmaxJobs = 64;
static const uint32_t kQ8MaxCols = 32768;
static const uint64_t kKsegPartInts = 1ull << 20;  // 4 MiB of K-segment partial results
static const int kRowsMax = 32;                      // batch rows of the tensor-core path
static const uint64_t kRowsAcc = 1ull << 19;          // int64 partial sums (4 MiB): nb * N of a K-split launch
static const int kRowsCnt = 1 << 19;                  // per-row arrival counts of a K-split launch (2 MiB)

namespace trx {
bool pdl_enabled() { return true; }
}  // namespace trx

namespace {

bool ternary_kind(int k) { return k == TRX_KIND_TERNARY || k == TRX_KIND_TERNARY5; }

trx_status check_entry(const trx_entry *e) {
    if (!e) return TRX_ERR_ARG;
    if (!ternary_kind(e->kind)) return TRX_ERR_LAYOUT;
    if (e->rows == 0 || e->cols == 0 || (e->cols % 128) != 0) return TRX_ERR_LAYOUT;
    if (e->cols > 32768u || e->rows > (1u << 30)) return TRX_ERR_UNSUPPORTED;
    if (e->rshift < 0 || e->rshift > 47 || e->bias < -64 || e->bias > 64) return TRX_ERR_ARG;
    return TRX_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

trx::MvJobs base_jobs(const trx_ctx *ctx, const trx_entry *e, const void *packed) {
    trx::MvJobs J{};
    J.w = static_cast<const uint8_t *>(packed);
    J.rows = (int)e->rows;
    J.cols = (int)e->cols;
    J.kind = e->kind;
    J.nseg = 1;
    J.seg[0].row_end = (int)e->rows;
    J.seg[0].B = e->bias;
    J.seg[0].R = e->rshift;
    J.njobs = 1;
    return J;
}

}  // namespace

extern "C" {

trx_status trx_create(trx_ctx **ctx, int device) {
    if (!ctx) return TRX_ERR_ARG;
    *ctx = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) return TRX_ERR_CUDA;
    trx_ctx *c = new (std::nothrow) trx_ctx{};
    if (!c) return TRX_ERR_ARG;
    c->device = device;
    if (cudaMalloc(&c->err, 256) != cudaSuccess) {
        delete c;
        return TRX_ERR_CUDA;
    }
    if (cudaMalloc(&c->lut, trx::lut_bytes()) != cudaSuccess) {
        cudaFree(c->err);
        delete c;
        return TRX_ERR_CUDA;
    }
    if (cudaMemset(c->err, 0, 256) != cudaSuccess ||
        cudaMalloc(&c->attn_part, kAttnPartFloats * 4) != cudaSuccess ||
        cudaMalloc(&c->attn_cnt, kAttnMaxKv * 4) != cudaSuccess || cudaMemset(c->attn_cnt, 0, kAttnMaxKv * 4) != cudaSuccess ||
        cudaMalloc(&c->amax_key, kMaxArgmaxJobs * 8) != cudaSuccess ||
        cudaMemset(c->amax_key, 0, kMaxArgmaxJobs * 8) != cudaSuccess ||
        cudaMalloc(&c->amax_cnt, 16) != cudaSuccess || cudaMemset(c->amax_cnt, 0, 16) != cudaSuccess ||
        cudaMalloc(&c->q8x, kQ8MaxCols + 16) != cudaSuccess ||
        cudaMalloc(&c->kseg_part, kKsegPartInts * 4) != cudaSuccess ||
        cudaMalloc(&c->rows_x8p, (size_t)kRowsMax * kQ8MaxCols) != cudaSuccess ||
        cudaMalloc(&c->rows_xsum, (size_t)32 * (kQ8MaxCols / 128) * 4) != cudaSuccess ||
        cudaMalloc(&c->rows_e8, kRowsMax * 4) != cudaSuccess ||
        cudaMalloc(&c->rows_acc, kRowsAcc * 8) != cudaSuccess ||
        cudaMemset(c->rows_acc, 0, kRowsAcc * 8) != cudaSuccess ||
        cudaMalloc(&c->rows_cnt, kRowsCnt * 4) != cudaSuccess ||
        cudaMemset(c->rows_cnt, 0, kRowsCnt * 4) != cudaSuccess ||
        trx::launch_build_lut(c->lut, 0) != TRX_OK ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(c->err);
        cudaFree(c->lut);
        cudaFree(c->attn_part);
        cudaFree(c->attn_cnt);
        cudaFree(c->amax_key);
        cudaFree(c->amax_cnt);
        cudaFree(c->q8x);
        cudaFree(c->kseg_part);
        cudaFree(c->rows_x8p);
        cudaFree(c->rows_xsum);
        cudaFree(c->rows_e8);
        cudaFree(c->rows_acc);
        cudaFree(c->rows_cnt);
        delete c;
        return TRX_ERR_CUDA;
    }
    *ctx = c;
    return TRX_OK;
}

trx_status trx_destroy(trx_ctx *ctx) {
    if (!ctx) return TRX_ERR_ARG;
    cudaFree(ctx->err);
    cudaFree(ctx->lut);
    cudaFree(ctx->attn_part);
    cudaFree(ctx->attn_cnt);
    cudaFree(ctx->amax_key);
    cudaFree(ctx->amax_cnt);
    cudaFree(ctx->q8x);
    cudaFree(ctx->kseg_part);
    cudaFree(ctx->rows_x8p);
    cudaFree(ctx->rows_xsum);
    cudaFree(ctx->rows_e8);
    cudaFree(ctx->rows_acc);
    cudaFree(ctx->rows_cnt);
    delete ctx;
    return TRX_OK;
}

trx_status trx_get_error(trx_ctx *ctx, cudaStream_t stream, uint32_t *bits) {
    if (!ctx || !bits) return TRX_ERR_ARG;
    uint32_t v = 0;
    if (cudaMemcpyAsync(&v, ctx->err, 4, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return TRX_ERR_CUDA;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return TRX_ERR_CUDA;
    *bits = v;
    if (v && cudaMemsetAsync(ctx->err, 0, 4, stream) != cudaSuccess) return TRX_ERR_CUDA;
    return TRX_OK;
}

const char *trx_last_cuda_error(void) { return trx::last_cuda_error(); }

uint64_t trx_row_bytes(uint32_t cols, int32_t kind) {
    if (kind == TRX_KIND_Q8) {
        if (cols == 0 || cols % 32) return 0;
        const uint64_t G = cols / 32;
        return (G + 15) / 16 * 32 + 32 * G;
    }
    if (!ternary_kind(kind) || cols == 0 || cols % 128) return 0;
    const uint64_t G = cols / 128;
    const uint64_t sb = (G + 15) / 16 * 32;
    const uint64_t cb = kind == TRX_KIND_TERNARY5 ? 26 * G : 32 * G;
    return sb + (cb + 31) / 32 * 32;
}

trx_status trx_matvec_i8(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const int8_t *d_x8,
                         int32_t *d_out, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x8 || !d_out || !aligned16(d_packed)) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x8 = d_x8;
    J.seg[0].y = d_out;
    J.out = trx::OUT_I32;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

static trx_status check_q8(const trx_ctx *ctx, const trx_entry *e, const void *packed) {
    if (!ctx || !e) return TRX_ERR_ARG;
    if (e->kind != TRX_KIND_Q8 || e->rows == 0 || e->cols == 0 || (e->cols % 32) != 0) return TRX_ERR_LAYOUT;
    if (e->cols > kQ8MaxCols || e->rows > (1u << 30)) return TRX_ERR_UNSUPPORTED;
    if (e->rshift < 0 || e->rshift > 47 || e->bias < -64 || e->bias > 64) return TRX_ERR_ARG;
    if (!packed || !aligned16(packed)) return TRX_ERR_ARG;
    return TRX_OK;
}

trx_status trx_matvec_q8(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const int8_t *d_x8, int32_t *d_out,
                         cudaStream_t stream) {
    trx_status s = check_q8(ctx, e, d_packed);
    if (s) return s;
    if (!d_x8 || !d_out) return TRX_ERR_ARG;
    return trx::launch_matvec_q8(static_cast<const uint8_t *>(d_packed), (int)e->rows, (int)e->cols, e->bias,
                                 e->rshift, d_x8, nullptr, d_out, ctx->err, stream);
}

trx_status trx_matvec_q8_f(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x, float *d_y,
                           cudaStream_t stream) {
    trx_status s = check_q8(ctx, e, d_packed);
    if (s) return s;
    if (!d_x || !d_y) return TRX_ERR_ARG;
    int *e8 = reinterpret_cast<int *>(ctx->q8x + kQ8MaxCols);
    s = trx::launch_quantize(d_x, (int)e->cols, ctx->q8x, e8, stream);
    if (s) return s;
    return trx::launch_matvec_q8(static_cast<const uint8_t *>(d_packed), (int)e->rows, (int)e->cols, e->bias,
                                 e->rshift, ctx->q8x, e8, d_y, ctx->err, stream);
}

static trx_status rows_tc(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x, const int8_t *d_x8,
                          int nb, int32_t *d_out_i, float *d_out_f, const float *d_resid, cudaStream_t stream) {
    trx::RowsSeg sg{(int)e->rows, e->bias, e->rshift, d_out_i, d_out_f, d_resid};
    return trx::launch_matvec_rows(static_cast<const uint8_t *>(d_packed), (int)e->cols, e->kind, &sg, 1, d_x, d_x8, nb,
                                   nullptr, 0.f, ctx->rows_x8p, ctx->rows_xsum, ctx->rows_e8, ctx->rows_acc, kRowsAcc,
                                   ctx->rows_cnt, kRowsCnt, ctx->err, trx::device_sms(), trx::device_reserved_smem(),
                                   stream);
}

trx_status trx_matvec_f_rows_kseg(trx_ctx *ctx, const trx_entry *segs, int nseg, const void *const *d_packed,
                                  const float *d_x, int nb, const float *d_resid, float *d_y, cudaStream_t stream) {
    if (!ctx || !segs || !d_packed || !d_x || !d_y || nb < 1 || nb > kRowsMax) return TRX_ERR_ARG;
    if (nseg != 2) return TRX_ERR_UNSUPPORTED;  // two ternary segments (every split of K <= 32768)
    const uint32_t rows = segs[0].rows;
    uint32_t K = 0;
    for (int i = 0; i < nseg; ++i) {
        if (trx_status s = check_entry(segs + i)) return s;
        if (!d_packed[i] || !aligned16(d_packed[i])) return TRX_ERR_ARG;
        if (segs[i].rows != rows || segs[i].bias != segs[0].bias || segs[i].rshift != segs[0].rshift ||
            segs[i].kind != segs[0].kind)
            return TRX_ERR_ARG;
        K += segs[i].cols;
    }
    if (K > kQ8MaxCols) return TRX_ERR_UNSUPPORTED;
    if ((uint64_t)nb * rows > kKsegPartInts) return TRX_ERR_UNSUPPORTED;
    // Segment 0: the prep over all K columns (one exponent per row), its int32 results; segment 1:
    // the same prepped activation from column cols0 on, plus segment 0's results, then the scaling.
    trx::RowsSeg s0{(int)rows, segs[0].bias, segs[0].rshift, ctx->kseg_part, nullptr, nullptr, nullptr};
    trx::RowsSeg s1{(int)rows, segs[1].bias, segs[1].rshift, nullptr, d_y, d_resid, ctx->kseg_part};
    const int sms = trx::device_sms(), res = trx::device_reserved_smem();
    trx_status s = trx::launch_matvec_rows(static_cast<const uint8_t *>(d_packed[0]), (int)segs[0].cols, segs[0].kind,
                                           &s0, 1, d_x, nullptr, nb, nullptr, 0.f, ctx->rows_x8p, ctx->rows_xsum,
                                           ctx->rows_e8, ctx->rows_acc, kRowsAcc, ctx->rows_cnt, kRowsCnt, ctx->err, sms,
                                           res, stream, (int)K, 0, true);
    if (s) return s;
    return trx::launch_matvec_rows(static_cast<const uint8_t *>(d_packed[1]), (int)segs[1].cols, segs[1].kind, &s1, 1,
                                   d_x, nullptr, nb, nullptr, 0.f, ctx->rows_x8p, ctx->rows_xsum, ctx->rows_e8,
                                   ctx->rows_acc, kRowsAcc, ctx->rows_cnt, kRowsCnt, ctx->err, sms, res, stream, (int)K,
                                   (int)segs[0].cols, false);
}

trx_status trx_matvec_f_rows(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x, int nb,
                             const float *d_resid, float *d_y, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_y || nb < 1 || nb > kRowsMax || !aligned16(d_packed)) return TRX_ERR_ARG;
    return rows_tc(ctx, e, d_packed, d_x, nullptr, nb, nullptr, d_y, d_resid, stream);
}

trx_status trx_matvec_f_rows_multi(trx_ctx *ctx, const trx_entry *entries, int nseg, const void *d_packed,
                                   const float *d_x, int nb, const float *d_norm_w, float eps, float *const *d_y,
                                   const float *const *d_resid, cudaStream_t stream) {
    if (!ctx || !entries || !d_y || nseg < 1 || nseg > trx::kRowsMaxSegs) return TRX_ERR_ARG;
    if (!d_packed || !d_x || nb < 1 || nb > kRowsMax || !aligned16(d_packed) || !(eps >= 0.f)) return TRX_ERR_ARG;
    trx::RowsSeg sg[trx::kRowsMaxSegs];
    for (int i = 0; i < nseg; ++i) {
        if (trx_status s = check_entry(entries + i)) return s;
        if (entries[i].cols != entries[0].cols || entries[i].kind != entries[0].kind || !d_y[i]) return TRX_ERR_ARG;
        sg[i] = trx::RowsSeg{(int)entries[i].rows, entries[i].bias, entries[i].rshift, nullptr, d_y[i],
                             d_resid ? d_resid[i] : nullptr};
    }
    return trx::launch_matvec_rows(static_cast<const uint8_t *>(d_packed), (int)entries[0].cols, entries[0].kind, sg,
                                   nseg, d_x, nullptr, nb, d_norm_w, eps, ctx->rows_x8p, ctx->rows_xsum, ctx->rows_e8,
                                   ctx->rows_acc, kRowsAcc, ctx->rows_cnt, kRowsCnt, ctx->err, trx::device_sms(),
                                   trx::device_reserved_smem(), stream);
}

trx_status trx_embed_lookup_rows(trx_ctx *ctx, const void *d_table, uint32_t vocab, uint32_t dim, int32_t f16,
                                 const int32_t *d_tokens, int32_t nrows, float *d_x, cudaStream_t stream) {
    if (!ctx || !d_table || !d_tokens || !d_x || vocab == 0 || dim == 0 || nrows < 1 || nrows > 65535)
        return TRX_ERR_ARG;
    return trx::launch_embed_rows(d_table, (int)vocab, (int)dim, f16 ? 1 : 0, d_tokens, nrows, d_x, ctx->err, stream);
}

trx_status trx_rmsnorm_rows(trx_ctx *ctx, const float *d_x, const float *d_w, uint32_t n, int32_t nrows, float eps,
                            float *d_y, cudaStream_t stream) {
    if (!ctx || !d_x || !d_w || !d_y || n == 0 || n > (1u << 24) || nrows < 1 || !(eps >= 0.f)) return TRX_ERR_ARG;
    return trx::launch_rmsnorm_rows(d_x, d_w, (int)n, nrows, eps, d_y, stream);
}

trx_status trx_silu_mul(trx_ctx *ctx, const float *d_g, const float *d_u, uint64_t n, float *d_act,
                        cudaStream_t stream) {
    if (!ctx || !d_g || !d_u || !d_act || n == 0) return TRX_ERR_ARG;
    return trx::launch_silu_mul(d_g, d_u, (long long)n, d_act, stream);
}

trx_status trx_argmax_rows(trx_ctx *ctx, const float *d_logits, uint32_t V, int32_t nrows, int32_t *d_tokens,
                           cudaStream_t stream) {
    if (!ctx || !d_logits || !d_tokens || V == 0 || nrows < 1) return TRX_ERR_ARG;
    return trx::launch_argmax_rows(d_logits, (int)V, nrows, d_tokens, stream);
}

trx_status trx_advance_positions(trx_ctx *ctx, int32_t *d_pos, int32_t count, int32_t n, cudaStream_t stream) {
    if (!ctx || !d_pos || count < 1) return TRX_ERR_ARG;
    return trx::launch_advance_rows(d_pos, count, n, stream);
}

trx_status trx_matvec_i8_rows(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const int8_t *d_x8, int nb,
                              int32_t *d_out, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x8 || !d_out || nb < 1 || nb > kRowsMax || !aligned16(d_packed)) return TRX_ERR_ARG;
    if (nb > 8) return rows_tc(ctx, e, d_packed, nullptr, d_x8, nb, d_out, nullptr, nullptr, stream);
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x8 = d_x8;
    J.x_stride = e->cols;
    J.seg[0].y = d_out;
    J.y_stride = e->rows;
    J.w_stride = 0;  // every row of x8 streams the same tensor
    J.njobs = nb;
    J.out = trx::OUT_I32;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_quantize_pow2(trx_ctx *ctx, const float *d_x, uint32_t n, int8_t *d_x8, int32_t *d_e8,
                             cudaStream_t stream) {
    if (!ctx || !d_x || !d_x8 || !d_e8 || n == 0 || n > (1u << 28)) return TRX_ERR_ARG;
    return trx::launch_quantize(d_x, (int)n, d_x8, d_e8, stream);
}

// A C-ABI tensor-parallel exchange as the kernels' TpXfer (all zero when t is NULL).  what: which
// parts apply to the call (copies to dst, a completion signal, a wait before the input is read).
enum { TP_PUSH = 1, TP_SIGNAL = 2, TP_WAIT = 4 };
static trx_status tp_resolve(const trx_tp_xfer *t, int what, trx::TpXfer &X) {
    X = trx::TpXfer{};
    if (!t) return TRX_OK;
    if (t->world < 1 || t->world > TRX_TP_MAX || t->rank >= t->world) return TRX_ERR_ARG;
    X.world = (int)t->world;
    X.rank = (int)t->rank;
    X.offset = (int)t->offset;
    if (what & TP_PUSH)
        for (uint32_t r = 0; r < t->world; ++r) X.dst[r] = t->dst[r];
    if ((what & TP_SIGNAL) && t->signal[0]) {
        for (uint32_t r = 0; r < t->world; ++r) {
            if (!t->signal[r]) return TRX_ERR_ARG;
            X.signal[r] = t->signal[r];
        }
        if (!t->arrive) return TRX_ERR_ARG;
        X.arrive = t->arrive;
    }
    if ((what & TP_WAIT) && t->wait) {
        if (!t->step) return TRX_ERR_ARG;
        X.wait = t->wait;
        X.step = t->step;
    }
    if (t->tag_points) {  // tagged words: every rank's dst for the output, the input polled
        if (!t->step || t->tag_out >= (int32_t)t->tag_points || t->tag_in >= (int32_t)t->tag_points) return TRX_ERR_ARG;
        X.tag_points = t->tag_points;
        X.step = t->step;
        X.tag_out = (what & TP_PUSH) ? t->tag_out : -1;
        X.tag_in = (what & TP_WAIT) ? t->tag_in : -1;
        if (X.tag_out >= 0) {
            for (uint32_t r = 0; r < t->world; ++r) {
                if (!t->dst[r] || (reinterpret_cast<uintptr_t>(t->dst[r]) & 7)) return TRX_ERR_ARG;
                X.dst[r] = t->dst[r];
            }
            for (int r = 0; r < trx::kTpMax; ++r) X.signal[r] = nullptr;  // no counters for a tagged output
            X.arrive = nullptr;
        }
        if (X.tag_in >= 0) X.wait = nullptr;
    } else {
        X.tag_out = X.tag_in = -1;
    }
    return TRX_OK;
}

trx_status trx_matvec_f(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                        const float *d_norm_w, float eps, const float *d_resid, float *d_y, cudaStream_t stream) {
    return trx_matvec_f_tp(ctx, e, d_packed, d_x, d_norm_w, eps, d_resid, d_y, nullptr, stream);
}

trx_status trx_matvec_f_tp(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                           const float *d_norm_w, float eps, const float *d_resid, float *d_y,
                           const trx_tp_xfer *tp, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_y || !aligned16(d_packed)) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    if ((s = tp_resolve(tp, TP_PUSH | TP_SIGNAL | TP_WAIT, J.tp))) return s;
    J.x = d_x;
    J.norm_w = d_norm_w;
    J.eps = eps;
    J.seg[0].resid = d_resid;
    J.seg[0].y = d_y;
    J.out = trx::OUT_F32;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_matvec_fp(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x, float *d_y,
                         cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_y) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x = d_x;
    J.seg[0].y = d_y;
    J.out = trx::OUT_F32;
    return trx::launch_matvec_fp(J, ctx->err, stream);
}

trx_status trx_matvec_fp_rows(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x, int32_t nrows,
                              const float *d_resid, float *d_y, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_y || nrows < 1 || nrows > (1 << 20)) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x = d_x;
    J.njobs = nrows;
    J.x_stride = e->cols;
    J.y_stride = e->rows;
    J.seg[0].y = d_y;
    J.seg[0].resid = d_resid;
    J.out = trx::OUT_F32;
    return trx::launch_matvec_fp(J, ctx->err, stream);
}

trx_status trx_matvec_swiglu(trx_ctx *ctx, const trx_entry *gate, const void *d_gate, const trx_entry *up,
                             const void *d_up, const float *d_x, const float *d_norm_w, float eps, float *d_act,
                             cudaStream_t stream) {
    return trx_matvec_swiglu_tp(ctx, gate, d_gate, up, d_up, d_x, d_norm_w, eps, d_act, nullptr, stream);
}

trx_status trx_matvec_swiglu_tp(trx_ctx *ctx, const trx_entry *gate, const void *d_gate, const trx_entry *up,
                                const void *d_up, const float *d_x, const float *d_norm_w, float eps,
                                float *d_act, const trx_tp_xfer *tp, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(gate);
    if (s) return s;
    s = check_entry(up);
    if (s) return s;
    if (gate->rows != up->rows || gate->cols != up->cols || gate->kind != up->kind) return TRX_ERR_ARG;
    if (!d_gate || !d_up || !d_x || !d_act || !aligned16(d_gate) || !aligned16(d_up)) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, gate, d_gate);
    if ((s = tp_resolve(tp, TP_PUSH | TP_SIGNAL | TP_WAIT, J.tp))) return s;
    J.w2 = static_cast<const uint8_t *>(d_up);
    J.B2 = up->bias;
    J.R2 = up->rshift;
    J.x = d_x;
    J.norm_w = d_norm_w;
    J.eps = eps;
    J.seg[0].y = d_act;
    J.out = trx::OUT_SWIGLU;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_validate_packed(trx_ctx *ctx, const trx_entry *e, const void *d_packed, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed) return TRX_ERR_ARG;
    if (e->kind != TRX_KIND_TERNARY5) return TRX_OK;  // every 2-bit byte decodes
    return trx::launch_validate_t5(static_cast<const uint8_t *>(d_packed), (int)e->rows, (int)e->cols, ctx->err,
                                   stream);
}

trx_status trx_matvec_f_batch(trx_ctx *ctx, const trx_entry *e, const void *d_packed, uint64_t w_stride,
                              const float *d_x, uint64_t x_stride, float *d_y, uint64_t y_stride, int njobs,
                              cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_y || njobs < 1 || !aligned16(d_packed) || (w_stride % 16) != 0)
        return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x = d_x;
    J.seg[0].y = d_y;
    J.w_stride = w_stride;
    J.x_stride = x_stride;
    J.y_stride = y_stride;
    J.njobs = njobs;
    J.out = trx::OUT_F32;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_matvec_f_multi(trx_ctx *ctx, const trx_entry *entries, int nseg, const void *d_packed,
                              const float *d_x, const float *d_norm_w, float eps, float *const *d_y,
                              const float *const *d_resid, cudaStream_t stream) {
    return trx_matvec_f_multi_tp(ctx, entries, nseg, d_packed, d_x, d_norm_w, eps, d_y, d_resid, nullptr, stream);
}

trx_status trx_matvec_f_multi_tp(trx_ctx *ctx, const trx_entry *entries, int nseg, const void *d_packed,
                                 const float *d_x, const float *d_norm_w, float eps, float *const *d_y,
                                 const float *const *d_resid, const trx_tp_xfer *tp, cudaStream_t stream) {
    if (!ctx || !entries || nseg < 1 || nseg > trx::kMaxSegs || !d_y) return TRX_ERR_ARG;
    uint64_t rows = 0;
    for (int i = 0; i < nseg; ++i) {
        trx_status s = check_entry(&entries[i]);
        if (s) return s;
        if (entries[i].cols != entries[0].cols || entries[i].kind != entries[0].kind || !d_y[i]) return TRX_ERR_ARG;
        rows += entries[i].rows;
    }
    if (rows > (1u << 30)) return TRX_ERR_UNSUPPORTED;
    if (!d_packed || !d_x || !aligned16(d_packed)) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, &entries[0], d_packed);
    if (trx_status st = tp_resolve(tp, TP_WAIT, J.tp)) return st;
    J.rows = (int)rows;
    J.nseg = nseg;
    int end = 0;
    for (int i = 0; i < nseg; ++i) {
        end += (int)entries[i].rows;
        J.seg[i].row_end = end;
        J.seg[i].B = entries[i].bias;
        J.seg[i].R = entries[i].rshift;
        J.seg[i].y = d_y[i];
        J.seg[i].resid = d_resid ? d_resid[i] : nullptr;
    }
    J.x = d_x;
    J.norm_w = d_norm_w;
    J.eps = eps;
    J.out = trx::OUT_F32;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_embed_lookup(trx_ctx *ctx, const void *d_table, uint32_t vocab, uint32_t dim, int32_t f16,
                            const int32_t *d_token, float *d_x, cudaStream_t stream) {
    if (!ctx || !d_table || !d_token || !d_x || vocab == 0 || dim == 0 || vocab > (1u << 30) || dim > (1u << 20))
        return TRX_ERR_ARG;
    return trx::launch_embed(d_table, (int)vocab, (int)dim, f16 ? 1 : 0, d_token, d_x, ctx->err, stream);
}

trx_status trx_embed_lookup_bfp16(trx_ctx *ctx, const int16_t *d_mant, const int32_t *d_exp, uint32_t vocab,
                                  uint32_t dim, const int32_t *d_token, float *d_x, cudaStream_t stream) {
    if (!ctx || !d_mant || !d_exp || !d_token || !d_x || vocab == 0 || dim == 0) return TRX_ERR_ARG;
    return trx::launch_embed_bfp16(d_mant, d_exp, (int)vocab, (int)dim, d_token, d_x, ctx->err, stream);
}

trx_status trx_rmsnorm(trx_ctx *ctx, const float *d_x, const float *d_w, uint32_t n, float eps, float *d_y,
                       cudaStream_t stream) {
    if (!ctx || !d_x || !d_w || !d_y || n == 0 || n > (1u << 24) || !(eps >= 0.f)) return TRX_ERR_ARG;
    return trx::launch_rmsnorm(d_x, d_w, (int)n, eps, d_y, stream);
}

trx_status trx_matvec_f_kseg(trx_ctx *ctx, const trx_entry *segs, int nseg, const void *const *d_packed,
                             const float *d_x, const float *d_resid, float *d_y, cudaStream_t stream) {
    return trx_matvec_f_kseg_tp(ctx, segs, nseg, d_packed, d_x, d_resid, d_y, nullptr, stream);
}

trx_status trx_matvec_f_kseg_tp(trx_ctx *ctx, const trx_entry *segs, int nseg, const void *const *d_packed,
                                const float *d_x, const float *d_resid, float *d_y, const trx_tp_xfer *tp,
                                cudaStream_t stream) {
    if (!ctx || !segs || !d_packed || !d_x || !d_y || nseg < 1 || nseg > 64) return TRX_ERR_ARG;
    trx::TpXfer X;
    if (trx_status s = tp_resolve(tp, TP_PUSH | TP_WAIT, X)) return s;
    if (X.world && (X.signal[0] || X.wait)) return TRX_ERR_UNSUPPORTED;  // tagged words only
    const bool tagged_in = X.tag_points && X.tag_in >= 0;
    const uint32_t rows = segs[0].rows;
    uint64_t K = 0;
    for (int i = 0; i < nseg; ++i) {
        const trx_entry *e = segs + i;
        const trx_status s = e->kind == TRX_KIND_Q8 ? check_q8(ctx, e, d_packed[i]) : check_entry(e);
        if (s) return s;
        if (!d_packed[i] || !aligned16(d_packed[i])) return TRX_ERR_ARG;
        if (e->rows != rows || e->bias != segs[0].bias || e->rshift != segs[0].rshift) return TRX_ERR_ARG;
        K += e->cols;
    }
    if (K > kQ8MaxCols) return TRX_ERR_UNSUPPORTED;
    if ((uint64_t)nseg * rows > kKsegPartInts) return TRX_ERR_UNSUPPORTED;
    // Two ternary segments (every ternary split of K <= 32768): two launches.  Each takes the
    // exponent of the whole input in its prologue and builds the activation words of its own
    // columns; the first writes its int32 results, the second adds them to its own before the
    // float scaling (the mirror's sum of the segments' results), then the residual and the
    // exchange.  Otherwise: the quantiser, one launch per segment and the combine.
    if (nseg == 2 && segs[0].kind != TRX_KIND_Q8 && segs[1].kind != TRX_KIND_Q8 && aligned16(d_x)) {
        trx::MvJobs J0 = base_jobs(ctx, segs, d_packed[0]), J1 = base_jobs(ctx, segs + 1, d_packed[1]);
        J0.x = J1.x = d_x;
        J0.x_cols = J1.x_cols = (int)K;
        J0.x_off = 0;
        J1.x_off = (int)segs[0].cols;
        J0.seg[0].y = ctx->kseg_part;
        J0.out = trx::OUT_I32;
        J1.part_in = ctx->kseg_part;
        J1.seg[0].y = d_y;
        J1.seg[0].resid = d_resid;
        J1.out = trx::OUT_F32;
        J1.tp = X;
        J0.tp = X;  // the tagged input only: its results stay on this rank
        J0.tp.tag_out = -1;
        if (trx::matvec_launchable(J0) && trx::matvec_launchable(J1)) {
            if (trx_status s = trx::launch_matvec(J0, ctx->lut, ctx->err, stream)) return s;
            return trx::launch_matvec(J1, ctx->lut, ctx->err, stream);
        }
    }
    int *e8 = reinterpret_cast<int *>(ctx->q8x + kQ8MaxCols);
    trx_status s = tagged_in ? trx::launch_quantize_tagged(d_x, (int)K, ctx->q8x, e8, X, ctx->err, stream)
                             : trx::launch_quantize(d_x, (int)K, ctx->q8x, e8, stream);
    if (s) return s;
    uint64_t c0 = 0;
    for (int i = 0; i < nseg; ++i) {
        const trx_entry *e = segs + i;
        int32_t *part = ctx->kseg_part + (size_t)i * rows;
        if (e->kind == TRX_KIND_Q8) {
            s = trx::launch_matvec_q8(static_cast<const uint8_t *>(d_packed[i]), (int)rows, (int)e->cols, e->bias,
                                      e->rshift, ctx->q8x + c0, nullptr, part, ctx->err, stream);
        } else {
            trx::MvJobs J = base_jobs(ctx, e, d_packed[i]);
            J.x8 = ctx->q8x + c0;
            J.seg[0].y = part;
            J.out = trx::OUT_I32;
            s = trx::launch_matvec(J, ctx->lut, ctx->err, stream);
        }
        if (s) return s;
        c0 += e->cols;
    }
    return trx::launch_kseg_combine(ctx->kseg_part, nseg, (int)rows, e8, segs[0].rshift, segs[0].bias, d_resid, d_y,
                                    stream, X.world ? &X : nullptr);
}

trx_status trx_advance_position(trx_ctx *ctx, int32_t *d_pos, int32_t n, cudaStream_t stream) {
    if (!ctx || !d_pos) return TRX_ERR_ARG;
    return trx::launch_advance(d_pos, n, stream);
}

trx_status trx_lmhead_argmax(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                             const float *d_norm_w, float eps, float *d_logits, int32_t *d_token,
                             cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_token || !aligned16(d_packed)) return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x = d_x;
    J.norm_w = d_norm_w;
    J.eps = eps;
    J.seg[0].y = d_logits;
    J.out = trx::OUT_F32;
    J.argmax = ctx->amax_key;
    J.token = d_token;
    J.arg_cnt = ctx->amax_cnt;
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_lmhead_argmax_key(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                                 const float *d_norm_w, float eps, uint32_t row_offset, float *d_logits,
                                 uint64_t *d_key, cudaStream_t stream) {
    return trx_lmhead_argmax_key_tp(ctx, e, d_packed, d_x, d_norm_w, eps, row_offset, d_logits, d_key, nullptr,
                                    stream);
}

trx_status trx_lmhead_argmax_key_tp(trx_ctx *ctx, const trx_entry *e, const void *d_packed, const float *d_x,
                                    const float *d_norm_w, float eps, uint32_t row_offset, float *d_logits,
                                    uint64_t *d_key, const trx_tp_xfer *tp, cudaStream_t stream) {
    if (!ctx) return TRX_ERR_ARG;
    trx_status s = check_entry(e);
    if (s) return s;
    if (!d_packed || !d_x || !d_key || !aligned16(d_packed) || (uint64_t)row_offset + e->rows > 0xffffffffull)
        return TRX_ERR_ARG;
    trx::MvJobs J = base_jobs(ctx, e, d_packed);
    J.x = d_x;
    J.norm_w = d_norm_w;
    J.eps = eps;
    J.seg[0].y = d_logits;
    J.out = trx::OUT_F32;
    J.argmax = ctx->amax_key;
    J.key_out = reinterpret_cast<unsigned long long *>(d_key);
    J.row_offset = (int)row_offset;
    J.arg_cnt = ctx->amax_cnt;
    if ((s = tp_resolve(tp, TP_PUSH | TP_SIGNAL | TP_WAIT, J.tp))) return s;
    J.tp.arrive = nullptr;  // the argmax tail's last CTA signals
    return trx::launch_matvec(J, ctx->lut, ctx->err, stream);
}

trx_status trx_argmax_token(trx_ctx *ctx, const uint64_t *d_keys, int32_t n, int32_t *d_token, cudaStream_t stream) {
    return trx_argmax_token_tp(ctx, d_keys, n, d_token, nullptr, stream);
}

trx_status trx_argmax_token_tp(trx_ctx *ctx, const uint64_t *d_keys, int32_t n, int32_t *d_token,
                               const trx_tp_xfer *tp, cudaStream_t stream) {
    if (!ctx || !d_keys || !d_token || n < 1) return TRX_ERR_ARG;
    trx::TpXfer X;
    if (trx_status s = tp_resolve(tp, TP_WAIT, X)) return s;
    return trx::launch_argmax_keys(reinterpret_cast<const unsigned long long *>(d_keys), n, d_token, X, ctx->err,
                                   stream);
}

trx_status trx_attn_decode(trx_ctx *ctx, const trx_attn_shape *sh, const float *d_q, const float *d_k,
                           const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                           const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                           float *d_out, cudaStream_t stream) {
    return trx_attn_decode_tp(ctx, sh, d_q, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope_freq, d_kcache, d_vcache, d_pos,
                              d_out, nullptr, stream);
}

// One decode-attention launch's arguments from the C ABI's (esize: bytes per cache element).
static trx_status attn_args(trx_ctx *ctx, const trx_attn_shape *sh, const float *d_q, const float *d_k,
                            const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                            const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                            float *d_out, int esize, trx::AttnArgs &A) {
    if (!ctx || !sh) return TRX_ERR_ARG;
    const uint32_t H = sh->n_head, Hkv = sh->n_kv, hd = sh->head_dim;
    if (H == 0 || Hkv == 0 || H % Hkv || Hkv > kAttnMaxKv || hd == 0 || hd % 8 || hd > 512) return TRX_ERR_ARG;
    if (sh->rope_dims % 2 || sh->rope_dims > hd || sh->max_pos == 0 || sh->max_pos > (1u << 24)) return TRX_ERR_ARG;
    if (!(sh->eps >= 0.f)) return TRX_ERR_ARG;
    if (!d_q || !d_k || !d_v || !d_qnorm_w || !d_knorm_w || !d_kcache || !d_vcache || !d_pos || !d_out)
        return TRX_ERR_ARG;
    if ((sh->rope_dims && !d_rope_freq) || !aligned16(d_kcache) || !aligned16(d_vcache)) return TRX_ERR_ARG;
    A = trx::AttnArgs{};
    A.H = (int)H;
    A.Hkv = (int)Hkv;
    A.hd = (int)hd;
    A.rope_half = (int)sh->rope_dims / 2;
    A.gated = sh->gated ? 1 : 0;
    A.qstride = (int)hd * (A.gated ? 2 : 1);
    A.max_pos = (int)sh->max_pos;
    A.chunk = trx::attn_chunk(A.max_pos, A.hd, esize);
    A.nsplit = (A.max_pos + A.chunk - 1) / A.chunk;
    A.eps = sh->eps;
    A.scale = 1.0f / sqrtf((float)hd);
    const uint32_t rep = H / Hkv;
    if ((uint64_t)Hkv * A.nsplit * rep * (hd + 2) > kAttnPartFloats) return TRX_ERR_UNSUPPORTED;
    // The merge stages 2 floats per partial in the tiles' shared memory.
    if (trx::attn_smem_bytes((int)hd, (int)rep, A.chunk, esize) > 226u * 1024u ||
        2ull * rep * A.nsplit * 4 > 2ull * A.chunk * (hd + 16 / esize) * esize)
        return TRX_ERR_UNSUPPORTED;
    A.q = d_q;
    A.k = d_k;
    A.v = d_v;
    A.qn = d_qnorm_w;
    A.kn = d_knorm_w;
    A.freq = d_rope_freq;
    A.pos = d_pos;
    A.kc = static_cast<__half *>(d_kcache);
    A.vc = static_cast<__half *>(d_vcache);
    A.out = d_out;
    A.part = ctx->attn_part;
    A.cnt = ctx->attn_cnt;
    A.f32cache = esize == 4 ? 1 : 0;
    return TRX_OK;
}

trx_status trx_attn_decode_tp(trx_ctx *ctx, const trx_attn_shape *sh, const float *d_q, const float *d_k,
                              const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                              const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                              float *d_out, const trx_tp_xfer *tp, cudaStream_t stream) {
    trx::AttnArgs A;
    if (trx_status s = attn_args(ctx, sh, d_q, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope_freq, d_kcache, d_vcache, d_pos,
                                 d_out, 2, A))
        return s;
    if (trx_status s = tp_resolve(tp, TP_PUSH | TP_SIGNAL, A.tp)) return s;
    return trx::launch_attn_decode(A, ctx->err, stream);
}

trx_status trx_attn_decode_rows(trx_ctx *ctx, const trx_attn_shape *sh, int32_t nseq, const float *d_q,
                                const float *d_k, const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                                const float *d_rope_freq, void *d_kcache, void *d_vcache, const int32_t *d_pos,
                                float *d_out, cudaStream_t stream) {
    trx::AttnArgs A;
    if (trx_status s = attn_args(ctx, sh, d_q, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope_freq, d_kcache, d_vcache, d_pos,
                                 d_out, 2, A))
        return s;
    if (nseq < 1 || nseq > 65535) return TRX_ERR_ARG;
    A.scratch_merge = 1;  // the kernel with a sequence dimension
    A.nseq = nseq;
    A.q_bs = (long long)A.H * A.qstride;
    A.kv_bs = (long long)A.Hkv * A.hd;
    A.cache_bs = (long long)A.max_pos * A.Hkv * A.hd;
    A.out_bs = (long long)A.H * A.hd;
    A.part_bs = (long long)A.Hkv * A.nsplit * (A.H / A.Hkv) * (A.hd + 2);
    if ((uint64_t)nseq * A.part_bs > kAttnPartFloats || (uint64_t)nseq * A.Hkv > kAttnMaxKv) return TRX_ERR_UNSUPPORTED;
    return trx::launch_attn_decode(A, ctx->err, stream);
}

trx_status trx_attn_decode_f32cache(trx_ctx *ctx, const trx_attn_shape *sh, const float *d_q, const float *d_k,
                                    const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                                    const float *d_rope_freq, float *d_kcache, float *d_vcache, const int32_t *d_pos,
                                    float *d_out, cudaStream_t stream) {
    trx::AttnArgs A;
    if (trx_status s = attn_args(ctx, sh, d_q, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope_freq, d_kcache, d_vcache, d_pos,
                                 d_out, 4, A))
        return s;
    A.scratch_merge = 1;  // the scratch-merge kernel is the one with an fp32-cache form
    return trx::launch_attn_decode(A, ctx->err, stream);
}

static trx_status deltanet_step(trx_ctx *ctx, const trx_deltanet_shape *sh, int32_t nseq, const float *d_qkv,
                                const float *d_z, const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                                const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                                float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                                const trx_tp_xfer *tp, cudaStream_t stream);

trx_status trx_deltanet_step(trx_ctx *ctx, const trx_deltanet_shape *sh, const float *d_qkv, const float *d_z,
                             const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                             const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                             float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                             cudaStream_t stream) {
    return deltanet_step(ctx, sh, 1, d_qkv, d_z, d_beta, d_alpha, d_dt_bias, d_ssm_a, d_conv_w, d_norm_w, d_conv_ring,
                         d_state, d_pos, d_out, nullptr, stream);
}

trx_status trx_deltanet_step_tp(trx_ctx *ctx, const trx_deltanet_shape *sh, const float *d_qkv, const float *d_z,
                                const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                                const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                                float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                                const trx_tp_xfer *tp, cudaStream_t stream) {
    return deltanet_step(ctx, sh, 1, d_qkv, d_z, d_beta, d_alpha, d_dt_bias, d_ssm_a, d_conv_w, d_norm_w, d_conv_ring,
                         d_state, d_pos, d_out, tp, stream);
}

trx_status trx_deltanet_int_step(trx_ctx *ctx, uint32_t nheads, uint32_t hv, uint32_t hk, int16_t *d_state,
                                 int32_t *d_exp, int32_t *d_maxabs, const float *d_k, const float *d_q, const float *d_v,
                                 const float *d_decay, const float *d_beta, float *d_out, cudaStream_t stream) {
    if (!ctx || nheads == 0 || nheads > (1u << 20) || hv == 0 || hk == 0) return TRX_ERR_ARG;
    if (!d_state || !d_exp || !d_maxabs || !d_k || !d_q || !d_v || !d_decay || !d_beta || !d_out) return TRX_ERR_ARG;
    if (hv > 256 || hk > 128) return TRX_ERR_UNSUPPORTED;
    trx::DnIntArgs A{};
    A.nh = (int)nheads;
    A.hv = (int)hv;
    A.hk = (int)hk;
    A.M = d_state;
    A.eM = d_exp;
    A.maxM = d_maxabs;
    A.k = d_k;
    A.q = d_q;
    A.v = d_v;
    A.decay = d_decay;
    A.beta = d_beta;
    A.out = d_out;
    return trx::launch_dn_int(A, ctx->err, stream);
}

trx_status trx_deltanet_step_rows(trx_ctx *ctx, const trx_deltanet_shape *sh, int32_t nseq, const float *d_qkv,
                                  const float *d_z, const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                                  const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                                  float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                                  cudaStream_t stream) {
    return deltanet_step(ctx, sh, nseq, d_qkv, d_z, d_beta, d_alpha, d_dt_bias, d_ssm_a, d_conv_w, d_norm_w,
                         d_conv_ring, d_state, d_pos, d_out, nullptr, stream);
}

static trx_status deltanet_step(trx_ctx *ctx, const trx_deltanet_shape *sh, int32_t nseq, const float *d_qkv,
                                const float *d_z, const float *d_beta, const float *d_alpha, const float *d_dt_bias,
                                const float *d_ssm_a, const float *d_conv_w, const float *d_norm_w,
                                float *d_conv_ring, float *d_state, const int32_t *d_pos, float *d_out,
                                const trx_tp_xfer *tp, cudaStream_t stream) {
    if (!ctx || !sh || nseq < 1 || nseq > 65535) return TRX_ERR_ARG;
    const uint32_t nk = sh->n_k_heads, hk = sh->k_head_dim, nv = sh->n_v_heads, hv = sh->v_head_dim;
    const uint32_t K = sh->conv_kernel;
    if (nk == 0 || nv == 0 || nv % nk || nv > kAttnMaxKv) return TRX_ERR_ARG;
    if (!(hk == 32 || hk == 64 || hk == 128 || hk == 256) || hv == 0 || hv > 1024 || K < 2 || K > 8) return TRX_ERR_ARG;
    if (!(sh->eps >= 0.f)) return TRX_ERR_ARG;
    if (!d_qkv || !d_z || !d_beta || !d_alpha || !d_dt_bias || !d_ssm_a || !d_conv_w || !d_norm_w || !d_conv_ring ||
        !d_state || !d_pos || !d_out)
        return TRX_ERR_ARG;
    if ((uint64_t)nseq * nv * hv > kAttnPartFloats || (uint64_t)nseq * nv > kAttnMaxKv) return TRX_ERR_UNSUPPORTED;
    trx::DnArgs A{};
    A.nseq = nseq;
    A.nk = (int)nk;
    A.hk = (int)hk;
    A.nv = (int)nv;
    A.hv = (int)hv;
    A.K = (int)K;
    A.C = (int)(2 * nk * hk + nv * hv);
    // Rows per CTA: about two CTAs per SM over all heads and sequences, at least 8 rows each.
    int nsplit = (int)((2 * 148 + (uint64_t)nv * nseq - 1) / ((uint64_t)nv * nseq));
    int rows = (int)((hv + nsplit - 1) / nsplit);
    if (rows < 8) rows = 8;
    A.rows = rows;
    A.nsplit = (int)((hv + rows - 1) / rows);
    A.eps = sh->eps;
    A.scale = 1.0f / sqrtf((float)hk);
    A.qkv = d_qkv;
    A.z = d_z;
    A.beta = d_beta;
    A.alpha = d_alpha;
    A.dt_bias = d_dt_bias;
    A.ssm_a = d_ssm_a;
    A.conv_w = d_conv_w;
    A.norm_w = d_norm_w;
    A.pos = d_pos;
    A.win = d_conv_ring;
    A.S = d_state;
    A.out = d_out;
    A.part = ctx->attn_part;
    A.cnt = ctx->attn_cnt;
    if (trx_status st = tp_resolve(tp, TP_PUSH, A.tp)) return st;
    if (A.tp.world && (nseq != 1 || A.tp.tag_out < 0)) return TRX_ERR_UNSUPPORTED;  // tagged words, one sequence
    return trx::launch_deltanet(A, ctx->err, stream);
}

}  // extern "C"
