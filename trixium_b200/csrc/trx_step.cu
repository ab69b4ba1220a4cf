// Small per-token kernels of the decode step: the embedding row of the current token and the
// position advance (model/mirror.py:1002-1004 embed_row; the step counter the attention and
// DeltaNet kernels read).
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

// x = table[token] as fp32 (fp16 or fp32 table rows).  A token outside [0, vocab) sets
// TRX_DEV_RANGE and writes zeros.
__global__ void embed_kernel(const void *table, int vocab, int dim, int f16, const int *token, float *x,
                             uint32_t *err) {
    pdl_trigger();
    pdl_wait();
    token += blockIdx.y;  // row y of a batch: its token and output row
    x += (size_t)blockIdx.y * dim;
    const int t = *token;
    const bool ok = t >= 0 && t < vocab;
    if (!ok && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, TRX_DEV_RANGE);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        float v = 0.f;
        if (ok)
            v = f16 ? __half2float(reinterpret_cast<const __half *>(table)[(size_t)t * dim + i])
                    : reinterpret_cast<const float *>(table)[(size_t)t * dim + i];
        x[i] = v;
    }
}

// x = mant[token] * 2^exps[token]: the int16 embedding table of a BONS image (model/mirror.py:777-783,
// exact in fp32).  A token outside [0, vocab) sets TRX_DEV_RANGE and writes zeros.
__global__ void embed_bfp16_kernel(const int16_t *mant, const int *exps, int vocab, int dim, const int *token,
                                   float *x, uint32_t *err) {
    pdl_trigger();
    pdl_wait();
    const int t = *token;
    const bool ok = t >= 0 && t < vocab;
    if (!ok && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, TRX_DEV_RANGE);
    const float sc = ok ? pow2f(exps[t]) : 0.f;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        x[i] = ok ? __fmul_rn((float)mant[(size_t)t * dim + i], sc) : 0.f;
}

// y = (x * r) * w, r = 1 / sqrt(ss / n + eps) with ss the canonical sum of squares: 64 sequential
// fp32 partials (partial j over x[j], x[j + 64], ... in index order), then the halving tree
// (model/mirror.py:576-591, :697-700).  One CTA of 256 threads.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, const float *w, int n, float eps, float *y) {
    __shared__ float part[64];
    pdl_trigger();
    pdl_wait();
    x += (size_t)blockIdx.x * n;  // one CTA per row
    y += (size_t)blockIdx.x * n;
    const int t = threadIdx.x;
    if (t < 64) {
        float p = 0.f;
        for (int i = t; i < n; i += 64) p = __fadd_rn(p, __fmul_rn(x[i], x[i]));
        part[t] = p;
    }
    __syncthreads();
    for (int h = 32; h >= 1; h >>= 1) {
        if (t < h) part[t] = __fadd_rn(part[t], part[t + h]);
        __syncthreads();
    }
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(part[0], (float)n), eps)));
    for (int i = t; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
}

// act = silu(g) * u elementwise (model/mirror.py:713,1020: x / (1 + exp(-x)) in fp32, mathematical
// profile), as the SwiGLU epilogue of the matvec kernel computes it.
__global__ void silu_mul_kernel(const float *g, const float *u, long long n, float *act) {
    pdl_trigger();
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float gv = g[i];
        act[i] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), u[i]);
    }
}

// Per row of logits [nrows][V]: the index of the largest value, ties to the smallest index (the
// greedy token, model/mirror.py:1031; doc/units.md:149).  One CTA per row.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const float *logits, int V, int *tokens) {
    __shared__ unsigned long long best_s[8];
    pdl_trigger();
    pdl_wait();
    const float *l = logits + (size_t)blockIdx.x * V;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long k = argmax_key(l[i], (uint32_t)i);
        best = k > best ? k : best;
    }
    for (int o = 16; o; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    if ((threadIdx.x & 31) == 0) best_s[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) best = best_s[w] > best ? best_s[w] : best;
        tokens[blockIdx.x] = best ? (int)(0xffffffffu - (uint32_t)best) : -1;
    }
}

__global__ void advance_rows_kernel(int *pos, int count, int n) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) pos[i] += n;
}

// The float result of a K-segmented projection (model/mirror.py:664-678): the segments' int32
// engine results added in int64, wrapped to int32, times 2^(e8 + R - B), plus the residual.
__global__ void kseg_combine_kernel(const int *parts, int nseg, int rows, const int *e8, int R, int B,
                                    const float *resid, float *y, TpXfer tp) {
    pdl_trigger();
    pdl_wait();
    const float sc = pow2f(*e8 + R - B);
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
        long long a = 0;
        for (int s = 0; s < nseg; ++s) a += parts[(size_t)s * rows + r];
        float v = __fmul_rn((float)(int)(uint32_t)(unsigned long long)a, sc);
        if (resid) v = __fadd_rn(resid[r], v);
        y[r] = v;
        if (tp.world) tp_push_all(tp, (size_t)r, v);  // tensor-parallel gather of the rows
    }
}

// The token of the largest of n argmax keys (one per shard of a row-sharded LM head).
__global__ void argmax_keys_kernel(const unsigned long long *keys, int n, int *token, TpXfer tp, uint32_t *err) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) {
        tp_wait(tp, err);  // the other ranks' keys, stored here by their launches
        unsigned long long best = 0ull;
        for (int i = 0; i < n; ++i) best = keys[i] > best ? keys[i] : best;
        *token = best ? (int)(0xffffffffu - (uint32_t)best) : -1;
    }
}

__global__ void advance_kernel(int *pos, int n) {
    pdl_trigger();
    pdl_wait();
    *pos += n;
}

trx_status launch_embed(const void *table, int vocab, int dim, int f16, const int *token, float *x, uint32_t *err,
                        cudaStream_t st) {
    const int blocks = (dim + 255) / 256 < 16 ? (dim + 255) / 256 : 16;
    return note_cuda(launch_kernel(embed_kernel, dim3(blocks), dim3(256), 0, st, table, vocab, dim, f16, token, x, err));
}

trx_status launch_embed_rows(const void *table, int vocab, int dim, int f16, const int *tokens, int nrows, float *x,
                             uint32_t *err, cudaStream_t st) {
    const int blocks = (dim + 255) / 256 < 16 ? (dim + 255) / 256 : 16;
    return note_cuda(
        launch_kernel(embed_kernel, dim3(blocks, nrows), dim3(256), 0, st, table, vocab, dim, f16, tokens, x, err));
}

trx_status launch_rmsnorm_rows(const float *x, const float *w, int n, int nrows, float eps, float *y,
                               cudaStream_t st) {
    return note_cuda(launch_kernel(rmsnorm_kernel, dim3(nrows), dim3(256), 0, st, x, w, n, eps, y));
}

trx_status launch_silu_mul(const float *g, const float *u, long long n, float *act, cudaStream_t st) {
    long long blocks = (n + 255) / 256;
    if (blocks > 1184) blocks = 1184;
    return note_cuda(launch_kernel(silu_mul_kernel, dim3((unsigned)blocks), dim3(256), 0, st, g, u, n, act));
}

trx_status launch_argmax_rows(const float *logits, int V, int nrows, int *tokens, cudaStream_t st) {
    return note_cuda(launch_kernel(argmax_rows_kernel, dim3(nrows), dim3(256), 0, st, logits, V, tokens));
}

trx_status launch_advance_rows(int *pos, int count, int n, cudaStream_t st) {
    return note_cuda(launch_kernel(advance_rows_kernel, dim3((count + 255) / 256), dim3(256), 0, st, pos, count, n));
}

trx_status launch_embed_bfp16(const int16_t *mant, const int *exps, int vocab, int dim, const int *token, float *x,
                              uint32_t *err, cudaStream_t st) {
    const int blocks = (dim + 255) / 256 < 16 ? (dim + 255) / 256 : 16;
    return note_cuda(
        launch_kernel(embed_bfp16_kernel, dim3(blocks), dim3(256), 0, st, mant, exps, vocab, dim, token, x, err));
}

trx_status launch_rmsnorm(const float *x, const float *w, int n, float eps, float *y, cudaStream_t st) {
    return note_cuda(launch_kernel(rmsnorm_kernel, dim3(1), dim3(256), 0, st, x, w, n, eps, y));
}

trx_status launch_kseg_combine(const int *parts, int nseg, int rows, const int *e8, int R, int B, const float *resid,
                               float *y, cudaStream_t st, const TpXfer *tp) {
    int blocks = (rows + 255) / 256;
    if (blocks > 148) blocks = 148;
    const TpXfer X = tp ? *tp : TpXfer{};
    return note_cuda(
        launch_kernel(kseg_combine_kernel, dim3(blocks), dim3(256), 0, st, parts, nseg, rows, e8, R, B, resid, y, X));
}

trx_status launch_argmax_keys(const unsigned long long *keys, int n, int *token, const TpXfer &tp, uint32_t *err,
                              cudaStream_t st) {
    return note_cuda(launch_kernel(argmax_keys_kernel, dim3(1), dim3(32), 0, st, keys, n, token, tp, err));
}

trx_status launch_advance(int *pos, int n, cudaStream_t st) {
    return note_cuda(launch_kernel(advance_kernel, dim3(1), dim3(1), 0, st, pos, n));
}

}  // namespace trx
