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

// The float result of a K-segmented projection (model/mirror.py:664-678): the segments' int32
// engine results added in int64, wrapped to int32, times 2^(e8 + R - B), plus the residual.
__global__ void kseg_combine_kernel(const int *parts, int nseg, int rows, const int *e8, int R, int B,
                                    const float *resid, float *y) {
    pdl_trigger();
    pdl_wait();
    const float sc = pow2f(*e8 + R - B);
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
        long long a = 0;
        for (int s = 0; s < nseg; ++s) a += parts[(size_t)s * rows + r];
        float v = __fmul_rn((float)(int)(uint32_t)(unsigned long long)a, sc);
        if (resid) v = __fadd_rn(resid[r], v);
        y[r] = v;
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
                               float *y, cudaStream_t st) {
    int blocks = (rows + 255) / 256;
    if (blocks > 148) blocks = 148;
    return note_cuda(
        launch_kernel(kseg_combine_kernel, dim3(blocks), dim3(256), 0, st, parts, nseg, rows, e8, R, B, resid, y));
}

trx_status launch_argmax_keys(const unsigned long long *keys, int n, int *token, const TpXfer &tp, uint32_t *err,
                              cudaStream_t st) {
    return note_cuda(launch_kernel(argmax_keys_kernel, dim3(1), dim3(32), 0, st, keys, n, token, tp, err));
}

trx_status launch_advance(int *pos, int n, cudaStream_t st) {
    return note_cuda(launch_kernel(advance_kernel, dim3(1), dim3(1), 0, st, pos, n));
}

}  // namespace trx
