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

trx_status launch_argmax_keys(const unsigned long long *keys, int n, int *token, const TpXfer &tp, uint32_t *err,
                              cudaStream_t st) {
    return note_cuda(launch_kernel(argmax_keys_kernel, dim3(1), dim3(32), 0, st, keys, n, token, tp, err));
}

trx_status launch_advance(int *pos, int n, cudaStream_t st) {
    return note_cuda(launch_kernel(advance_kernel, dim3(1), dim3(1), 0, st, pos, n));
}

}  // namespace trx
