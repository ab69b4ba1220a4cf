// The engine's Q8 row-dot matvec (model/bitexact.py:127-144, matvec_q8) over KIND_Q8 row packets
// (model/layout.py:41,47,189-217; model/bons.py:150-169): each row is ceil(G/16) beats of fp16
// group scales, then G beats of 32 int8 weights, G = K/32.
//
//   gs(g)  = sum over the group's 32 lanes of q8w * x8            exact int32, |gs| <= 32*128*128
//   acc    = sum_g (gs * m11(g)) shifted by e16(g) + B             int64 (floor on right shifts)
//   result = acc >> R                                              int32
//
// A group of lpr lanes per row (lpr = 32 for rows of 2048 weights and more; 16, 8, ... for shorter
// rows, so that every lane keeps kQ8Unroll 16-byte words in flight), rows strided over one wave of
// resident CTAs.  The row's 16-byte words are dealt round-robin to its group (word i to lane
// i % lpr), so a group's loads cover 16*lpr contiguous bytes and lane pair (2j, 2j+1) holds one
// whole group of 32 weights: each lane takes its half-group sum with four dp4a against the
// matching x8 word (x8 staged once per CTA in shared memory), the pair adds the halves by one
// shuffle and the even lane applies the group's scale.  Integer addition is exact, so the order
// of the reduction does not change the result.  The weights are read once with an evict-first
// hint; the launch is bound by HBM bandwidth.
#include <cstdint>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

namespace {

#ifndef TRX_Q8_UNROLL
#define TRX_Q8_UNROLL 4
#endif
#ifndef TRX_Q8_MINB
#define TRX_Q8_MINB 1
#endif
constexpr int kQ8Warps = 8;                 // rows in flight per CTA, one per warp
constexpr int kQ8Unroll = TRX_Q8_UNROLL;    // 16-byte weight words in flight per lane

// F32: the float projection of a Q8 tensor (model/mirror.py:664-678 with matvec_q8): x8 and its
// exponent e8 come from the quantiser launched just before, y = fp32(result) * 2^(e8 + R - B).
template <bool F32>
__global__ void __launch_bounds__(kQ8Warps * 32, TRX_Q8_MINB)
    q8_matvec_kernel(const uint8_t *w, int rows, int cols, int B, int R, int lpr_log2, const int8_t *x8, const int *e8,
                     void *out, uint32_t *err) {
    extern __shared__ uint4 xs[];  // x8 as cols/16 words
    pdl_trigger();
    pdl_wait();
    const int nw = cols >> 4;  // 16-byte words per row, even (cols is a multiple of 32)
    const int G = cols >> 5;
    const size_t sb = (size_t)((G + 15) >> 4) * 32;
    const size_t rb = sb + (size_t)cols;
    if ((reinterpret_cast<uintptr_t>(x8) & 15u) == 0) {
        for (int i = threadIdx.x; i < nw; i += blockDim.x) xs[i] = reinterpret_cast<const uint4 *>(x8)[i];
    } else {
        for (int i = threadIdx.x; i < cols; i += blockDim.x) reinterpret_cast<int8_t *>(xs)[i] = x8[i];
    }
    __syncthreads();
    // A row is read by a group of lpr = 2^lpr_log2 lanes (2 <= lpr <= 32, chosen so that a short
    // row still gives every lane kQ8Unroll words in flight); a warp reads 32/lpr rows at a time.
    const int lane = threadIdx.x & 31;
    const int lpr = 1 << lpr_log2;
    const int sl = lane & (lpr - 1);          // lane within the row's group
    const int sub = lane >> lpr_log2;         // the group's row within the warp's set
    const int rpw = 32 >> lpr_log2;           // rows per warp per pass
    const ScaleFast F = scale_fast(B);
    const float ysc = F32 ? pow2f(*e8 + R - B) : 0.f;
    for (int r0 = (blockIdx.x * kQ8Warps + (threadIdx.x >> 5)) * rpw; r0 < rows; r0 += gridDim.x * kQ8Warps * rpw) {
        const int row = r0 + sub;
        const int wend = row < rows ? nw : 0;  // a group past the last row loads nothing
        const uint8_t *rp = w + (size_t)(row < rows ? row : 0) * rb;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(rp);
        const uint4 *cw = reinterpret_cast<const uint4 *>(rp + sb);
        long long acc = 0;
        for (int w0 = 0; w0 < nw; w0 += lpr * kQ8Unroll) {  // the same trip count in every lane
            uint4 c[kQ8Unroll];
            uint32_t s[kQ8Unroll];
#pragma unroll
            for (int u = 0; u < kQ8Unroll; ++u) {
                const int i = w0 + u * lpr + sl;
                if (i < wend) {
                    c[u] = __ldcs(cw + i);
                    s[u] = __ldg(sc + (i >> 1));
                } else {
                    c[u] = make_uint4(0u, 0u, 0u, 0u);
                    s[u] = 0u;
                }
            }
#pragma unroll
            for (int u = 0; u < kQ8Unroll; ++u) {
                const int i = w0 + u * lpr + sl;
                const uint4 xv = xs[i < nw ? i : 0];
                int gs = __dp4a((int)c[u].x, (int)xv.x, 0);
                gs = __dp4a((int)c[u].y, (int)xv.y, gs);
                gs = __dp4a((int)c[u].z, (int)xv.z, gs);
                gs = __dp4a((int)c[u].w, (int)xv.w, gs);
                gs += __shfl_xor_sync(0xffffffffu, gs, 1);  // the partner lane's half of the group
                if (!(lane & 1) && i < wend) acc += contrib(gs, s[u], B, F);
            }
        }
        for (int o = lpr >> 1; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (sl == 0 && row < rows) {
            if (acc_bad(acc, R)) atomicOr(err, TRX_DEV_OVERFLOW);
            if (F32)
                reinterpret_cast<float *>(out)[row] = __fmul_rn((float)(int)(acc >> R), ysc);
            else
                reinterpret_cast<int32_t *>(out)[row] = (int)(acc >> R);
        }
    }
}

// Resident CTAs of the kernel on the whole GPU (SMs x CTAs per SM at the given shared memory).
template <bool F32>
int q8_resident(size_t smem) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, q8_matvec_kernel<F32>, kQ8Warps * 32, smem) != cudaSuccess ||
        per <= 0)
        per = 4;
    return sms * per;
}

}  // namespace

trx_status launch_matvec_q8(const uint8_t *w, int rows, int cols, int B, int R, const int8_t *x8, const int *e8,
                            void *out, uint32_t *err, cudaStream_t st) {
    const size_t smem = (size_t)cols;  // <= 32 KiB: within the default dynamic shared memory limit
    const int nw = cols / 16;
    int lg = 5;  // lanes per row: the largest power of two <= 32 giving each lane kQ8Unroll words
    while (lg > 1 && (1 << lg) * kQ8Unroll > nw) --lg;
    const long long rows_per_cta = (long long)kQ8Warps * (32 >> lg);
    long long grid = ((long long)rows + rows_per_cta - 1) / rows_per_cta;
    const int resident = e8 ? q8_resident<true>(smem) : q8_resident<false>(smem);
    if (grid > resident) grid = resident;  // one wave; the warps stride over the remaining rows
    const dim3 g((unsigned)grid), b(kQ8Warps * 32);
    if (e8)
        return note_cuda(launch_kernel(q8_matvec_kernel<true>, g, b, smem, st, w, rows, cols, B, R, lg, x8, e8, out, err));
    return note_cuda(launch_kernel(q8_matvec_kernel<false>, g, b, smem, st, w, rows, cols, B, R, lg, x8, e8, out, err));
}

}  // namespace trx
