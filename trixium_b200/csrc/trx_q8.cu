// The engine's Q8 row-dot matvec (model/bitexact.py:127-144, matvec_q8) over KIND_Q8 row packets
// (model/layout.py:41,47,189-217; model/bons.py:150-169): each row is ceil(G/16) beats of fp16
// group scales, then G beats of 32 int8 weights, G = K/32.
//
//   gs(g)  = sum over the group's 32 lanes of q8w * x8            exact int32, |gs| <= 32*128*128
//   acc    = sum_g (gs * m11(g)) shifted by e16(g) + B             int64 (floor on right shifts)
//   result = acc >> R                                              int32
//
// One warp per row, rows strided over one wave of resident CTAs.  The row's 16-byte words are
// dealt round-robin to the lanes (word i to lane i % 32), so a warp's loads cover 512 contiguous
// bytes and lane pair (2j, 2j+1) holds one whole group: each lane takes its half-group sum with
// four dp4a against the matching x8 word (x8 staged once per CTA in shared memory), the pair adds
// the halves by one shuffle and the even lane applies the group's scale.  Integer addition is
// exact, so the order of the warp reduction does not change the result.  The weights are read
// once with an evict-first hint; the launch is bound by HBM bandwidth.
#include <cstdint>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

namespace {

constexpr int kQ8Warps = 8;   // rows in flight per CTA, one per warp
constexpr int kQ8Unroll = 4;  // 16-byte weight words in flight per lane

// F32: the float projection of a Q8 tensor (model/mirror.py:664-678 with matvec_q8): x8 and its
// exponent e8 come from the quantiser launched just before, y = fp32(result) * 2^(e8 + R - B).
template <bool F32>
__global__ void __launch_bounds__(kQ8Warps * 32) q8_matvec_kernel(const uint8_t *w, int rows, int cols, int B, int R,
                                                                   const int8_t *x8, const int *e8, void *out,
                                                                   uint32_t *err) {
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
    const int lane = threadIdx.x & 31;
    const ScaleFast F = scale_fast(B);
    const float ysc = F32 ? pow2f(*e8 + R - B) : 0.f;
    for (int row = blockIdx.x * kQ8Warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kQ8Warps) {
        const uint8_t *rp = w + (size_t)row * rb;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(rp);
        const uint4 *cw = reinterpret_cast<const uint4 *>(rp + sb);
        long long acc = 0;
        for (int w0 = 0; w0 < nw; w0 += 32 * kQ8Unroll) {
            uint4 c[kQ8Unroll];
            uint32_t s[kQ8Unroll];
#pragma unroll
            for (int u = 0; u < kQ8Unroll; ++u) {
                const int i = w0 + u * 32 + lane;
                if (i < nw) {
                    c[u] = __ldcs(cw + i);
                    s[u] = __ldg(sc + (i >> 1));
                } else {
                    c[u] = make_uint4(0u, 0u, 0u, 0u);
                    s[u] = 0u;
                }
            }
#pragma unroll
            for (int u = 0; u < kQ8Unroll; ++u) {
                const int i = w0 + u * 32 + lane;
                const uint4 xv = xs[i < nw ? i : 0];
                int gs = __dp4a((int)c[u].x, (int)xv.x, 0);
                gs = __dp4a((int)c[u].y, (int)xv.y, gs);
                gs = __dp4a((int)c[u].z, (int)xv.z, gs);
                gs = __dp4a((int)c[u].w, (int)xv.w, gs);
                gs += __shfl_xor_sync(0xffffffffu, gs, 1);  // the partner lane's half of the group
                if (!(lane & 1) && i < nw) acc += contrib(gs, s[u], B, F);
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
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
    long long grid = ((long long)rows + kQ8Warps - 1) / kQ8Warps;
    const int resident = e8 ? q8_resident<true>(smem) : q8_resident<false>(smem);
    if (grid > resident) grid = resident;  // one wave; the warps stride over the remaining rows
    const dim3 g((unsigned)grid), b(kQ8Warps * 32);
    if (e8)
        return note_cuda(launch_kernel(q8_matvec_kernel<true>, g, b, smem, st, w, rows, cols, B, R, x8, e8, out, err));
    return note_cuda(launch_kernel(q8_matvec_kernel<false>, g, b, smem, st, w, rows, cols, B, R, x8, e8, out, err));
}

}  // namespace trx
