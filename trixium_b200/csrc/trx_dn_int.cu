// The integer gated-DeltaNet head step for B200 (sm_100a): model/deltanet.py:99-147 (head_step), the
// vector unit's int16-state recurrence, bit-exact.  One CTA per head (heads are independent):
//  * q16_head of k and q (warps 0 and 1): int16 mantissas with one exponent, |m| in [2^14, 2^15) at
//    the max (model/deltanet.py:60-68), rounding half away from zero in double as the reference's
//    lroundf on float64 does;
//  * pass A, one warp per state row j: dot_j = M_j . k16 in int64, shifted to units of 2^-19, times
//    the Q15 decay (floor), plus -v_j (units 2^-19), times -beta Q15 (floor) = delta_j; the max
//    |delta| by a shared atomic;
//  * the exponent ratchet (model/deltanet.py:82-89) by one thread in double, the pass-B constants
//    (:91-97);
//  * pass B, one warp per row: M' = rne(M * d15n + delta_s * k16, 15) written back as int16, the max
//    |M'| for the next token, o_j = (M'_j . q16) >> 8 scaled to fp32 (model/deltanet.py:127-147).
// Where the reference asserts (a value outside its int range) the kernel sets TRX_DEV_OVERFLOW.
#include <cstdint>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

constexpr int kDnIntThreads = 256;
constexpr int kDnIntWarps = kDnIntThreads / 32;
constexpr int kDnIntMaxHk = 128;
constexpr int kDnIntMaxHv = 256;
constexpr int kDnDeltaFrac = 19;                 // model/deltanet.py:49
constexpr int kDnOShift = 8;                     // model/deltanet.py:50
constexpr double kDnStateLim = (1 << 15) - 4;    // model/deltanet.py:51

// Round half away from zero of a double (model/deltanet.py:55-58 on float64 values).
__device__ __forceinline__ long long lround_away(double x) {
    return (long long)(x >= 0.0 ? floor(x + 0.5) : ceil(x - 0.5));
}

// A [0, 1] fp32 constant as Q15 (model/deltanet.py:70-72): the fp32 product by 2^15 (exact), then
// the rounding in double, clipped to [0, 32767].
__device__ __forceinline__ int q15_of(float x, int shift) {
    const long long r = lround_away((double)__fmul_rn(x, pow2f(shift)));
    return (int)(r < 0 ? 0 : (r > 32767 ? 32767 : r));
}

// Shift left when k >= 0, floor right otherwise (model/bitexact.py:47-50).
__device__ __forceinline__ long long arith_shift_ll(long long v, int k) {
    return k >= 0 ? (long long)((unsigned long long)v << k) : (v >> (-k));
}

// Round-to-nearest-even right shift by 15 (model/bitexact.py:35-45).
__device__ __forceinline__ long long rne_shift15(long long v) {
    const long long q = v >> 15;
    const long long rb = (v >> 14) & 1;
    const long long sticky = (v & 0x3fff) != 0;
    return q + (rb & (sticky | (q & 1)));
}

__device__ __forceinline__ long long warp_sum_ll(long long v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ long long llabs_(long long v) { return v < 0 ? -v : v; }

__global__ void __launch_bounds__(kDnIntThreads) dn_int_kernel(DnIntArgs A, uint32_t *err) {
    __shared__ int k16[kDnIntMaxHk], q16[kDnIntMaxHk];
    __shared__ long long dl[kDnIntMaxHv];  // delta_j, then delta_s_j
    __shared__ int ek_s, eq_s, k16max_s, eM2_s, sh_s, d15n_s, bad_s;
    __shared__ long long rnd_s;
    __shared__ unsigned long long maxD_s;
    __shared__ unsigned maxM_s, maxM2_s;
    pdl_trigger();
    pdl_wait();
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hv = A.hv, hk = A.hk;
    int16_t *const M = A.M + (size_t)h * hv * hk;
    if (tid == 0) {
        maxD_s = 0ull;
        maxM_s = 0u;
        maxM2_s = 0u;
        bad_s = 0;
    }
    __syncthreads();
    // q16_head of k (warp 0) and q (warp 1).
    if (warp < 2) {
        const float *x = (warp ? A.q : A.k) + (size_t)h * hk;
        int *m = warp ? q16 : k16;
        uint32_t am = 0u;
        for (int c = lane; c < hk; c += 32) am = max(am, __float_as_uint(fabsf(x[c])));
        am = __reduce_max_sync(0xffffffffu, am);
        const int e = am ? frexp_exp(__uint_as_float(am)) - 15 : 0;
        const float sc = pow2f(-e);
        int mm = 0;
        for (int c = lane; c < hk; c += 32) {
            long long r = am ? lround_away((double)__fmul_rn(x[c], sc)) : 0;
            r = r < -32767 ? -32767 : (r > 32767 ? 32767 : r);
            m[c] = (int)r;
            mm = max(mm, (int)llabs_(r));
        }
        mm = __reduce_max_sync(0xffffffffu, (unsigned)mm);
        if (lane == 0) {
            if (warp)
                eq_s = e;
            else {
                ek_s = e;
                k16max_s = mm;
            }
        }
    }
    const bool need_max = A.maxM[h] < 0;  // the reference's maxM=None: max |M| of the state
    if (need_max) {
        unsigned m = 0u;
        for (int i = tid; i < hv * hk; i += kDnIntThreads) m = max(m, (unsigned)abs((int)M[i]));
        m = __reduce_max_sync(0xffffffffu, m);
        if (lane == 0) atomicMax(&maxM_s, m);
    }
    __syncthreads();
    const int eM = A.eM[h];
    const float decay = A.decay[h], beta = A.beta[h];
    const int ek = ek_s;
    const int shift_a = kDnDeltaFrac + eM + ek;  // model/deltanet.py:74-80
    const int d15 = q15_of(decay, 15), nbq = -q15_of(beta, 15);
    bool bad = false;
    // Pass A.
    for (int j = warp; j < hv; j += kDnIntWarps) {
        long long dot = 0;
        for (int c = lane; c < hk; c += 32) dot += (long long)M[(size_t)j * hk + c] * (long long)k16[c];
        dot = warp_sum_ll(dot);
        if (lane == 0) {
            const long long dot_r = arith_shift_ll(dot, shift_a);
            bad |= llabs_(dot_r) >= (1ll << 31);
            const long long ddr = (dot_r * d15) >> 15;
            const long long nv = -lround_away((double)A.v[(size_t)h * hv + j] * (double)(1 << kDnDeltaFrac));
            bad |= llabs_(nv) >= (1ll << 31);
            const long long delta = ((ddr + nv) * nbq) >> 15;
            dl[j] = delta;
            atomicMax(&maxD_s, (unsigned long long)llabs_(delta));
        }
    }
    __syncthreads();
    if (tid == 0) {  // the exponent ratchet and the pass-B constants, model/deltanet.py:82-97
        const int maxM = need_max ? (int)maxM_s : A.maxM[h];
        const double kmax = ldexp((double)k16max_s, ek);
        const double t = ((double)maxM * (double)decay +
                          (double)maxD_s * ldexp(1.0, -kDnDeltaFrac) * kmax * ldexp(1.0, -eM)) / kDnStateLim;
        int n = 0;
        if (t > 1.0) {  // ceil(log2(t)): t = f 2^e with f in [0.5, 1)
            int e;
            const double f = frexp(t, &e);
            n = f == 0.5 ? e - 1 : e;
        }
        eM2_s = eM + n;
        sh_s = eM + n + 7 - ek;
        d15n_s = q15_of(decay, 15 - n);
        rnd_s = sh_s > 0 ? (1ll << (sh_s - 1)) : 0ll;
    }
    __syncthreads();
    const int sh = sh_s, d15n = d15n_s, eM2 = eM2_s;
    for (int j = tid; j < hv; j += kDnIntThreads) {  // delta_s = (8 delta + rnd) shifted by -sh
        const long long d8 = 8 * dl[j] + rnd_s;
        bad |= llabs_(d8) >= (1ll << 31);
        const long long ds = arith_shift_ll(d8, -sh);
        bad |= llabs_(ds) >= (1ll << 16);
        dl[j] = ds;
    }
    __syncthreads();
    // Pass B.
    const double osc = ldexp(1.0, eM2 + eq_s + kDnOShift);
    for (int j = warp; j < hv; j += kDnIntWarps) {
        const long long ds = dl[j];
        long long o = 0;
        unsigned mm = 0u;
        for (int c = lane; c < hk; c += 32) {
            int16_t *pm = M + (size_t)j * hk + c;
            const long long nm = rne_shift15((long long)*pm * d15n + ds * (long long)k16[c]);
            bad |= llabs_(nm) > 32767;
            *pm = (int16_t)nm;
            mm = max(mm, (unsigned)llabs_(nm));
            o += nm * (long long)q16[c];
        }
        o = warp_sum_ll(o);
        mm = __reduce_max_sync(0xffffffffu, mm);
        if (lane == 0) {
            atomicMax(&maxM2_s, mm);
            const long long o_r = o >> kDnOShift;
            bad |= llabs_(o_r) >= (1ll << 31);
            A.out[(size_t)h * hv + j] = __double2float_rn((double)o_r * osc);
        }
    }
    if (bad) atomicOr(&bad_s, 1);
    __syncthreads();
    if (tid == 0) {
        A.eM[h] = eM2;
        A.maxM[h] = (int)maxM2_s;
        if (bad_s) atomicOr(err, TRX_DEV_OVERFLOW);
    }
}

trx_status launch_dn_int(const DnIntArgs &A, uint32_t *err, cudaStream_t st) {
    if (A.hk < 1 || A.hk > kDnIntMaxHk || A.hv < 1 || A.hv > kDnIntMaxHv || A.nh < 1) return TRX_ERR_UNSUPPORTED;
    return note_cuda(launch_kernel(dn_int_kernel, dim3(A.nh), dim3(kDnIntThreads), 0, st, A, err));
}

}  // namespace trx
