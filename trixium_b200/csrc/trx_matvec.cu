// Ternary matvec kernels for B200 (sm_100a): the TriXium engine's group-128 matvec over the
// converter's row packets (2-bit and 5-trit codes), bit-exact with model/bitexact.py:101-119,
// with the firmware's float wrapper (quantise -> engine -> scale, firmware/infer_float.c:398)
// fused in, and the fp-mode projection of model/fastref.py:103-125.
//
// Work decomposition:
//  * Persistent: one CTA of 16 warps per SM, a contiguous range of rows (of one or more jobs).
//  * A row is split into nck slabs of CW groups (CW a power of two <= 32; one slab when the row
//    has <= 32 groups).  A warp owns one slab for a whole job: each lane owns one group of it, and
//    the activation's permuted int8 words for that group live in the lane's registers, so the
//    inner loop reads only codes (and, for trit5, the byte LUT) from shared memory.
//  * A block is BR consecutive rows of the warp's slab.  Every warp streams its own blocks
//    global -> shared through a private D-deep ring with 16-byte cp.async copies (coalesced:
//    consecutive lanes copy consecutive 16-byte chunks of a row packet), cp.async.wait_group
//    tracking completion -- no producer warp, no CTA-wide barrier inside the job.  Measured on
//    B200, 1-D bulk (TMA) copies complete one after another per SM with ~0.8 us exposed each and a
//    227 KB ring cannot hold enough of them in flight while blocks are decoded; per-warp rings keep
//    ~100 KB in flight per SM.
//  * Group sums are exact int32 (dp4a / dp2a); the scale/shift contribution is int64, summed over
//    the slot's lanes with two 32-bit warp reductions of an exact hi/lo split.  A whole row's sum
//    is finished by the slot's leader lane (>> R, overflow checks, float scaling, epilogue); a row
//    split over slabs is summed with 64-bit atomics in a self-cleaning global accumulator and
//    finished by the last slab to arrive.
//  * trit5 decode: a 256-entry byte LUT (digits d0, d1, d2 and d3+3*d4 as bytes), replicated 32x
//    (one copy per lane, so lookups never bank-conflict), addressed with one PRMT per byte.
//    dp4a adds d0*x0+d1*x1+d2*x2+(d3+3d4)*x3; the d4 correction d4*(x4-3*x3) is a dp2a on
//    16-bit activation pairs, d4 = (d3+3d4)/3 computed for four bytes at once.
//  * 2-bit decode: four masks per word; dp4a on (code << 2p) bytes into four accumulators.
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

// Launch shape and shared-memory plan --------------------------------------------------------------
constexpr int kWarpsMv = 16;
constexpr int kMvThreads = kWarpsMv * 32;
constexpr int kLutWords = 256 * 64;              // 256 entries x 256-byte stride (32 replicas used)
constexpr int kLutBytes = kLutWords * 4;         // 64 KiB
constexpr int kXWordsT5 = 40;                    // 26 dp4a words + 14 dp2a words per group
constexpr int kXWords2b = 32;
constexpr int kSmemMax = 227 * 1024;
constexpr int kMaxDepth = 8;                     // blocks in flight per warp (ring slots)
constexpr int kRingTarget = 14 * 1024;           // bytes of ring per warp to aim for
constexpr int kMaxNpb = 4;

// Geometry of one launch, derived on the host (plan_matvec) and passed by value.
struct MvGeom {
    int G;        // groups per row
    int CW;       // groups per slab = lanes per slot (power of two <= 32)
    int nck;      // slabs per row
    int RPW;      // rows a warp decodes at once (32 / CW slots)
    int NPB;      // passes (of RPW rows) per block
    int BR;       // rows per block = RPW * NPB
    int D;        // ring depth (blocks)
    int rb;       // row packet bytes in global memory
    int sbytes;   // scale-region bytes of a packet
    int s_off, s_len;   // slab c's scales: packet bytes [s_off*c, +s_len) (s_len 16-byte rounded)
    int c_off, c_len;   // slab c's codes: packet bytes [sbytes + c_off*c, +c_len)
    int srow;     // bytes of one row in the ring (s_len + c_len, or rb for a single slab)
    int slot_bytes;     // BR * srow * nw
    int nbj;      // blocks per job (segments are whole blocks, except a single segment's tail)
    int nw;       // tensors per block (2 for SwiGLU)
    int xwords;   // permuted activation words per group
    int smem;     // dynamic shared bytes
};

// Quantisation helpers ----------------------------------------------------------------------------
// 2^k as an fp32, exact for k in [-149, 127] (the scale of the power-of-two quantiser).
__device__ __forceinline__ float pow2f(int k) { return ldexpf(1.0f, k); }

// The value the quantiser sees at position k: x[k], or the RMS-normalised x[k]*r*w[k].
__device__ __forceinline__ float prologue_value(const float *x, const float *w, float r, int k) {
    float v = __ldg(x + k);
    if (w) v = __fmul_rn(__fmul_rn(v, r), __ldg(w + k));
    return v;
}

__device__ __forceinline__ int8_t quant_one(float v, float inv) {
    int q = lround_mirror(__fmul_rn(v, inv));
    q = q > 127 ? 127 : (q < -127 ? -127 : q);
    return (int8_t)q;
}

// Canonical sum of squares (model/mirror.py:576-591; doc/units.md "Sum of squares"): 64
// sequential fp32 partials in increasing index order, then the halving tree.  All threads call it.
__device__ float block_sumsq64(const float *x, int n, float *red64) {
    const int ct = threadIdx.x;
    if (ct < 64) {
        float p = 0.f;
        for (int i = ct; i < n; i += 64) {
            const float v = __ldg(x + i);
            p = __fadd_rn(p, __fmul_rn(v, v));
        }
        red64[ct] = p;
    }
    __syncthreads();
    for (int w = 32; w >= 1; w >>= 1) {
        if (ct < w) red64[ct] = __fadd_rn(red64[ct], red64[ct + w]);
        __syncthreads();
    }
    const float ss = red64[0];
    __syncthreads();
    return ss;
}

// Build the permuted int8 activation of one job in shared memory (all threads).
// q8: K bytes, xp: G*xwords words, xsum: G ints.  Returns e8.
template <int KIND>
__device__ int build_activation(const float *x, const int8_t *x8g, const float *nw, float eps, int K, int8_t *q8,
                                uint32_t *xp, int *xsum, uint32_t *amax_s, float *red64) {
    const int ct = threadIdx.x;
    const int nt = blockDim.x;
    int e8 = 0;
    if (x8g) {
        for (int k = ct; k < K; k += nt) q8[k] = x8g[k];
    } else {
        float r = 0.f;
        if (nw) {
            const float ss = block_sumsq64(x, K, red64);
            r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
        }
        if (ct == 0) *amax_s = 0u;
        __syncthreads();
        uint32_t m = 0;
        for (int k = ct; k < K; k += nt) {
            const uint32_t a = __float_as_uint(fabsf(prologue_value(x, nw, r, k)));
            m = a > m ? a : m;
        }
        m = __reduce_max_sync(0xffffffffu, m);
        if ((ct & 31) == 0) atomicMax(amax_s, m);
        __syncthreads();
        const uint32_t amax = *amax_s;
        if (amax == 0u) {
            for (int k = ct; k < K; k += nt) q8[k] = 0;
        } else {
            e8 = frexp_exp(__uint_as_float(amax)) - 7;
            const float inv = pow2f(-e8);
            for (int k = ct; k < K; k += nt) q8[k] = quant_one(prologue_value(x, nw, r, k), inv);
        }
    }
    __syncthreads();
    const int G = K / 128;
    if (KIND == TRX_KIND_TERNARY5) {
        // Per group: words 0..25 = bytes (x[5i], x[5i+1], x[5i+2], x[5i+3]);
        // words 26..39 = 16-bit pairs (y[2j], y[2j+1]) with y[i] = x[5i+4] - 3*x[5i+3];
        // lanes 128/129 (digits 3/4 of byte 25) see x = 0.
        for (int idx = ct; idx < G * kXWordsT5; idx += nt) {
            const int g = idx / kXWordsT5, j = idx % kXWordsT5;
            const int8_t *qg = q8 + g * 128;
            uint32_t w = 0;
            if (j < 26) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int l = 5 * j + k;
                    const uint32_t b = l < 128 ? (uint32_t)(uint8_t)qg[l] : 0u;
                    w |= b << (8 * k);
                }
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = 2 * (j - 26) + h;
                    int y = 0;
                    if (i < 26) {
                        const int l3 = 5 * i + 3, l4 = 5 * i + 4;
                        const int x3 = l3 < 128 ? qg[l3] : 0, x4 = l4 < 128 ? qg[l4] : 0;
                        y = x4 - 3 * x3;
                    }
                    w |= ((uint32_t)y & 0xffffu) << (16 * h);
                }
            }
            xp[idx] = w;
        }
    } else {
        // Per group: word (w*4 + p) = bytes x[16w + 4b + p], b = 0..3.
        for (int idx = ct; idx < G * kXWords2b; idx += nt) {
            const int g = idx / kXWords2b, j = idx % kXWords2b;
            const int wq = j >> 2, p = j & 3;
            const int8_t *qg = q8 + g * 128;
            uint32_t w = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) w |= (uint32_t)(uint8_t)qg[16 * wq + 4 * b + p] << (8 * b);
            xp[idx] = w;
        }
    }
    // Group sums of x8: one warp per group.
    for (int g = ct >> 5; g < G; g += nt >> 5) {
        const int lane = ct & 31;
        const int8_t *qg = q8 + g * 128 + 4 * lane;
        int s = (int)qg[0] + (int)qg[1] + (int)qg[2] + (int)qg[3];
        s = __reduce_add_sync(0xffffffffu, s);
        if (lane == 0) xsum[g] = s;
    }
    __syncthreads();
    return e8;
}

// Group sums -----------------------------------------------------------------------------------------
// trit5: the 26 code bytes of one group start at `p` (2-byte aligned).  Returns sum(digit*x).
__device__ __forceinline__ int gsum_t5(const uint8_t *p, int odd, const char *lut, uint32_t lane4,
                                       const uint32_t *xa, const uint32_t *yy) {
    const uint32_t *wp = reinterpret_cast<const uint32_t *>(p - 2 * odd);
    uint32_t w[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) w[i] = wp[i];
    const uint32_t sel = odd ? 0x5432u : 0x3210u;
    int acc[4] = {0, 0, 0, 0};  // independent chains (byte position within a quad)
#pragma unroll
    for (int q = 0; q < 7; ++q) {
        const uint32_t W = __byte_perm(w[q], q < 6 ? w[q + 1] : w[q], sel);
        const int nb = q < 6 ? 4 : 2;
        uint32_t E[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (i < nb) {
                // a = byte * 256 + lane * 4: this lane's replica of the entry, no bank conflict.
                const uint32_t a = __byte_perm(W, lane4, 0x5504u | (i << 4));
                E[i] = *reinterpret_cast<const uint32_t *>(lut + a);
                acc[i] = dp4a_ss(E[i], xa[4 * q + i], acc[i]);
            }
        }
        if (nb == 4) {
            const uint32_t d01 = __byte_perm(E[0], E[1], 0x0073u);
            const uint32_t d23 = __byte_perm(E[2], E[3], 0x0073u);
            const uint32_t D = ((__byte_perm(d01, d23, 0x5410u) * 11u) >> 5) & 0x03030303u;
            acc[q & 3] = dp2a_lo(yy[2 * q], D, acc[q & 3]);
            acc[(q + 2) & 3] = dp2a_hi(yy[2 * q + 1], D, acc[(q + 2) & 3]);
        } else {
            const uint32_t D = ((__byte_perm(E[0], E[1], 0x0073u) * 11u) >> 5) & 0x03030303u;
            acc[3] = dp2a_lo(yy[2 * q], D, acc[3]);
        }
    }
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// 2-bit: the 32 code bytes of one group at `p` (16-byte aligned).  Returns sum(code*x).
__device__ __forceinline__ int gsum_2b(const uint8_t *p, const uint32_t *xw) {
    const uint4 c0 = reinterpret_cast<const uint4 *>(p)[0];
    const uint4 c1 = reinterpret_cast<const uint4 *>(p)[1];
    const uint32_t c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        a0 = dp4a_us(c[w] & 0x03030303u, xw[4 * w + 0], a0);
        a1 = dp4a_us(c[w] & 0x0c0c0c0cu, xw[4 * w + 1], a1);
        a2 = dp4a_us(c[w] & 0x30303030u, xw[4 * w + 2], a2);
        a3 = dp4a_us(c[w] & 0xc0c0c0c0u, xw[4 * w + 3], a3);
    }
    return a0 + (a1 >> 2) + (a2 >> 4) + (a3 >> 6);
}

// (gs*m11) shifted by e16+B as int64 (model/bitexact.py:111-115).  Common case: a normal fp16
// scale with 0 <= e16+B <= 19, where m11 << (e16+B) = scale * 2^B is an integer below 2^30, so the
// contribution is one wide multiply by F2I(fp32(scale) * 2^B) (both steps exact).  Otherwise the
// general floor/left shift.
__device__ __forceinline__ long long contrib_fast(int gs, uint32_t sbits, int B, float pow2B) {
    const int E = (sbits >> 10) & 31;
    const int sh = E - 25 + B;
    if (E != 0 && (unsigned)sh <= 19u)
        return (long long)gs * (long long)__float2int_rz(__fmul_rn(__half2float(__ushort_as_half((unsigned short)sbits)), pow2B));
    return group_contrib(gs, sbits, B);
}

// Exact int64 sum over the CW lanes of this lane's slot (CW a power of two <= 32), without
// divergence: c = hi*2^24 + lo (lo in [0, 2^24)); 32-bit warp reductions of the slot-masked
// parts (CW >= 16), or xor-shuffles (CW < 16).
__device__ __forceinline__ long long slot_sum64(long long c, int CW, int lane) {
    if (CW >= 16) {
        const uint32_t lo = (uint32_t)(c & 0xffffffll);
        const int hi = (int)(c >> 24);
        if (CW == 32) {
            const uint32_t slo = __reduce_add_sync(0xffffffffu, lo);
            const int shi = __reduce_add_sync(0xffffffffu, hi);
            return ((long long)shi << 24) + (long long)slo;
        }
        const bool upper = lane >= 16;
        const uint32_t lo1 = __reduce_add_sync(0xffffffffu, upper ? lo : 0u);
        const int hi1 = __reduce_add_sync(0xffffffffu, upper ? hi : 0);
        const uint32_t lo0 = __reduce_add_sync(0xffffffffu, upper ? 0u : lo);
        const int hi0 = __reduce_add_sync(0xffffffffu, upper ? 0 : hi);
        return upper ? ((long long)hi1 << 24) + (long long)lo1 : ((long long)hi0 << 24) + (long long)lo0;
    }
    for (int o = CW >> 1; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    return c;
}

// The float epilogue value of one finished row (the firmware's int32 -> float scaling).
__device__ __forceinline__ float row_float(long long acc, int R, int e8, int B) {
    const int res = (int)(acc >> R);
    return __fmul_rn((float)res, pow2f(e8 + R - B));
}

__device__ __forceinline__ bool acc_bad(long long a, int R) {
    const long long r = a >> R;
    return a >= (1ll << 47) || a <= -(1ll << 47) || r >= (1ll << 31) || r <= -(1ll << 31);
}

__device__ __forceinline__ float silu_f32(float g) {
    // x / (1 + exp(-x)) in fp32 (model/mirror.py:713, mathematical profile).
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}


// Row output --------------------------------------------------------------------------------------
// Segment s of a launch holds rows [seg_start(s), seg[s].row_end) of the packed tensor.
__device__ __forceinline__ int seg_start(const MvJobs &J, int s) { return s ? J.seg[s - 1].row_end : 0; }

// Per-block output context (uniform over a block: blocks never straddle segments).
struct RowOut {
    int R, R2, B;
    float sc, sc2;         // 2^(e8 + R - B) of the tensor(s)
    char *y;               // output of the segment's row 0 (this job)
    const float *resid;    // residual of the segment's row 0, or nullptr
};

__device__ __forceinline__ RowOut row_out(const MvJobs &J, int job, int s, int e8) {
    const MvSeg &S = J.seg[s];
    RowOut o;
    o.R = S.R;
    o.B = S.B;
    o.R2 = J.R2;
    o.sc = pow2f(e8 + S.R - S.B);
    o.sc2 = pow2f(e8 + J.R2 - J.B2);
    o.y = S.y ? reinterpret_cast<char *>(S.y) + (uint64_t)job * J.y_stride * 4 : nullptr;
    o.resid = S.resid;
    return o;
}

// Finish one row (srow: index within its segment) from its int64 sum(s): >> R, the overflow
// checks of model/bitexact.py:116,118, then the launch's output.  SwiGLU: a = gate, a2 = up.
// Returns the row's argmax key (0 when the launch keeps no argmax).
__device__ __forceinline__ unsigned long long finish_row(const MvJobs &J, const RowOut &o, int row, int srow,
                                                         long long a, long long a2, uint32_t *err) {
    bool bad = acc_bad(a, o.R);
    unsigned long long key = 0ull;
    if (J.out == OUT_I32) {
        reinterpret_cast<int *>(o.y)[srow] = (int)(a >> o.R);
    } else if (J.out == OUT_F32) {
        float v = __fmul_rn((float)(int)(a >> o.R), o.sc);
        if (o.resid) v = __fadd_rn(o.resid[srow], v);
        if (o.y) reinterpret_cast<float *>(o.y)[srow] = v;
        if (J.argmax) key = argmax_key(v, (uint32_t)row);
    } else {  // OUT_SWIGLU
        bad = bad || acc_bad(a2, o.R2);
        const float gv = __fmul_rn((float)(int)(a >> o.R), o.sc);
        const float uv = __fmul_rn((float)(int)(a2 >> o.R2), o.sc2);
        reinterpret_cast<float *>(o.y)[srow] = __fmul_rn(silu_f32(gv), uv);
    }
    if (bad) atomicOr(err, TRX_DEV_OVERFLOW);
    return key;
}

// Warp-wide max of argmax keys, one atomic per warp.
__device__ __forceinline__ void argmax_commit(const MvJobs &J, int job, unsigned long long best, int lane) {
    for (int o = 16; o; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    if (lane == 0 && best) atomicMax(J.argmax + job, best);
}

// cp.async (16-byte, L2 only) -----------------------------------------------------------------------
__device__ __forceinline__ void cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_wait_n(int n) {  // n <= kMaxDepth - 1
    switch (n) {
        case 0: cp_wait<0>(); break;
        case 1: cp_wait<1>(); break;
        case 2: cp_wait<2>(); break;
        case 3: cp_wait<3>(); break;
        case 4: cp_wait<4>(); break;
        case 5: cp_wait<5>(); break;
        case 6: cp_wait<6>(); break;
        default: cp_wait<7>(); break;
    }
}

// Issue the copies of one block (rows [r, r+nr) of slab c) into ring slot `dst`.
__device__ __forceinline__ void issue_block(const MvJobs &J, const MvGeom &M, int job, int r, int nr, int c,
                                            unsigned char *dst, int lane) {
    const uint64_t jbase = (uint64_t)job * J.w_stride;
    for (int w = 0; w < M.nw; ++w) {
        const uint8_t *base = (w ? J.w2 : J.w) + jbase;
        unsigned char *d = dst + (size_t)w * M.BR * M.srow;
        if (M.nck == 1) {  // whole rows: one contiguous range
            const int n16 = nr * M.rb / 16;
            const uint8_t *src = base + (uint64_t)r * M.rb;
            for (int i = lane; i < n16; i += 32) cp16(d + 16 * i, src + 16 * i);
        } else {           // per row: the slab's scales, then its codes
            const int ns = M.s_len / 16, nc = M.c_len / 16, per = ns + nc;
            for (int i = lane; i < nr * per; i += 32) {
                const int rr = i / per, j = i - rr * per;
                const uint8_t *row = base + (uint64_t)(r + rr) * M.rb;
                const uint8_t *src = j < ns ? row + M.s_off * c + 16 * j : row + M.sbytes + M.c_off * c + 16 * (j - ns);
                cp16(d + rr * M.srow + 16 * j, src);
            }
        }
    }
}

// The matvec kernel ---------------------------------------------------------------------------------
template <int KIND>
__global__ void __launch_bounds__(kMvThreads, 1) tmv_kernel(MvJobs J, MvGeom M, const uint32_t *lut_g, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    if (J.skip && *J.skip) return;

    // Carve shared memory (must match plan_matvec).
    unsigned char *p = smem;
    char *lut = nullptr;
    if (KIND == TRX_KIND_TERNARY5) {
        lut = reinterpret_cast<char *>(p);
        p += kLutBytes;
    }
    unsigned char *const ring = p + (size_t)warp * M.D * M.slot_bytes;
    p += (size_t)kWarpsMv * M.D * M.slot_bytes;
    long long *const wred = reinterpret_cast<long long *>(p) + warp * 2 * M.BR;  // this warp's row sums
    p += kWarpsMv * 2 * M.BR * 8;
    uint32_t *const xp = reinterpret_cast<uint32_t *>(p);
    p += M.G * M.xwords * 4;
    int *const xsum = reinterpret_cast<int *>(p);
    p += ((M.G * 4 + 15) / 16) * 16;
    float *const red64 = reinterpret_cast<float *>(p);
    p += 64 * 4;
    uint32_t *const amax_s = reinterpret_cast<uint32_t *>(p);
    p += 16;
    int8_t *const q8 = reinterpret_cast<int8_t *>(p);

    // This CTA's share of the (job, block) space; a block is BR rows of one segment.
    const long long total = (long long)J.njobs * M.nbj;
    const long long q0 = (long long)blockIdx.x * total / gridDim.x;
    const long long q1 = (long long)(blockIdx.x + 1) * total / gridDim.x;
    if (q0 >= q1) return;

    if (KIND == TRX_KIND_TERNARY5) {  // the trit5 LUT (replicated, 256-byte stride)
        const uint4 *src = reinterpret_cast<const uint4 *>(lut_g);
        uint4 *dst = reinterpret_cast<uint4 *>(lut);
        for (int i = tid; i < kLutBytes / 16; i += blockDim.x) dst[i] = src[i];
    }

    // Warp -> slab(s) and its share of the blocks.
    const int CW = M.CW, nck = M.nck;
    int c0, nsub, sub;
    if (nck <= kWarpsMv) {
        c0 = warp % nck;
        sub = warp / nck;
        nsub = (kWarpsMv - c0 + nck - 1) / nck;
    } else {
        c0 = warp;
        sub = 0;
        nsub = 1;
    }
    const int slot = lane / CW;              // which of the RPW rows of a pass
    const int gl = lane % CW;                // group within the slab
    const bool leader = gl == 0;
    const uint32_t lane4 = (uint32_t)lane * 4u;
    uint32_t xr[kXWordsT5 > kXWords2b ? kXWordsT5 : kXWords2b];

    for (long long q = q0; q < q1;) {
        const int job = (int)(q / M.nbj);
        const long long jb0 = (long long)job * M.nbj;
        const int pb0 = (int)(q - jb0);                                   // first block of the piece
        const int pb1 = (int)min((long long)M.nbj, q1 - jb0);             // end block of the piece
        q = jb0 + pb1;
        __syncthreads();  // the previous job's activation is no longer read
        const float *xj = J.x ? J.x + (uint64_t)job * J.x_stride : nullptr;
        const int8_t *x8j = J.x8 ? J.x8 + (uint64_t)job * J.x_stride : nullptr;
        const int e8 = build_activation<KIND>(xj, x8j, J.norm_w, J.eps, J.cols, q8, xp, xsum, amax_s, red64);
        unsigned long long best = 0ull;
        const int nmine = pb1 - pb0 > sub ? (pb1 - pb0 - sub + nsub - 1) / nsub : 0;  // this warp's blocks

        for (int c = c0; c < nck; c += kWarpsMv) {
            const int g = c * CW + gl;
            const bool gvalid = g < M.G;
            if (gvalid) {
#pragma unroll
                for (int i = 0; i < (KIND == TRX_KIND_TERNARY5 ? kXWordsT5 : kXWords2b); ++i)
                    xr[i] = xp[g * M.xwords + i];
            }
            const int xs = gvalid ? xsum[g] : 0;
            const int gi = nck == 1 ? g : gl;  // group index inside a ring row
            const int code_off = (nck == 1 ? M.sbytes : M.s_len) + (KIND == TRX_KIND_TERNARY5 ? 26 : 32) * gi;
            const int lane_row = slot * M.srow;  // this lane's row within a pass
            // Prime the ring with the first D-1 blocks.
            for (int d = 0; d < M.D - 1; ++d) {
                if (d < nmine) {
                    const int r = (pb0 + sub + d * nsub) * M.BR;
                    issue_block(J, M, job, r, min(M.BR, J.rows - r), c, ring + (size_t)d * M.slot_bytes, lane);
                }
                cp_commit();
            }
            int rs = M.D - 1, cs = 0, cur_seg = -1, Bs = 0, sb0 = 0;
            float p2B = 1.f;
            const float p2B2 = pow2f(J.B2);
            RowOut ro{};
            for (int j = 0; j < nmine; ++j) {
                if (j + M.D - 1 < nmine) {
                    const int r = (pb0 + sub + (j + M.D - 1) * nsub) * M.BR;
                    issue_block(J, M, job, r, min(M.BR, J.rows - r), c, ring + (size_t)rs * M.slot_bytes, lane);
                }
                cp_commit();
                rs = rs + 1 == M.D ? 0 : rs + 1;
                cp_wait_n(M.D - 1);
                __syncwarp();
                const int r = (pb0 + sub + j * nsub) * M.BR;
                const int nr = min(M.BR, J.rows - r);
                {  // segment of this block (blocks never straddle segments)
                    int sg = 0;
#pragma unroll
                    for (int i = 0; i < kMaxSegs - 1; ++i) sg += (i < J.nseg - 1 && r >= J.seg[i].row_end) ? 1 : 0;
                    if (sg != cur_seg) {
                        cur_seg = sg;
                        ro = row_out(J, job, sg, e8);
                        Bs = ro.B;
                        p2B = pow2f(Bs);
                        sb0 = seg_start(J, sg);
                    }
                }
                const unsigned char *blk = ring + (size_t)cs * M.slot_bytes + lane_row;
                for (int pass = 0; pass < M.NPB; ++pass) {
                    const int rr = pass * M.RPW + slot;
                    auto unit = [&](int w) -> long long {
                        long long cc = 0;
                        if (gvalid) {  // rows past nr decode stale slot bytes; masked below
                            const unsigned char *row = blk + (w * M.BR + pass * M.RPW) * M.srow;
                            const uint32_t sbits = reinterpret_cast<const uint16_t *>(row)[gi];
                            int gs;
                            if (KIND == TRX_KIND_TERNARY5)
                                gs = gsum_t5(row + code_off, gi & 1, lut, lane4, xr, xr + 26) - xs;
                            else
                                gs = gsum_2b(row + code_off, xr) - xs;
                            cc = contrib_fast(gs, sbits, w ? J.B2 : Bs, w ? p2B2 : p2B);
                            cc = rr < nr ? cc : 0ll;
                        }
                        return slot_sum64(cc, CW, lane);
                    };
                    const long long sum0 = unit(0);
                    if (leader) wred[rr] = sum0;
                    if (M.nw == 2) {
                        const long long sum1 = unit(1);
                        if (leader) wred[M.BR + rr] = sum1;
                    }
                }
                __syncwarp();  // every lane is done with the slot; the row sums are in wred
                cs = cs + 1 == M.D ? 0 : cs + 1;
                // Finish the block's rows, one lane per row.
                for (int rr = lane; rr < nr; rr += 32) {
                    const int row = r + rr;
                    const long long a = wred[rr];
                    const long long a2 = M.nw == 2 ? wred[M.BR + rr] : 0ll;
                    if (nck == 1) {
                        const unsigned long long k = finish_row(J, ro, row, row - sb0, a, a2, err);
                        best = k > best ? k : best;
                    } else {
                        // Split row: add this slab's sums; the last slab to arrive finishes it.
                        const uint64_t ix = (uint64_t)job * J.rows + row;
                        unsigned long long *acc = J.acc + 2 * ix;
                        atomicAdd(acc, (unsigned long long)a);
                        if (M.nw == 2) atomicAdd(acc + 1, (unsigned long long)a2);
                        __threadfence();
                        if (atomicAdd(J.cnt + ix, 1u) == (unsigned)(nck - 1)) {
                            __threadfence();
                            const long long t = (long long)atomicExch(acc, 0ull);
                            const long long t2 = M.nw == 2 ? (long long)atomicExch(acc + 1, 0ull) : 0ll;
                            J.cnt[ix] = 0u;
                            const unsigned long long k = finish_row(J, ro, row, row - sb0, t, t2, err);
                            best = k > best ? k : best;
                        }
                    }
                }
                __syncwarp();  // wred is reused by the next block
            }
            cp_wait<0>();
            __syncwarp();
        }
        if (J.argmax) argmax_commit(J, job, best, lane);
    }
}

// fp-mode kernel (model/fastref.py:103-125): thread per (row, group); x fp32 in shared memory;
// per-group fp32 sums of (code-1)*x, times the fp32 scale, reduced over groups in group order.
template <int KIND>
__global__ void __launch_bounds__(256) tmv_fp_kernel(MvJobs J, int TR, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);
    float *part = xs + J.cols;  // [TR][G+1]
    const int G = J.cols / 128, K = J.cols;
    const int sbytes = (G + 15) / 16 * 32;
    const int rb = sbytes + ((KIND == TRX_KIND_TERNARY5 ? 26 : 32) * G + 31) / 32 * 32;
    for (int k = threadIdx.x; k < K; k += blockDim.x) xs[k] = J.x[k];
    __syncthreads();
    const int units = TR * G;
    for (int r0 = blockIdx.x * TR; r0 < J.rows; r0 += gridDim.x * TR) {
        const int nr = min(TR, J.rows - r0);
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
            const int rr = u / G, g = u % G;
            if (rr >= nr) continue;
            const uint8_t *row = J.w + (uint64_t)(r0 + rr) * rb;
            const float *xg = xs + g * 128;
            float s = 0.f;
            if (KIND == TRX_KIND_TERNARY5) {
                const uint8_t *cb = row + sbytes + 26 * g;
                for (int i = 0; i < 26; ++i) {
                    uint32_t b = cb[i];
                    for (int k = 0; k < 5; ++k) {
                        const int l = 5 * i + k;
                        const int d = (int)(b % 3u);
                        b /= 3u;
                        if (l < 128) s = __fadd_rn(s, __fmul_rn((float)(d - 1), xg[l]));
                    }
                }
            } else {
                const uint8_t *cb = row + sbytes + 32 * g;
                for (int l = 0; l < 128; ++l) {
                    const int c = (cb[l >> 2] >> (2 * (l & 3))) & 3;
                    s = __fadd_rn(s, __fmul_rn((float)(c - 1), xg[l]));
                }
            }
            const float sc = __half2float(reinterpret_cast<const __half *>(row)[g]);
            part[rr * (G + 1) + g] = __fmul_rn(s, sc);
        }
        __syncthreads();
        for (int rr = threadIdx.x; rr < nr; rr += blockDim.x) {
            float a = 0.f;
            for (int g = 0; g < G; ++g) a = __fadd_rn(a, part[rr * (G + 1) + g]);
            reinterpret_cast<float *>(J.seg[0].y)[r0 + rr] = a;
        }
        __syncthreads();
    }
}

// Standalone quantiser (trx_quantize_pow2): one CTA, grid-stride.
__global__ void __launch_bounds__(1024) quantize_kernel(const float *x, int n, int8_t *x8, int *e8_out) {
    __shared__ uint32_t amax_s;
    if (threadIdx.x == 0) amax_s = 0;
    __syncthreads();
    uint32_t m = 0;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const uint32_t a = __float_as_uint(fabsf(x[k]));
        m = a > m ? a : m;
    }
    for (int o = 16; o; o >>= 1) {
        const uint32_t o2 = __shfl_xor_sync(0xffffffffu, m, o);
        m = o2 > m ? o2 : m;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(&amax_s, m);
    __syncthreads();
    const uint32_t amax = amax_s;
    const int e8 = amax ? frexp_exp(__uint_as_float(amax)) - 7 : 0;
    const float inv = pow2f(-e8);
    for (int k = threadIdx.x; k < n; k += blockDim.x) x8[k] = amax ? quant_one(x[k], inv) : (int8_t)0;
    if (threadIdx.x == 0) *e8_out = e8;
}

// Validation of trit5 bytes (> 242 is invalid).
__global__ void validate_t5_kernel(const uint8_t *w, int rows, int rb, int sbytes, int G, uint32_t *err) {
    const int cb = 26 * G;
    const long long total = (long long)rows * cb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / cb, c = i % cb;
        if (w[r * rb + sbytes + c] > 242) atomicOr(err, TRX_DEV_BADBYTE);
    }
}

__global__ void build_lut_kernel(uint32_t *lut) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // i over 256 * 64
    if (i < kLutWords) {
        const int b = i / 64, l = i % 64;
        lut[i] = l < 32 ? trit5_lut_entry((uint32_t)b) : 0u;
    }
}



// Host side ------------------------------------------------------------------------------------------
static thread_local cudaError_t g_last_cuda = cudaSuccess;

trx_status note_cuda(cudaError_t e) {
    if (e == cudaSuccess) return TRX_OK;
    g_last_cuda = e;
    return TRX_ERR_CUDA;
}

const char *last_cuda_error() { return cudaGetErrorString(g_last_cuda); }

static int round_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

// Plan a launch.  Rows with more than 32 groups are split into equal slabs of CW groups (a power
// of two >= 8 dividing G, so every slab starts on a 16-byte boundary); others are one slab.
bool plan_matvec(const MvJobs &J, int cols, int kind, int nw, MvGeom &M) {
    M.G = cols / 128;
    if (M.G <= 32) {
        M.CW = round_pow2(M.G);
        M.nck = 1;
    } else {
        int cw = M.G & -M.G;
        if (cw > 32) cw = 32;
        if (cw < 8) return false;  // K > 4096 must be a multiple of 1024
        M.CW = cw;
        M.nck = M.G / cw;
    }
    M.RPW = 32 / M.CW;
    M.sbytes = (M.G + 15) / 16 * 32;
    const int gb = kind == TRX_KIND_TERNARY5 ? 26 : 32;
    M.rb = M.sbytes + (gb * M.G + 31) / 32 * 32;
    M.nw = nw;
    M.xwords = kind == TRX_KIND_TERNARY5 ? kXWordsT5 : kXWords2b;
    if (M.nck == 1) {
        M.s_off = M.s_len = M.c_off = M.c_len = 0;
        M.srow = M.rb;
    } else {
        M.s_off = 2 * M.CW;
        M.s_len = (2 * M.CW + 15) / 16 * 16;
        M.c_off = gb * M.CW;
        M.c_len = (gb * M.CW + 15) / 16 * 16;
        M.srow = M.s_len + M.c_len;
    }
    // Passes per block: blocks of about 4 KiB (2 KiB beside the trit5 LUT), and in a launch of
    // several segments, a block size that divides every segment.
    int npb = (kind == TRX_KIND_TERNARY5 ? 2048 : 4096) / (M.RPW * M.srow * nw);
    npb = npb < 1 ? 1 : (npb > kMaxNpb ? kMaxNpb : npb);
    for (; npb > 1; --npb) {
        bool ok = true;
        for (int i = 0; i < J.nseg - 1 && J.nseg > 1; ++i)
            if ((J.seg[i].row_end - (i ? J.seg[i - 1].row_end : 0)) % (M.RPW * npb)) ok = false;
        if (ok) break;
    }
    M.NPB = npb;
    M.BR = M.RPW * M.NPB;
    for (int i = 0; i < J.nseg - 1; ++i)
        if ((J.seg[i].row_end - (i ? J.seg[i - 1].row_end : 0)) % M.BR) return false;
    M.nbj = (J.rows + M.BR - 1) / M.BR;
    M.slot_bytes = M.BR * M.srow * nw;
    const int fixed = (kind == TRX_KIND_TERNARY5 ? kLutBytes : 0) + kWarpsMv * 2 * M.BR * 8 + M.G * M.xwords * 4 +
                      ((M.G * 4 + 15) / 16) * 16 + 64 * 4 + 16 + cols + 128;
    int d = kRingTarget / M.slot_bytes;
    if (d > kMaxDepth) d = kMaxDepth;
    if (d < 2) d = 2;
    while (d > 2 && fixed + kWarpsMv * d * M.slot_bytes > kSmemMax) --d;
    M.D = d;
    M.smem = (fixed + kWarpsMv * d * M.slot_bytes + 127) / 128 * 128;
    return M.smem <= kSmemMax;
}

static int g_num_sms = 0;

static int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

template <int KIND>
static trx_status launch_tmv(const MvJobs &J, const MvGeom &M, int grid, const uint32_t *lut, uint32_t *err,
                             cudaStream_t st) {
    static int configured = 0;
    if (M.smem > configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(tmv_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return note_cuda(e);
        configured = kSmemMax;
    }
    tmv_kernel<KIND><<<grid, kMvThreads, M.smem, st>>>(J, M, lut, err);
    return note_cuda(cudaGetLastError());
}

trx_status launch_matvec(const MvJobs &J, const uint32_t *lut, uint32_t *err, cudaStream_t st) {
    MvGeom M;
    if (!plan_matvec(J, J.cols, J.kind, J.w2 ? 2 : 1, M)) return TRX_ERR_UNSUPPORTED;
    if (M.nck > 1 && (!J.acc || !J.cnt || (uint64_t)J.njobs * (uint64_t)J.rows > J.acc_rows))
        return TRX_ERR_UNSUPPORTED;
    long long want = ((long long)J.njobs * M.nbj + 1) / 2;  // at least a couple of blocks per CTA
    int grid = num_sms();
    if (want < grid) grid = (int)(want < 1 ? 1 : want);
    if (J.kind == TRX_KIND_TERNARY5) return launch_tmv<TRX_KIND_TERNARY5>(J, M, grid, lut, err, st);
    return launch_tmv<TRX_KIND_TERNARY>(J, M, grid, lut, err, st);
}

trx_status launch_matvec_fp(const MvJobs &J, uint32_t *err, cudaStream_t st) {
    const int G = J.cols / 128;
    const int TR = 16;
    const int smem = J.cols * 4 + TR * (G + 1) * 4;
    if (smem > kSmemMax) return TRX_ERR_UNSUPPORTED;
    int grid = (J.rows + TR - 1) / TR;
    if (grid > num_sms() * 4) grid = num_sms() * 4;
    cudaError_t e;
    if (J.kind == TRX_KIND_TERNARY5) {
        e = cudaFuncSetAttribute(tmv_fp_kernel<TRX_KIND_TERNARY5>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return note_cuda(e);
        tmv_fp_kernel<TRX_KIND_TERNARY5><<<grid, 256, smem, st>>>(J, TR, err);
    } else {
        e = cudaFuncSetAttribute(tmv_fp_kernel<TRX_KIND_TERNARY>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return note_cuda(e);
        tmv_fp_kernel<TRX_KIND_TERNARY><<<grid, 256, smem, st>>>(J, TR, err);
    }
    return note_cuda(cudaGetLastError());
}

trx_status launch_quantize(const float *x, int n, int8_t *x8, int *e8, cudaStream_t st) {
    quantize_kernel<<<1, 1024, 0, st>>>(x, n, x8, e8);
    return note_cuda(cudaGetLastError());
}

trx_status launch_validate_t5(const uint8_t *w, int rows, int cols, uint32_t *err, cudaStream_t st) {
    const int G = cols / 128;
    const int sb = (G + 15) / 16 * 32;
    const int rb = sb + (26 * G + 31) / 32 * 32;
    long long total = (long long)rows * 26 * G;
    int grid = (int)((total + 255) / 256);
    if (grid > num_sms() * 8) grid = num_sms() * 8;
    if (grid < 1) grid = 1;
    validate_t5_kernel<<<grid, 256, 0, st>>>(w, rows, rb, sb, G, err);
    return note_cuda(cudaGetLastError());
}

trx_status launch_build_lut(uint32_t *lut, cudaStream_t st) {
    build_lut_kernel<<<kLutWords / 256, 256, 0, st>>>(lut);
    return note_cuda(cudaGetLastError());
}

size_t lut_bytes() { return kLutBytes; }

}  // namespace trx
