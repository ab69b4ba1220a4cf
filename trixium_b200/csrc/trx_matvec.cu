// Ternary matvec kernels for B200 (sm_100a): the TriXium engine's group-128 matvec over the
// converter's row packets (2-bit and 5-trit codes), bit-exact with model/bitexact.py:101-119,
// with the firmware's float wrapper (quantise -> engine -> scale, firmware/infer_float.c:398)
// fused in, and the fp-mode projection of model/fastref.py:103-125.
//
// Work decomposition (row per lane):
//  * A row block is 32 consecutive output rows; lane l of a warp owns row l of the block for the
//    whole of it and keeps that row's exact int64 sum in a register, so no cross-lane reduction
//    exists anywhere on the path.
//  * A row is cut into chunks of 4 groups (512 weights).  A block is one chunk of the 32 rows:
//    per row 16 bytes of scales and the chunk's codes (104 bytes of trit5, 128 of 2-bit), laid
//    out in shared memory at a 144-byte row stride (9 x 16 B, odd: the 32 lanes' 16-byte loads
//    of their own rows never conflict).
//  * Row blocks are dealt to CTAs (up to 16 warps, one CTA per SM) in contiguous ranges of
//    (job, row block) space.  A warp streams its blocks global -> shared through a private ring of
//    D slots: one elected lane issues a block's TMA boxes (per tensor, the codes box {cb bytes, 32
//    rows} and the scales box {16 bytes, 32 rows} of the packed tensor viewed as [jobs][rows][row
//    bytes]) on the slot's mbarrier; the lanes wait on it (bounded) and the slot is refilled with
//    the block D ahead.  No producer warp and no CTA barrier inside a job.  (Measured on B200: the
//    2-D boxes keep the rings' bytes in flight without the per-copy issue cost of 16-byte cp.async;
//    the 96-copy config-0 batch went from 2.4 to 3.2 TB/s for trit5 and from 3.9 to 4.7 TB/s for
//    2-bit.)
//  * When a CTA holds fewer row blocks than warps (a single decode matvec), S warps share a row
//    block, each taking a range of its chunks; after every round the S partial int64 sums per row
//    are added in a fixed order through shared memory behind a named barrier (exact, no atomics).
//  * The quantised activation of the job is built once per CTA in shared memory (x staged once,
//    then quantised straight into the per-group permuted words the decoders multiply with, read as
//    broadcast 16-byte loads).
//  * Group sums are exact int32 (dp4a / dp2a).  The scale contribution (gs*m11) << (e16+B) is
//    one int32 x int32 -> int64 multiply in the common case.  The warp that finishes a row applies
//    >> R, the overflow checks, the float scaling and the epilogue.
//  * Every launch is a programmatic dependent of its predecessor: the LUT is built and the first
//    weight blocks are requested before griddepcontrol.wait; the activation is read after it.
//  * trit5 decode: a 256-entry byte LUT (digits d0, d1, d2 and d3+3*d4 as bytes), replicated 32x
//    (one copy per lane, so lookups never bank-conflict), addressed with one PRMT per byte.
//    dp4a adds d0*x0+d1*x1+d2*x2+(d3+3d4)*x3; the d4 correction d4*(x4-3*x3) is a dp2a on
//    16-bit activation pairs, d4 = (d3+3d4)/3 computed for four bytes at once.
//  * 2-bit decode: four masks per word; dp4a on (code << 2p) bytes into four accumulators.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cuda.h>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

// Launch shape and shared-memory plan --------------------------------------------------------------
#ifndef TRX_MV_MAX_WARPS
#define TRX_MV_MAX_WARPS 16
#endif
// Rows per lane of a full-size trit5 / 2-bit launch (a launch whose CTAs share row blocks between
// warps, or a SwiGLU pair, always takes one).  Measured on B200 (config-0 batch): two rows per lane
// (the activation words loaded once for both) ran slower for both kinds than one row per lane with
// more warps (trit5 2.2 against 3.1-3.2 TB/s; 2-bit 4.3 against 4.7 TB/s), so one is the default.
#ifndef TRX_MV_R_T5
#define TRX_MV_R_T5 1
#endif
#ifndef TRX_MV_R_2B
#define TRX_MV_R_2B 1
#endif
constexpr int kMaxWarps = TRX_MV_MAX_WARPS;
constexpr int kMvThreads = kMaxWarps * 32;       // launch bound (a launch may use fewer warps)
constexpr int kLutWords = 256 * 64;              // 256 entries x 256-byte stride (32 replicas used)
constexpr int kLutBytes = kLutWords * 4;         // 64 KiB
constexpr int kXwT5 = 44;    // words per group: 26 dp4a words, 14 dp2a words, sum(x), 3 zero
constexpr int kXw2b = 36;    // words per group: 32 dp4a words, sum(x), 3 zero
constexpr int kCG = 4;                           // groups per chunk
constexpr int kCbT5 = 112;   // trit5 codes box per row: the chunk's 104 bytes from the 16-byte boundary at or below them
constexpr int kCb2b = 144;   // 2-bit codes box per row: the chunk's 128 bytes and the next 16 (an odd 16-byte stride)
constexpr int kScBox = 16;   // scales box per row: the 8 fp16 scales of chunks 2j, 2j+1
constexpr int kMaxD = 3;     // ring slots per warp at most
constexpr int kSmemMax = 227 * 1024;

// Geometry of one launch, derived on the host (plan_matvec) and passed by value.
struct MvGeom {
    int G;        // groups per row
    int nch;      // chunks per row (the last may hold fewer than kCG groups)
    int cpt;      // chunks per warp per row block
    int S;        // warps sharing a row block (a power of two; 1: a warp owns whole row blocks)
    int R;        // rows per lane (a row block is 32 R rows)
    int nrb;      // row blocks per job
    int grid;     // CTAs
    int rb;       // row packet bytes in global memory
    int sbytes;   // scale-region bytes of a packet
    int nw;       // tensors per block (2 for SwiGLU)
    int warps;    // warps per CTA
    int D;        // ring depth (blocks)
    int xw;       // activation words per group
    int cb;       // codes box bytes per row (kCbT5 or kCb2b)
    int cbytes;   // codes bytes of one tensor in a slot (32 R rows x cb)
    int slot;     // bytes of one ring slot: NW codes boxes, then NW scales boxes
    int wjob;     // the tensor maps have a job dimension (jobs read distinct weights)
    int fixed;    // bytes of activation words, reductions and barriers (128-byte rounded): rings A start here
    int red_off;  // shared offset of the combine area of warps sharing a row block
    int bar_off;  // shared offset of the ring barriers ([kMaxWarps][kMaxD] uint64)
    int na;       // warps whose ring lies in region A (the rest: region C, after the trit5 LUT)
    int sreg;     // the staging area lies in region C (1) or A (0)
    int stage_off;  // its shared offset: the last bands (slot D-1, D-2, ...) of that region
    int ebl;      // slots of a staging-region warp below the staging area
    int xfast;    // float x takes the bulk-copy-staged prologue (build_activation_cp)
    int stage;    // bytes of that staging region
    int base;     // shared-window address of the dynamic shared memory the plan assumes
    int smem;     // dynamic shared bytes
};

// TMA tensor maps of one launch: per tensor (NW), the codes box {cb bytes, 32 R rows, 1 job} and
// the scales box {16 bytes, 32 R rows, 1 job} over the packed tensor viewed as [jobs][rows][row
// packet bytes].  Boxes past the tensor's rows or a row's end are zero-filled by the copy engine.
struct MvMaps {
    CUtensorMap codes[2];
    CUtensorMap scales[2];
};

// Quantisation helpers ----------------------------------------------------------------------------
// The value the quantiser sees at position k: x[k], or the RMS-normalised x[k]*r*w[k].
__device__ __forceinline__ float prologue_value(const float *x, const float *w, float r, int k) {
    float v = __ldg(x + k);
    if (w) v = __fmul_rn(__fmul_rn(v, r), __ldg(w + k));
    return v;
}

// The quantiser's value: clamp(lround_mirror(v * inv), -127, 127), without conversion
// instructions (a quarter of the ALU rate): a = fp32(|t| + 0.5) is the mirror's own rounded sum
// (fp32 addition is symmetric, so fp32(t - 0.5) = -a for t < 0), and floor(a) for a < 2^23 is the
// mantissa of fp32_round_down(a + 2^23).  a >= 128 (and inf) clamps to 127.
__device__ __forceinline__ int8_t quant_one(float v, float inv) {
    const float t = __fmul_rn(v, inv);
    const float a = __fadd_rn(fabsf(t), 0.5f);
    uint32_t m = __float_as_uint(__fadd_rd(a, 8388608.0f)) & 0x7fffffu;
    m = a < 128.0f ? m : 127u;
    return (int8_t)(t < 0.f ? -(int)m : (int)m);
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

// Canonical sum of squares by one warp from shared memory: lane j runs partials j and j+32
// (x[j]^2 + x[j+64]^2 + ... in index order, model/mirror.py:576-591) side by side, loads ahead of
// the ordered adds, then the halving tree red[j] + red[j+32], 16, 8, ... in the same warp.  The
// sum is returned in lane 0.
__device__ __forceinline__ float warp_sumsq64(const float *xs, int K) {
    const int j = threadIdx.x & 31;
    float p0 = 0.f, p1 = 0.f;
    int i = j;
    for (; i + 7 * 64 + 32 < K; i += 8 * 64) {  // eight steps of both chains per round, loads first
        float a[8], b[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            a[u] = xs[i + u * 64];
            b[u] = xs[i + u * 64 + 32];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            p0 = __fadd_rn(p0, __fmul_rn(a[u], a[u]));
            p1 = __fadd_rn(p1, __fmul_rn(b[u], b[u]));
        }
    }
    for (; i < K; i += 64) {
        p0 = __fadd_rn(p0, __fmul_rn(xs[i], xs[i]));
        if (i + 32 < K) p1 = __fadd_rn(p1, __fmul_rn(xs[i + 32], xs[i + 32]));
    }
    float a2 = __fadd_rn(p0, p1);
    for (int o = 16; o; o >>= 1) a2 = __fadd_rn(a2, __shfl_down_sync(0xffffffffu, a2, o));
    return a2;
}

// Quantise x (fp32 in shared memory) straight into the permuted activation words, one warp per
// group: each lane quantises the values of the words it writes; the group sum by a warp reduction.
template <int KIND>
__device__ __forceinline__ void permute_groups(const float *xs, float inv, int G, uint32_t *xp) {
    const int lane = threadIdx.x & 31;
    for (int g = threadIdx.x >> 5; g < G; g += blockDim.x >> 5) {
        const float *xg = xs + g * 128;
        if (KIND == TRX_KIND_TERNARY5) {
            uint32_t *w = xp + g * kXwT5;
            // Lane i < 26: byte i's activations x[5i .. 5i+4] (weights 128/129 see 0): word i, and
            // y_i = x[5i+4] - 3*x[5i+3] for the 16-bit pairs (y[2m], y[2m+1]) of words 26 + m.
            int q[5] = {0, 0, 0, 0, 0};
            if (lane < 26) {
#pragma unroll
                for (int k = 0; k < 5; ++k) {
                    const int l = 5 * lane + k;
                    q[k] = l < 128 ? (int)quant_one(xg[l], inv) : 0;
                }
                w[lane] = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
                          ((uint32_t)(q[3] & 0xff) << 24);
            }
            const int y = q[4] - 3 * q[3];
            const int yn = __shfl_down_sync(0xffffffffu, y, 1);
            if (lane < 28 && !(lane & 1)) w[26 + (lane >> 1)] = ((uint32_t)y & 0xffffu) | ((uint32_t)yn << 16);
            const int sum = __reduce_add_sync(0xffffffffu, q[0] + q[1] + q[2] + q[3] + q[4]);
            if (lane == 0) w[40] = (uint32_t)sum;
            if (lane >= 1 && lane < 4) w[40 + lane] = 0u;
        } else {
            uint32_t *w = xp + g * kXw2b;
            // Lane j = 4*wq + p: bytes x[16wq + 4b + p], b = 0..3 (the activations that meet bit
            // pair p of code bytes 4wq .. 4wq+3).
            const int wq = lane >> 2, p = lane & 3;
            int q[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) q[b] = (int)quant_one(xg[16 * wq + 4 * b + p], inv);
            w[lane] = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
                      ((uint32_t)(q[3] & 0xff) << 24);
            const int sum = __reduce_add_sync(0xffffffffu, q[0] + q[1] + q[2] + q[3]);
            if (lane == 0) w[32] = (uint32_t)sum;
            if (lane >= 1 && lane < 4) w[32 + lane] = 0u;
        }
    }
}

// Build the permuted int8 activation of one job in shared memory (all threads of the CTA).
// q8: K bytes of staging, xp: G * xw words.  xs (or NULL): 4K bytes of shared staging for x, so x
// and the norm weight are read from global memory once.  Returns e8.
template <int KIND>
__device__ int build_activation(const float *x, const int8_t *x8g, const float *nw, float eps, int K, int8_t *q8,
                                float *xs, uint32_t *xp, uint32_t *amax_s, float *red64) {
    const int ct = threadIdx.x;
    const int nt = blockDim.x;
    int e8 = 0;
    if (x8g) {
        for (int k = ct; k < K; k += nt) q8[k] = x8g[k];
    } else if (xs) {
        // x -> shared (one coalesced pass), then the canonical sum of squares, the prologue values
        // (x*r)*w in place with their max, and the quantiser, all from shared memory.
        for (int i = ct; i < K / 4; i += nt)
            reinterpret_cast<float4 *>(xs)[i] = __ldg(reinterpret_cast<const float4 *>(x) + i);
        if (ct == 0) *amax_s = 0u;
        __syncthreads();
        float r = 0.f;
        if (nw) {
            if (ct < 32) {
                const float a = warp_sumsq64(xs, K);
                if (ct == 0) red64[0] = a;
            }
            __syncthreads();
            r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red64[0], (float)K), eps)));
        }
        uint32_t m = 0;
        for (int i = ct; i < K / 4; i += nt) {
            float4 v = reinterpret_cast<float4 *>(xs)[i];
            if (nw) {
                const float4 wv = __ldg(reinterpret_cast<const float4 *>(nw) + i);
                v.x = __fmul_rn(__fmul_rn(v.x, r), wv.x);
                v.y = __fmul_rn(__fmul_rn(v.y, r), wv.y);
                v.z = __fmul_rn(__fmul_rn(v.z, r), wv.z);
                v.w = __fmul_rn(__fmul_rn(v.w, r), wv.w);
                reinterpret_cast<float4 *>(xs)[i] = v;
            }
            const uint32_t a = max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                                   max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w))));
            m = a > m ? a : m;
        }
        m = __reduce_max_sync(0xffffffffu, m);
        uint32_t *const wmax = reinterpret_cast<uint32_t *>(red64) + 32;  // per-warp maxima
        if ((ct & 31) == 0) wmax[ct >> 5] = m;
        __syncthreads();
        uint32_t amax = 0u;
        for (int w = 0; w < (nt >> 5); ++w) amax = max(amax, wmax[w]);
        e8 = amax ? frexp_exp(__uint_as_float(amax)) - 7 : 0;
        const float inv = amax ? pow2f(-e8) : 0.f;  // all-zero x: every q is 0
        permute_groups<KIND>(xs, inv, K / 128, xp);
        __syncthreads();
        return e8;
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
    constexpr int XW = KIND == TRX_KIND_TERNARY5 ? kXwT5 : kXw2b;
    constexpr int XS = KIND == TRX_KIND_TERNARY5 ? 40 : 32;  // the word holding sum(x) of the group
    for (int idx = ct; idx < G * XW; idx += nt) {
        const int g = idx / XW, j = idx % XW;
        const int8_t *qg = q8 + g * 128;
        uint32_t w = 0;
        if (j == XS) continue;  // written below
        if (KIND == TRX_KIND_TERNARY5) {
            // Words 0..25 = bytes (x[5i], x[5i+1], x[5i+2], x[5i+3]); words 26..39 = 16-bit pairs
            // (y[2j], y[2j+1]) with y[i] = x[5i+4] - 3*x[5i+3]; lanes 128/129 (digits 3/4 of byte
            // 25) see x = 0.
            if (j < 26) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int l = 5 * j + k;
                    const uint32_t b = l < 128 ? (uint32_t)(uint8_t)qg[l] : 0u;
                    w |= b << (8 * k);
                }
            } else if (j < 40) {
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
        } else if (j < 32) {
            // Word (w*4 + p) = bytes x[16w + 4b + p], b = 0..3: the activations that meet bit
            // pair p of code bytes 4w..4w+3.
            const int wq = j >> 2, p = j & 3;
#pragma unroll
            for (int b = 0; b < 4; ++b) w |= (uint32_t)(uint8_t)qg[16 * wq + 4 * b + p] << (8 * b);
        }
        xp[idx] = w;
    }
    // Group sums of x8: one warp per group.
    for (int g = ct >> 5; g < G; g += nt >> 5) {
        const int lane = ct & 31;
        const int8_t *qg = q8 + g * 128 + 4 * lane;
        int s = (int)qg[0] + (int)qg[1] + (int)qg[2] + (int)qg[3];
        s = __reduce_add_sync(0xffffffffu, s);
        if (lane == 0) xp[g * XW + XS] = (uint32_t)s;
    }
    __syncthreads();
    return e8;
}

// Staged prologue: x is copied into shared memory with cp.async (every copy in flight at once, no
// registers held), the norm weight likewise (issued before the predecessor is waited for, when the
// caller passes nw_ready).  The canonical sum-of-squares chains, the normalisation and the max run
// over shared memory; the quantiser then reads one float4 per lane (group g = a warp's 32 float4)
// and builds the decoders' activation words with warp shuffles.  Bit-identical to
// build_activation (same values, same order of every rounded operation).  Needs x and nw 16-byte
// aligned; xs: K floats of shared memory, nws: K more when nw is given.  Returns e8.
__device__ __forceinline__ uint32_t absmax4(float4 v) {
    return max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
               max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w))));
}

// x as tagged words (tensor-parallel exchange): every thread polls its words, eight loads in flight,
// until each carries `tag`, and writes the values to xs.  False when a wait ran out (recorded).
__device__ __forceinline__ bool gather_tagged(const unsigned long long *xt, unsigned tag, int K, float *xs,
                                              uint32_t *err) {
    constexpr int U = 8;
    const ulonglong2 *const p = reinterpret_cast<const ulonglong2 *>(xt);
    float2 *const xs2 = reinterpret_cast<float2 *>(xs);
    const int n2 = K / 2, nt = blockDim.x;
    unsigned long long t0 = 0ull;
    for (int base = threadIdx.x; base < n2; base += U * nt) {
        ulonglong2 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (base + u * nt < n2) v[u] = ld_tagged2(p + base + u * nt);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * nt;
            if (i < n2) {
                while ((unsigned)(v[u].x >> 32) != tag || (unsigned)(v[u].y >> 32) != tag) {
                    if (!t0) {
                        t0 = global_ns();
                    } else if (global_ns() - t0 > kWaitNs) {
                        atomicOr(err, TRX_DEV_TIMEOUT);
                        return false;
                    }
                    v[u] = ld_tagged2(p + i);
                }
                xs2[i] = make_float2(__uint_as_float((uint32_t)v[u].x), __uint_as_float((uint32_t)v[u].y));
            }
        }
    }
    return true;
}

template <int KIND>
__device__ int build_activation_cp(const float *x, const float *nw, bool nw_ready, float eps, int K, float *xs,
                                   float *nws, uint32_t *xp, float *red64, uint64_t *mb, uint32_t parity,
                                   uint32_t *err, bool &ok, unsigned xtag, int Kw, int x_off) {
    // K: the elements of x (the exponent and any norm cover them all); the activation words are built
    // for the Kw columns from x_off on.
    const int ct = threadIdx.x, lane = ct & 31, warp = ct >> 5, nwarps = blockDim.x >> 5;
    const int G = Kw / 128, n4 = K / 4;
    float4 *const xs4 = reinterpret_cast<float4 *>(xs);
    // One bulk copy each (tracked by its own barrier, not by the weight rings' barriers); thread 0
    // waits, bounded, and the block learns the outcome at the barrier.  (Measured on B200 in decode
    // launches: the bulk copy of x reaches the built activation sooner than coalesced loads by
    // every thread.)  xtag != 0: x is tagged words, polled by every thread instead.
    uint32_t *const flag = reinterpret_cast<uint32_t *>(red64) + 48;
    if (ct == 0) {
        fence_proxy_async();  // earlier generic accesses to these bytes come first
        if (!xtag) {
            mbar_arrive_expect_tx(mb, 4u * K);
            bulk_g2s(xs, x, 4u * K, mb);
        }
        if (nw && !nw_ready) {
            mbar_arrive_expect_tx(mb + 1, 4u * K);
            bulk_g2s(nws, nw, 4u * K, mb + 1);
        }
        bool w = xtag ? true : mbar_wait_bounded(mb, parity, err);
        if (nw) w = mbar_wait_bounded(mb + 1, parity, err) && w;
        *flag = w ? 1u : 0u;
    }
    const bool tbad = xtag ? !gather_tagged(reinterpret_cast<const unsigned long long *>(x), xtag, K, xs, err) : false;
    const int anybad = __syncthreads_or(tbad ? 1 : 0);
    ok = *flag != 0u && !anybad;
    if (!ok) return 0;
    uint32_t m = 0;
    if (nw) {
        if (warp == 0) {
            const float a = warp_sumsq64(xs, K);
            if (lane == 0) red64[0] = a;
        }
        __syncthreads();
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red64[0], (float)K), eps)));
        const float4 *const nw4 = reinterpret_cast<const float4 *>(nws);
        for (int i = ct; i < n4; i += blockDim.x) {
            float4 v = xs4[i];
            const float4 w = nw4[i];
            v.x = __fmul_rn(__fmul_rn(v.x, r), w.x);
            v.y = __fmul_rn(__fmul_rn(v.y, r), w.y);
            v.z = __fmul_rn(__fmul_rn(v.z, r), w.z);
            v.w = __fmul_rn(__fmul_rn(v.w, r), w.w);
            xs4[i] = v;
            const uint32_t a = absmax4(v);
            m = a > m ? a : m;
        }
    } else {
        for (int i = ct; i < n4; i += blockDim.x) {
            const uint32_t a = absmax4(xs4[i]);
            m = a > m ? a : m;
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    uint32_t *const wmax = reinterpret_cast<uint32_t *>(red64) + 32;  // per-warp maxima
    if (lane == 0) wmax[warp] = m;
    __syncthreads();
    const uint32_t amax = __reduce_max_sync(0xffffffffu, lane < nwarps ? wmax[lane] : 0u);
    const int e8 = amax ? frexp_exp(__uint_as_float(amax)) - 7 : 0;
    const float inv = amax ? pow2f(-e8) : 0.f;  // all-zero x: every q is 0
#pragma unroll 2
    for (int g = warp; g < G; g += nwarps) {
        const float4 v = xs4[(x_off >> 2) + g * 32 + lane];
        const int q0 = quant_one(v.x, inv), q1 = quant_one(v.y, inv), q2 = quant_one(v.z, inv),
                  q3 = quant_one(v.w, inv);
        // This lane's bytes x8[4l .. 4l+3] of the group.
        const uint32_t W = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
                           ((uint32_t)(q3 & 0xff) << 24);
        const int sum = __reduce_add_sync(0xffffffffu, q0 + q1 + q2 + q3);
        if (KIND == TRX_KIND_TERNARY5) {
            uint32_t *w = xp + g * kXwT5;
            // Lane i < 26: word i = bytes x8[5i .. 5i+3], y_i = x8[5i+4] - 3*x8[5i+3] (bytes 128 and
            // 129 of the last code byte are 0); the bytes come from lanes 5i/4 and 5i/4+1.
            const int a = (5 * lane) >> 2, off = (5 * lane) & 3;
            const uint32_t lo = __shfl_sync(0xffffffffu, W, a & 31);
            const uint32_t hi0 = __shfl_sync(0xffffffffu, W, (a + 1) & 31);
            const uint32_t hi = a + 1 < 32 ? hi0 : 0u;
            const uint32_t w1 = __funnelshift_rc(lo, hi, 8 * off);      // x8[5i .. 5i+3]
            const uint32_t w2 = __funnelshift_rc(lo, hi, 8 * off + 8);  // x8[5i+1 .. 5i+4]
            const int y = lane < 26 ? (int)(int8_t)(w2 >> 24) - 3 * (int)(int8_t)(w1 >> 24) : 0;
            const int yn = __shfl_down_sync(0xffffffffu, y, 1);
            if (lane < 26) w[lane] = w1;
            if (lane < 28 && !(lane & 1)) w[26 + (lane >> 1)] = ((uint32_t)y & 0xffffu) | ((uint32_t)yn << 16);
            if (lane == 0) w[40] = (uint32_t)sum;
            if (lane >= 1 && lane < 4) w[40 + lane] = 0u;
        } else {
            uint32_t *w = xp + g * kXw2b;
            // Word 4wq+p = bytes x8[16wq + 4b + p], b = 0..3: a 4x4 byte transpose across each quad
            // of lanes (lane 4wq+b holds x8[16wq + 4b .. 16wq + 4b + 3]).
            const uint32_t s1 = __shfl_xor_sync(0xffffffffu, W, 1);
            const uint32_t A = (lane & 1) ? __byte_perm(W, s1, 0x3715u) : __byte_perm(W, s1, 0x6240u);
            const uint32_t s2 = __shfl_xor_sync(0xffffffffu, A, 2);
            w[lane] = (lane & 2) ? __byte_perm(A, s2, 0x3276u) : __byte_perm(A, s2, 0x5410u);
            if (lane == 0) w[32] = (uint32_t)sum;
            if (lane >= 1 && lane < 4) w[32 + lane] = 0u;
        }
    }
    __syncthreads();
    return e8;
}

// Group sums -----------------------------------------------------------------------------------------
// The activation words of one group, loaded once per group and shared by the R rows of a lane.
template <int N>
__device__ __forceinline__ void load_xwords(const uint32_t *xg, uint32_t (&xa)[N]) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
        const uint4 v = reinterpret_cast<const uint4 *>(xg)[i];
        xa[4 * i] = v.x;
        xa[4 * i + 1] = v.y;
        xa[4 * i + 2] = v.z;
        xa[4 * i + 3] = v.w;
    }
}

// trit5, group g of a chunk whose 104 code bytes start at byte H (0 or 8) of the 28-word window
// cw.  xa: the group's 44 activation words.  Returns sum((digit - 1) * x).
template <int H, int g>
__device__ __forceinline__ int gsum_t5(const uint32_t (&cw)[28], uint32_t lane4x, const uint32_t (&xa)[kXwT5]) {
    int acc[4] = {0, 0, 0, 0};  // independent chains (byte position within a quad)
#pragma unroll
    for (int q = 0; q < 7; ++q) {
        const int nb = q < 6 ? 4 : 2;
        uint32_t E[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (i < nb) {
                constexpr int base = H + 26 * g;
                const int pb = base + 4 * q + i;  // byte of the window (compile time)
                // a = 0x10000 + byte * 256 + lane * 4: the shared address of this lane's replica of
                // the entry (the LUT sits at window address 0x10000), no bank conflict.
                const uint32_t a = __byte_perm(cw[pb >> 2], lane4x, 0x7604u | ((pb & 3) << 4));
                asm("ld.shared.u32 %0, [%1];" : "=r"(E[i]) : "r"(a));
                acc[i] = dp4a_ss(E[i], xa[4 * q + i], acc[i]);
            }
        }
        if (nb == 4) {
            const uint32_t d01 = __byte_perm(E[0], E[1], 0x0073u);
            const uint32_t d23 = __byte_perm(E[2], E[3], 0x0073u);
            const uint32_t D = __umulhi(__byte_perm(d01, d23, 0x5410u), 11u << 27) & 0x03030303u;
            acc[q & 3] = dp2a_lo(xa[26 + 2 * q], D, acc[q & 3]);
            acc[(q + 2) & 3] = dp2a_hi(xa[26 + 2 * q + 1], D, acc[(q + 2) & 3]);
        } else {
            const uint32_t D = __umulhi(__byte_perm(E[0], E[1], 0x0073u), 11u << 27) & 0x03030303u;
            acc[3] = dp2a_lo(xa[26 + 2 * q], D, acc[3]);
        }
    }
    return (acc[0] + acc[1]) + (acc[2] + acc[3]) - (int)xa[40];
}

// 2-bit, one group: the 32 code bytes at cp (shared, 16-byte aligned), xw its 36 activation words.
// Returns sum((code - 1) * x).
__device__ __forceinline__ int gsum_2b(const uint4 *cp, const uint32_t (&xw)[kXw2b]) {
    const uint4 c0 = cp[0], c1 = cp[1];
    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t c = cw[w];
        a0 = dp4a_us(c & 0x03030303u, xw[4 * w + 0], a0);
        a1 = dp4a_us(c & 0x0c0c0c0cu, xw[4 * w + 1], a1);
        a2 = dp4a_us(c & 0x30303030u, xw[4 * w + 2], a2);
        a3 = dp4a_us(c & 0xc0c0c0c0u, xw[4 * w + 3], a3);
    }
    return a0 + (a1 >> 2) + (a2 >> 4) + (a3 >> 6) - (int)xw[32];
}

__device__ __forceinline__ uint32_t scale_bits(uint2 s, int g) {
    const uint32_t w = g < 2 ? s.x : s.y;
    return g & 1 ? w >> 16 : w & 0xffffu;
}

// One chunk c (ng <= 4 groups) of the R rows of this lane held in a ring slot: codes at `codes`
// (row r of the lane at (lane + 32 r) * cb; trit5: the chunk's bytes from byte H = 8 (c & 1) of
// the row's window), scales at `scales` (16 bytes per row, this chunk's 4 at byte soff = 8 (c & 1)).
// Group by group, the activation words are loaded once and used for every row.
template <int KIND, int R, int H>
__device__ __forceinline__ void chunk_rows(const unsigned char *codes, const unsigned char *scales, int soff, int lane,
                                           int ng, const uint32_t *xg, uint32_t lane4x, const int (&Bv)[R],
                                           const ScaleFast (&Fv)[R], long long (&acc)[R]) {
    uint2 sc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) sc[r] = *reinterpret_cast<const uint2 *>(scales + (lane + 32 * r) * kScBox + soff);
    if (KIND == TRX_KIND_TERNARY5) {
        uint32_t cw[R][28];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint4 *rp = reinterpret_cast<const uint4 *>(codes + (lane + 32 * r) * kCbT5);
#pragma unroll
            for (int i = 0; i < 7; ++i) {
                const uint4 v = rp[i];
                cw[r][4 * i] = v.x;
                cw[r][4 * i + 1] = v.y;
                cw[r][4 * i + 2] = v.z;
                cw[r][4 * i + 3] = v.w;
            }
        }
        uint32_t xa[kXwT5];
        load_xwords(xg, xa);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += contrib(gsum_t5<H, 0>(cw[r], lane4x, xa), scale_bits(sc[r], 0), Bv[r], Fv[r]);
        if (ng > 1) {
            load_xwords(xg + kXwT5, xa);
#pragma unroll
            for (int r = 0; r < R; ++r)
                acc[r] += contrib(gsum_t5<H, 1>(cw[r], lane4x, xa), scale_bits(sc[r], 1), Bv[r], Fv[r]);
        }
        if (ng > 2) {
            load_xwords(xg + 2 * kXwT5, xa);
#pragma unroll
            for (int r = 0; r < R; ++r)
                acc[r] += contrib(gsum_t5<H, 2>(cw[r], lane4x, xa), scale_bits(sc[r], 2), Bv[r], Fv[r]);
        }
        if (ng > 3) {
            load_xwords(xg + 3 * kXwT5, xa);
#pragma unroll
            for (int r = 0; r < R; ++r)
                acc[r] += contrib(gsum_t5<H, 3>(cw[r], lane4x, xa), scale_bits(sc[r], 3), Bv[r], Fv[r]);
        }
    } else {
#pragma unroll
        for (int g = 0; g < kCG; ++g) {
            if (g < ng) {
                uint32_t xw[kXw2b];
                load_xwords(xg + g * kXw2b, xw);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const uint4 *cp = reinterpret_cast<const uint4 *>(codes + (lane + 32 * r) * kCb2b) + 2 * g;
                    acc[r] += contrib(gsum_2b(cp, xw), scale_bits(sc[r], g), Bv[r], Fv[r]);
                }
            }
        }
    }
}

// The float epilogue value of one finished row (the firmware's int32 -> float scaling).
__device__ __forceinline__ float row_float(long long acc, int R, int e8, int B) {
    const int res = (int)(acc >> R);
    return __fmul_rn((float)res, pow2f(e8 + R - B));
}

__device__ __forceinline__ float silu_f32(float g) {
    // x / (1 + exp(-x)) in fp32 (model/mirror.py:713, mathematical profile).
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}


// Row output --------------------------------------------------------------------------------------
// Segment s of a launch holds rows [seg_start(s), seg[s].row_end) of the packed tensor.  The
// kernel reads the segment table from a shared copy made before the dependency wait (a lookup by
// a row-dependent index into the parameter block would miss the constant cache on the critical
// path).
__device__ __forceinline__ int seg_start(const MvSeg *segs, int s) { return s ? segs[s - 1].row_end : 0; }

// Per-block output context (uniform over a block: blocks never straddle segments).
struct RowOut {
    int R, R2, B;
    float sc, sc2;         // 2^(e8 + R - B) of the tensor(s)
    char *y;               // output of the segment's row 0 (this job)
    const float *resid;    // residual of the segment's row 0, or nullptr
};

__device__ __forceinline__ RowOut row_out(const MvJobs &J, const MvSeg *segs, int job, int s, int e8) {
    const MvSeg &S = segs[s];
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

// A result's copies into the ranks' destinations (tensor-parallel all-gather by stores over peer
// memory).
__device__ __forceinline__ void tp_push(const TpXfer &T, int i, float v) {
    if (T.world) tp_push_all(T, (size_t)i, v);
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
        // The earlier K-segments' int32 sum, added as the mirror sums the segments' results (int64,
        // then the int32 wrap).
        const int res = J.part_in ? (int)(uint32_t)(unsigned long long)((long long)J.part_in[srow] + (a >> o.R))
                                  : (int)(a >> o.R);
        float v = __fmul_rn((float)res, o.sc);
        if (o.resid) v = __fadd_rn(o.resid[srow], v);
        if (o.y) reinterpret_cast<float *>(o.y)[srow] = v;
        if (J.argmax) key = argmax_key(v, (uint32_t)(row + J.row_offset));
        if (!J.key_out) tp_push(J.tp, srow, v);  // a key launch exchanges its key, not its rows
    } else {  // OUT_SWIGLU
        bad = bad || acc_bad(a2, o.R2);
        const float gv = __fmul_rn((float)(int)(a >> o.R), o.sc);
        const float uv = __fmul_rn((float)(int)(a2 >> o.R2), o.sc2);
        const float v = __fmul_rn(silu_f32(gv), uv);
        reinterpret_cast<float *>(o.y)[srow] = v;
        tp_push(J.tp, srow, v);
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


// This lane's output context for one of the rows it owns in the current task.
struct LaneRow {
    int row;        // row of the packed tensor (or -1 past the end)
    int srow;       // row within its segment
    int B;          // scale bias of the row's tensor
    ScaleFast F;    // its fast scale range
    RowOut o;
};

__device__ __forceinline__ void lane_row(const MvJobs &J, const MvSeg *segs, int job, int row, int e8,
                                         const LaneRow &one, LaneRow &L) {
    if (J.nseg == 1) {  // one tensor: the context of segment 0, computed once per job
        L = one;
        L.row = row < J.rows ? row : -1;
        L.srow = row;
        return;
    }
    L.row = row < J.rows ? row : -1;
    int sg = 0;
#pragma unroll
    for (int i = 0; i < kMaxSegs - 1; ++i) sg += (i < J.nseg - 1 && row >= segs[i].row_end) ? 1 : 0;
    L.o = row_out(J, segs, job, sg, e8);
    L.B = L.o.B;
    L.F = scale_fast(L.B);
    L.srow = row - seg_start(segs, sg);
}

// The matvec kernel ---------------------------------------------------------------------------------
// Default ring depth (plan_matvec): trit5 shares shared memory with its 64 KiB LUT, a SwiGLU pair
// streams two tensors.
#ifndef TRX_MV_D_T5
#define TRX_MV_D_T5 2
#endif

// Work decomposition: a row block is 32 R rows (lane l owns rows l, l + 32, ...); a block is one
// chunk (4 groups) of a row block.  Each warp streams its blocks through a private ring of D slots:
// one elected lane issues the block's TMA boxes (codes and scales of each tensor) on the slot's
// mbarrier; the lanes wait on it (bounded), decode, and the slot is refilled with the block D
// ahead.  No producer warp, no CTA barrier inside a job.
template <int KIND, int NW, int R, int D>
__global__ void __launch_bounds__(kMvThreads, 1)
    tmv_kernel(const __grid_constant__ MvMaps maps, MvJobs J, MvGeom M, uint32_t *err) {
    // D: ring depth, chosen per launch by plan_matvec (M.D), a compile-time constant of the kernel.
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    pdl_trigger();

    // Carve shared memory (must match plan_matvec): [activation words, reductions, barriers][rings A]
    // [trit5 LUT at window address 0x10000][rings C]; 2-bit: one ring region, no LUT.
    uint32_t *const xp = reinterpret_cast<uint32_t *>(smem);
    unsigned char *p = smem + M.G * M.xw * 4;
    float *const red64 = reinterpret_cast<float *>(p);
    p += 64 * 4;
    uint32_t *const amax_s = reinterpret_cast<uint32_t *>(p);
    uint64_t *const mb = reinterpret_cast<uint64_t *>(p + 16);  // bulk-copy barriers: x, norm weight
    MvSeg *const segs = reinterpret_cast<MvSeg *>(p + 32);      // the segment table
    if (tid < J.nseg) segs[tid] = J.seg[tid];                    // visible after the piece barrier
    const uint32_t bars = smem_u32(smem + M.bar_off) + (uint32_t)(warp * kMaxD * 8);  // this warp's slot barriers
    // Offsets (not pointers chosen between regions) keep every access provably shared.
    const int lut_off = 0x10000 - M.base, c_off = lut_off + kLutBytes;
    if (KIND == TRX_KIND_TERNARY5 && smem_u32(smem) != (uint32_t)M.base) {
        pdl_wait();
        if (tid == 0) atomicOr(err, TRX_DEV_INTERNAL);  // the window is not where the plan put the LUT
        return;
    }
    unsigned char *const lut = smem + lut_off;  // trit5 only
    // Rings are slot-major within a region: slot d of the region's k-th warp lies at region +
    // (d * n + k) * slot (n warps in the region), so the last slots of a region's warps form one
    // band, where the prologue stages its inputs.
    const int sstride = (warp < M.na ? M.na : M.warps - M.na) * M.slot;
    const int ring_off = warp < M.na ? M.fixed + warp * M.slot : c_off + (warp - M.na) * M.slot;
    unsigned char *const ring = smem + ring_off;
    const uint32_t ring_s = smem_u32(ring);
    int8_t *const q8 = reinterpret_cast<int8_t *>(smem + M.stage_off);  // staging; those slots idle then

    // Combine area of warps sharing a row block: [2 parities][warps][32 lanes][NW * R] int64.
    long long *const red = reinterpret_cast<long long *>(smem + M.red_off);

    // This CTA's share of the (job, row block) space.
    const long long total = (long long)J.njobs * M.nrb;
    const long long t0 = (long long)blockIdx.x * total / gridDim.x;
    const long long t1 = (long long)(blockIdx.x + 1) * total / gridDim.x;
    if (t0 >= t1) {
        pdl_wait();
        return;
    }

    if (KIND == TRX_KIND_TERNARY5) {  // the trit5 LUT: entry b at b*256, one replica per lane
        // The 256 entries once (in lane 0's replica words), then every lane copies them into its
        // own replica: each store instruction writes 32 distinct banks.
        uint32_t *lw = reinterpret_cast<uint32_t *>(lut);
        for (int b = tid; b < 256; b += blockDim.x) lw[b * 64] = trit5_lut_entry((uint32_t)b);
        __syncthreads();
        if (lane)
            for (int b = warp; b < 256; b += blockDim.x >> 5) lw[b * 64 + lane] = lw[b * 64];
    }
    const uint32_t lane4x = 0x10000u | ((uint32_t)lane * 4u);
    const ScaleFast F2 = scale_fast(J.B2);
    // Warp w: group gi = w / S (row block gi of each round of Rr = warps/S row blocks), chunks
    // [cA, cB) of that row block.
    const int Rr = M.warps / M.S;
    const int gi = warp / M.S, sub = warp - gi * M.S;
    const int cA = sub * M.cpt, cB = min(M.nch, cA + M.cpt);
    const int nc = cB > cA ? cB - cA : 0;
    const int Kx = J.x_cols ? J.x_cols : J.cols;  // elements of x
    float *const xs = M.stage >= ((J.cols + 15) / 16) * 16 + 4 * Kx
                          ? reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(q8) + ((J.cols + 15) / 16) * 16)
                          : nullptr;

    // Issue cursor of the current piece: (round, chunk) and blocks issued, of `nitems`.
    // The CTA's row blocks go to the warp groups round-robin over its whole range (u = t - t0 is
    // group u % Rr's), so the groups' totals differ by one at most even when the range spans jobs.
    int job = 0, pa = 0, pb = 0, gsh = 0, kval = 0, nitems = 0, ik = 0, ic = 0, issued = 0;
    uint32_t inflight = 0;  // bit d: slot d has copies in flight
    auto piece_begin = [&](long long t) {
        job = (int)(t / M.nrb);
        const long long jb = (long long)job * M.nrb;
        pa = (int)(t - jb);                          // this piece: row blocks [pa, pb) of `job`
        pb = (int)(min(t1, jb + M.nrb) - jb);
        gsh = (int)(((long long)gi - (t - t0) % Rr + Rr) % Rr);  // this group's first row block: pa + gsh
        kval = pb - pa > gsh ? (pb - pa - gsh + Rr - 1) / Rr : 0;  // rounds with a row block for gi
        nitems = kval * nc;                                         // blocks this warp streams
        ik = ic = issued = 0;
    };
    // Issue the next block of this warp's sequence into slot d: lane 0 arms the slot's barrier
    // with the slot's bytes (full boxes: the copy engine counts zero-filled bytes too) and issues
    // the boxes.  The caller has made every lane's reads of the slot complete (__syncwarp).
    auto issue_next = [&](int d) {
        if (issued < nitems) {
            if (lane == 0) {
                const int rbk = pa + gsh + ik * Rr, c = cA + ic;
                const uint32_t dst = ring_s + (uint32_t)(d * sstride);
                const uint32_t bar = bars + 8u * d;
                const int y = rbk * 32 * R, z = M.wjob ? job : 0;
                const int xc = KIND == TRX_KIND_TERNARY5 ? M.sbytes + 104 * c - 8 * (c & 1) : M.sbytes + 128 * c;
                const int xsc = 16 * (c >> 1);
                fence_proxy_async();  // this warp's reads of the slot come before the copy engine's writes
                mbar_expect_tx_s(bar, (uint32_t)M.slot);
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    tma_load_3d(dst + w * M.cbytes, &maps.codes[w], xc, y, z, bar);
                    tma_load_3d(dst + NW * M.cbytes + w * 32 * R * kScBox, &maps.scales[w], xsc, y, z, bar);
                }
            }
            if (++ic == nc) {
                ic = 0;
                ++ik;
            }
            ++issued;
            inflight |= 1u << d;
        }
    };
    uint32_t phase = 0;  // bit d: the parity of slot d's next completion
    // Before any early return: wait (bounded) for this warp's copies in flight into its slots.
    auto drain = [&]() {
#pragma unroll
        for (int d = 0; d < D; ++d)
            if (inflight & (1u << d)) {
                mbar_wait_bounded_s(bars + 8u * d, (phase >> d) & 1u, err);
                phase ^= 1u << d;
            }
        inflight = 0;
    };
    // The staging area [q8 bytes][x fp32][norm weight fp32] has a region of its own when shared
    // memory has room (decode-size launches), else it covers the last bands of the staging region.
    // The first piece's blocks for every slot outside it (weights: written by no kernel) are
    // requested before waiting for the predecessor: a decode-size launch streams its whole weight
    // share while the previous kernel still runs.
    const bool fast = M.xfast && J.x;
    const int xs_off = M.stage_off + ((J.cols + 15) / 16) * 16;
    float *const nws = reinterpret_cast<float *>(smem + xs_off + 4 * Kx);
    const int ne = (warp < M.na) == (M.sreg == 0) ? min(D, M.ebl) : D;
    if (lane == 0) {
#pragma unroll
        for (int d = 0; d < D; ++d) mbar_init_s(bars + 8u * d, 1);
    }
    if (tid == 0) {
        mbar_init(mb, 1);
        mbar_init(mb + 1, 1);
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            tma_prefetch_map(&maps.codes[w]);
            tma_prefetch_map(&maps.scales[w]);
        }
    }
    if (lane == 0) mbar_fence_init();
    __syncwarp();
    if (tid == 0 && fast && J.norm_w) {  // the norm weight is written by no kernel: requested before the wait
        mbar_arrive_expect_tx(mb + 1, 4u * Kx);
        bulk_g2s(nws, J.norm_w, 4u * Kx, mb + 1);
    }
    piece_begin(t0);
#pragma unroll
    for (int d = 0; d < D; ++d)
        if (d < ne) issue_next(d);
    pdl_wait();
    if (J.tp.wait) {  // the input's other ranks' parts are stored here by their launches
        if (tid == 0) tp_wait(J.tp, err);
        __syncthreads();
    }
    // A tagged input: the tag its words carry once this step's producers (every rank's) stored them.
    const unsigned xtag = (J.tp.tag_points && J.tp.tag_in >= 0) ? tp_tag(J.tp, J.tp.tag_in) : 0u;
    if (J.skip && *J.skip) {
        drain();
        return;
    }

    int npiece = 0;
    bool dead = false;  // a slot's wait ran out (recorded): no further waits or copies
    for (long long t = t0; t < t1;) {
        const bool first = t == t0;
        if (!first) piece_begin(t);
        t = (long long)job * M.nrb + pb;
        __syncthreads();  // the previous piece's activation and rings are no longer in use
        const float *xj = J.x ? J.x + (uint64_t)job * J.x_stride : nullptr;
        const int8_t *x8j = J.x8 ? J.x8 + (uint64_t)job * J.x_stride : nullptr;
        bool ok = true;
        const int e8 = fast ? build_activation_cp<KIND>(xj, J.norm_w, first, J.eps, Kx, xs, nws, xp, red64, mb,
                                                        (uint32_t)(npiece & 1), err, ok, xtag, J.cols, J.x_off)
                            : build_activation<KIND>(xj, x8j, J.norm_w, J.eps, J.cols, q8, xs, xp, amax_s, red64);
        ++npiece;
        if (!ok) {  // a staging copy timed out (recorded)
            drain();
            return;
        }
        unsigned long long best = 0ull;

        const int rounds = (pb - pa + Rr - 1) / Rr;
        __syncwarp();
#pragma unroll
        for (int d = 0; d < D; ++d)
            if (d >= (first ? ne : 0)) issue_next(d);
        int slot = 0;
        LaneRow one;
        one.o = row_out(J, segs, job, 0, e8);
        one.B = one.o.B;
        one.F = scale_fast(one.B);
        one.row = -1;
        one.srow = 0;
        LaneRow L[R];
#pragma unroll
        for (int r = 0; r < R; ++r) L[r] = one;
        for (int k = 0; k < rounds; ++k) {
            const int rbk = pa + gsh + k * Rr;
            const bool valid = k < kval;
            long long acc0[R], acc1[R];
            int Bv[R];
            ScaleFast Fv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                acc0[r] = acc1[r] = 0;
                if (valid) lane_row(J, segs, job, rbk * 32 * R + lane + 32 * r, e8, one, L[r]);
                Bv[r] = L[r].B;
                Fv[r] = L[r].F;
            }
            for (int c = cA; valid && c < cB; ++c) {
                if (!dead) dead = !mbar_wait_bounded_s(bars + 8u * slot, (phase >> slot) & 1u, err);
                if (!dead) {
                    phase ^= 1u << slot;
                    inflight &= ~(1u << slot);
                }
                const int ng = min(kCG, M.G - c * kCG);
                const uint32_t *xg = xp + c * kCG * M.xw;
                const unsigned char *sp = ring + (size_t)slot * sstride;
                const int soff = (c & 1) * 8;
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    const unsigned char *codes = sp + w * M.cbytes;
                    const unsigned char *scales = sp + NW * M.cbytes + w * 32 * R * kScBox;
                    if (w == 0) {
                        if (KIND == TRX_KIND_TERNARY5 && (c & 1))
                            chunk_rows<KIND, R, 8>(codes, scales, soff, lane, ng, xg, lane4x, Bv, Fv, acc0);
                        else
                            chunk_rows<KIND, R, 0>(codes, scales, soff, lane, ng, xg, lane4x, Bv, Fv, acc0);
                    } else {
                        int B2v[R];
                        ScaleFast F2v[R];
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            B2v[r] = J.B2;
                            F2v[r] = F2;
                        }
                        if (KIND == TRX_KIND_TERNARY5 && (c & 1))
                            chunk_rows<KIND, R, 8>(codes, scales, soff, lane, ng, xg, lane4x, B2v, F2v, acc1);
                        else
                            chunk_rows<KIND, R, 0>(codes, scales, soff, lane, ng, xg, lane4x, B2v, F2v, acc1);
                    }
                }
                __syncwarp();  // every lane is done with the slot before it is refilled
                if (!dead) issue_next(slot);  // the block D ahead of the one just consumed
                slot = slot + 1 == D ? 0 : slot + 1;
            }
            if (M.S > 1) {
                // The S warps of the group add their partial sums in a fixed order (exact int64).
                long long *rd = red + (size_t)(k & 1) * M.warps * 32 * NW * R;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    rd[((warp * 32 + lane) * R + r) * NW] = acc0[r];
                    if (NW == 2) rd[((warp * 32 + lane) * R + r) * NW + 1] = acc1[r];
                }
                asm volatile("bar.sync %0, %1;" ::"r"(1 + gi), "r"(M.S * 32) : "memory");
                if (sub == 0 && valid) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        acc0[r] = acc1[r] = 0;
                        for (int s2 = 0; s2 < M.S; ++s2) {
                            acc0[r] += rd[(((gi * M.S + s2) * 32 + lane) * R + r) * NW];
                            if (NW == 2) acc1[r] += rd[(((gi * M.S + s2) * 32 + lane) * R + r) * NW + 1];
                        }
                    }
                }
            }
            if (valid && sub == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (L[r].row >= 0) {
                        const unsigned long long key = finish_row(J, L[r].o, L[r].row, L[r].srow, acc0[r], acc1[r], err);
                        best = key > best ? key : best;
                    }
                }
            }
        }
        __syncwarp();
        if (J.argmax) argmax_commit(J, job, best, lane);
    }
    if (dead) drain();  // the slots whose copies never completed: one more bounded wait each
    if (!J.key_out) tp_signal(J.tp, gridDim.x);
    if (J.token || J.key_out) {  // greedy tokens: the last CTA to arrive hands out each job's key
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            amax_s[1] = atomicAdd(J.arg_cnt, 1u) == gridDim.x - 1 ? 1u : 0u;
        }
        __syncthreads();
        if (amax_s[1]) {
            __threadfence();
            for (int j = tid; j < J.njobs; j += blockDim.x) {
                const unsigned long long k = atomicExch(J.argmax + j, 0ull);
                if (J.token) J.token[j] = k ? (int)(0xffffffffu - (uint32_t)k) : -1;
                if (J.key_out) {
                    J.key_out[j] = k;
                    for (int r = 0; r < J.tp.world; ++r)
                        if (r != J.tp.rank && J.tp.dst[r])
                            reinterpret_cast<unsigned long long *>(J.tp.dst[r])[J.tp.offset + j] = k;
                }
            }
            if (tid == 0) *J.arg_cnt = 0u;
            if (J.key_out && J.tp.signal[0]) {  // this launch is complete on this rank
                __syncthreads();
                if (tid == 0) {
                    __threadfence_system();
                    for (int r = 0; r < J.tp.world; ++r) atomicAdd_system(J.tp.signal[r], 1u);
                }
            }
        }
    }
}

// fp-mode kernel (model/fastref.py:103-125, HybridRef.matmul): Y[t] = X[t] . W^T in fp32 for the
// launch's J.njobs rows of X (x_stride / y_stride apart), W = (code - 1) * scale (exact in the fp16
// weight cache the reference builds).  Thread per (row, group): the group's 128 codes are decoded
// once per chunk of TT rows of X staged in shared memory, each row's group sum (code - 1) * x in
// fp32 times the fp32 scale, then the groups added in group order (+ the optional residual).
template <int KIND>
__global__ void __launch_bounds__(256) tmv_fp_kernel(MvJobs J, int TR, int TT, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_trigger();
    pdl_wait();
    const int G = J.cols / 128, K = J.cols;
    float *xs = reinterpret_cast<float *>(smem);  // [TT][K]
    float *part = xs + (size_t)TT * K;            // [TT][TR][G + 1]
    const int sbytes = (G + 15) / 16 * 32;
    const int rb = sbytes + ((KIND == TRX_KIND_TERNARY5 ? 26 : 32) * G + 31) / 32 * 32;
    const int units = TR * G;
    float *const y = reinterpret_cast<float *>(J.seg[0].y);
    for (int t0 = 0; t0 < J.njobs; t0 += TT) {
        const int nt = min(TT, J.njobs - t0);
        __syncthreads();  // the previous chunk is done with xs and part
        for (int i = threadIdx.x; i < nt * K; i += blockDim.x)
            xs[i] = J.x[(uint64_t)(t0 + i / K) * J.x_stride + i % K];
        __syncthreads();
        for (int r0 = blockIdx.x * TR; r0 < J.rows; r0 += gridDim.x * TR) {
            const int nr = min(TR, J.rows - r0);
            for (int u = threadIdx.x; u < units; u += blockDim.x) {
                const int rr = u / G, g = u % G;
                if (rr >= nr) continue;
                const uint8_t *row = J.w + (uint64_t)(r0 + rr) * rb;
                float s[4] = {0.f, 0.f, 0.f, 0.f};
                auto add = [&](int l, int d) {  // weight l of the group is d - 1
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        if (t < nt) s[t] = __fadd_rn(s[t], __fmul_rn((float)(d - 1), xs[t * K + g * 128 + l]));
                };
                if (KIND == TRX_KIND_TERNARY5) {
                    const uint8_t *cb = row + sbytes + 26 * g;
                    for (int i = 0; i < 26; ++i) {
                        uint32_t b = cb[i];
                        for (int k = 0; k < 5; ++k) {
                            const int l = 5 * i + k;
                            const int d = (int)(b % 3u);
                            b /= 3u;
                            if (l < 128) add(l, d);
                        }
                    }
                } else {
                    const uint8_t *cb = row + sbytes + 32 * g;
                    for (int l = 0; l < 128; ++l) add(l, (cb[l >> 2] >> (2 * (l & 3))) & 3);
                }
                const float sc = __half2float(reinterpret_cast<const __half *>(row)[g]);
                for (int t = 0; t < nt; ++t) part[(t * TR + rr) * (G + 1) + g] = __fmul_rn(s[t], sc);
            }
            __syncthreads();
            for (int i = threadIdx.x; i < nt * nr; i += blockDim.x) {
                const int t = i / nr, rr = i - t * nr;
                float a = 0.f;
                for (int g = 0; g < G; ++g) a = __fadd_rn(a, part[(t * TR + rr) * (G + 1) + g]);
                const uint64_t o = (uint64_t)(t0 + t) * J.y_stride + r0 + rr;
                if (J.seg[0].resid) a = __fadd_rn(J.seg[0].resid[o], a);
                y[o] = a;
            }
            __syncthreads();
        }
    }
}

// Standalone quantiser (trx_quantize_pow2): one CTA, grid-stride.
__global__ void __launch_bounds__(1024) quantize_kernel(const float *x, int n, int8_t *x8, int *e8_out) {
    __shared__ uint32_t amax_s;
    pdl_trigger();
    pdl_wait();
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
    pdl_trigger();
    pdl_wait();
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

// Per-device launch facts: SM count and the shared memory the driver reserves per block (the
// dynamic shared memory starts at that window address).
struct DevInfo {
    int sms, reserved;
};

static DevInfo dev_info() {
    static DevInfo info[64];
    static bool have[64];
    int dev = 0;
    cudaGetDevice(&dev);
    dev &= 63;
    if (!have[dev]) {
        int v = 0;
        info[dev].sms = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0 ? v : 148;
        v = 0;
        info[dev].reserved =
            cudaDeviceGetAttribute(&v, cudaDevAttrReservedSharedMemoryPerBlock, dev) == cudaSuccess ? v : 1024;
        have[dev] = true;
    }
    return info[dev];
}

static int num_sms() { return dev_info().sms; }
int device_sms() { return dev_info().sms; }
int device_reserved_smem() { return dev_info().reserved; }

// Plan a launch: chunks, rows per lane, tasks (rows split over tasks only when the launch has too
// few row blocks to give every warp slot of the GPU one), warps and ring depth that fit shared
// memory.
// The rings and shared-memory carve-up of a launch whose row-block split is decided (M.R, M.nrb,
// M.grid, M.D set): the warps, the regions and the prologue's staging area.
static bool plan_rings(const MvJobs &J, int reserved, bool split, long long rbc, MvGeom &M) {
    const bool t5 = J.kind == TRX_KIND_TERNARY5;
    const int nw = M.nw;
    M.cbytes = 32 * M.R * M.cb;
    M.slot = nw * 32 * M.R * (M.cb + kScBox);
    int fixed = M.G * M.xw * 4 + 64 * 4 + 16 + 16 + kMaxSegs * (int)sizeof(MvSeg);
    fixed = (fixed + 7) / 8 * 8;
    M.bar_off = fixed;
    fixed = (fixed + kMaxWarps * kMaxD * 8 + 127) / 128 * 128;
    M.red_off = fixed;
    fixed += split ? 2 * kMaxWarps * 32 * nw * M.R * 8 : 0;
    M.fixed = (fixed + 127) / 128 * 128;
    const int ring = M.D * M.slot;  // one warp's ring
    // The trit5 LUT sits at shared-window address 0x10000 (its PRMT-built addresses need no add):
    // ring region A below it, region C above it.  2-bit: region A only.
    const int lut_off = 0x10000 - reserved, c_off = lut_off + kLutBytes;
    int na_max, nc_max;
    if (t5) {
        if (M.fixed > lut_off) return false;
        na_max = (lut_off - M.fixed) / ring;
        nc_max = (kSmemMax - c_off) / ring;
    } else {
        na_max = (kSmemMax - M.fixed) / ring;
        nc_max = 0;
    }
    M.warps = std::min(kMaxWarps, na_max + nc_max);
    if (M.warps < 2) return false;
    M.S = 1;
    if (split) {
        int w = 1;
        while (w * 2 <= M.warps) w *= 2;  // sharing groups need a power-of-two warp count
        M.warps = w;
        // Rr row blocks at a time, S = warps/Rr warps per row block: the fewest chunk steps per warp,
        // ceil(rbc/Rr) rounds of ceil(nch/S) chunks; ties go to the larger Rr (fewer sharers).
        int bestR = 1;
        long long best = -1;
        for (int Rr = 1; Rr <= M.warps; Rr *= 2) {
            const int S = M.warps / Rr;
            const long long cost = ((rbc + Rr - 1) / Rr) * (long long)((M.nch + S - 1) / S);
            if (best < 0 || cost <= best) {
                best = cost;
                bestR = Rr;
            }
        }
        M.S = M.warps / bestR;
    }
    M.cpt = (M.nch + M.S - 1) / M.S;
    M.na = std::min(na_max, M.warps);
    const int nc = M.warps - M.na;
    M.base = t5 ? reserved : 0;
    M.smem = t5 ? c_off + nc * ring : M.fixed + M.warps * ring;
    // The quantiser's staging (q8, then x as fp32) lives in the larger ring region, idle then.
    // The staging area: the last bands of the region with the wider band (a band is the slot d of
    // every warp of the region), as few as hold [q8 bytes][x fp32][norm weight fp32]; float4 loads
    // need 16-byte aligned rows, else only the q8 bytes (the global prologue path).
    M.sreg = nc > M.na ? 1 : 0;
    const int band = (M.sreg ? nc : M.na) * M.slot;
    const bool aligned = !(reinterpret_cast<uintptr_t>(J.x) & 15) && !(reinterpret_cast<uintptr_t>(J.norm_w) & 15) &&
                         !(J.x_stride & 3);
    const int Kx = J.x_cols ? J.x_cols : J.cols;  // elements of x
    const int need = aligned ? (J.cols + 15) / 16 * 16 + 4 * Kx * (J.norm_w ? 2 : 1) : J.cols;
    const int own = (M.smem + 127) / 128 * 128;
    if (own + need <= kSmemMax) {  // a region of its own after the rings: no slot waits for the prologue
        M.stage_off = own;
        M.stage = need;
        M.ebl = M.D;
        M.xfast = aligned ? 1 : 0;
        M.smem = own + need;
        return true;
    }
    const int nb = std::min(M.D, (need + band - 1) / band);
    M.stage = nb * band;
    if (M.stage < J.cols) return false;
    M.stage_off = (M.sreg ? c_off : M.fixed) + (M.D - nb) * band;
    M.ebl = M.D - nb;
    if (!aligned) M.stage = J.cols;  // no x staging in shared memory: the global prologue path
    M.xfast = aligned && M.stage >= need ? 1 : 0;
    return M.smem <= kSmemMax;
}

bool plan_matvec(const MvJobs &J, int nw, int sms, int reserved, MvGeom &M) {
    const int kind = J.kind;
    const bool t5 = kind == TRX_KIND_TERNARY5;
    M.G = J.cols / 128;
    M.nch = (M.G + kCG - 1) / kCG;
    M.sbytes = (M.G + 15) / 16 * 32;
    M.rb = M.sbytes + ((t5 ? 26 : 32) * M.G + 31) / 32 * 32;
    M.nw = nw;
    M.xw = t5 ? kXwT5 : kXw2b;
    M.cb = t5 ? kCbT5 : kCb2b;
    // Two slots per warp: 16 warps fit (measured on B200, a single 2-bit tensor: depth 2 with 16 warps
    // against depth 3 with 14 streamed the config-0 batch at 4.80 against 4.40 TB/s).
    M.D = t5 ? (nw == 2 ? 2 : TRX_MV_D_T5) : 2;
    M.wjob = (J.njobs > 1 && J.w_stride != 0) ? 1 : 0;
    // Row blocks are dealt to CTAs; when a CTA gets fewer row blocks than it has warps, the warps
    // share row blocks (S per row block, chunks split between them, sums combined in shared memory)
    // and a lane owns one row; otherwise R rows.
    bool split = false;
    long long rbc = 0;
    for (int R = nw == 2 ? 1 : (t5 ? TRX_MV_R_T5 : TRX_MV_R_2B);; R = 1) {
        M.R = R;
        M.nrb = (J.rows + 32 * R - 1) / (32 * R);
        const long long rbt = (long long)J.njobs * M.nrb;
        M.grid = (int)std::min<long long>(sms, rbt);
        rbc = (rbt + M.grid - 1) / M.grid;
        split = rbc < kMaxWarps && M.nch > 1;
        if (!split || R == 1) break;
    }
    // A decode-size launch (warps share row blocks) whose CTA share of the weights is more than the
    // rings hold at the default depth (with the warps that depth leaves, a power of two): shallower
    // rings when that gives the full warp count with the prologue's staging in a region of its own,
    // so the weights still go in flight before the dependency wait and twice the warps decode them.
    // (Measured on B200, 8B decode: 1.854 -> 1.810 ms per token, from the gate/up pair; making the
    // rings shallower where the default rings hold the whole share made the step slower.)
    bool default_holds = false;
    {
        MvGeom T = M;
        if (plan_rings(J, reserved, split, rbc, T))
            default_holds = (long long)T.warps * T.D * T.slot >= (rbc * 32 * T.R) * (long long)T.rb * T.nw;
    }
    if (split && !default_holds) {
        for (int D = M.D - 1; D >= 1; --D) {
            MvGeom T = M;
            T.D = D;
            if (plan_rings(J, reserved, split, rbc, T) && T.warps == kMaxWarps && T.ebl == T.D) {
                M = T;
                return true;
            }
        }
    }
    return plan_rings(J, reserved, split, rbc, M);
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (the library links
// only the CUDA runtime).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static std::atomic<EncodeTiledFn> fn{nullptr};
    EncodeTiledFn f = fn.load(std::memory_order_acquire);
    if (!f) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f = reinterpret_cast<EncodeTiledFn>(p);
        fn.store(f, std::memory_order_release);
    }
    return f;
}

// A uint8 box map over [njobs][rows][rb] bytes (job stride s1 bytes), box {bx bytes, by rows, 1}.
static bool encode_box(CUtensorMap *m, const void *base, uint64_t rb, uint64_t rows, uint64_t njobs, uint64_t s1,
                       uint32_t bx, uint32_t by) {
    const EncodeTiledFn f = encode_tiled();
    if (!f) return false;
    const cuuint64_t dims[3] = {rb, rows, njobs};
    const cuuint64_t strides[2] = {rb, s1};
    const cuuint32_t box[3] = {bx, by, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static trx_status encode_maps(const MvJobs &J, const MvGeom &M, MvMaps &maps) {
    memset(&maps, 0, sizeof(maps));
    const uint64_t njobs = M.wjob ? (uint64_t)J.njobs : 1;
    const uint64_t s1 = M.wjob ? J.w_stride : (uint64_t)J.rows * M.rb;
    if (s1 % 16) return TRX_ERR_UNSUPPORTED;
    for (int w = 0; w < M.nw; ++w) {
        const void *base = w ? J.w2 : J.w;
        if (!encode_box(&maps.codes[w], base, M.rb, J.rows, njobs, s1, M.cb, 32 * M.R) ||
            !encode_box(&maps.scales[w], base, M.rb, J.rows, njobs, s1, kScBox, 32 * M.R))
            return TRX_ERR_CUDA;
    }
    return TRX_OK;
}

template <int KIND, int NW, int R, int D>
static trx_status launch_tmv_d(const MvJobs &J, const MvGeom &M, const MvMaps &maps, uint32_t *err, cudaStream_t st) {
    static DevBits configured{0};  // devices whose attribute is set
    const cudaError_t e = once_per_device(configured, [] {
        return cudaFuncSetAttribute(tmv_kernel<KIND, NW, R, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
    });
    if (e != cudaSuccess) return note_cuda(e);
    return note_cuda(
        launch_kernel(tmv_kernel<KIND, NW, R, D>, dim3(M.grid), dim3(M.warps * 32), M.smem, st, maps, J, M, err));
}

// The depths plan_matvec gives: the default 2, or 1 for a decode-size launch.
template <int KIND, int NW, int R>
static trx_status launch_tmv(const MvJobs &J, const MvGeom &M, const MvMaps &maps, uint32_t *err, cudaStream_t st) {
    if (M.D == 1) return launch_tmv_d<KIND, NW, R, 1>(J, M, maps, err, st);
    if (M.D == 2) return launch_tmv_d<KIND, NW, R, 2>(J, M, maps, err, st);
    return TRX_ERR_UNSUPPORTED;
}

bool matvec_launchable(const MvJobs &J) {
    MvGeom M;
    const DevInfo di = dev_info();
    if (!plan_matvec(J, J.w2 ? 2 : 1, di.sms, di.reserved, M)) return false;
    return !(((J.tp.tag_points && J.tp.tag_in >= 0) || J.x_cols) && (!M.xfast || !J.x || J.njobs != 1));
}

trx_status launch_matvec(const MvJobs &J, const uint32_t *lut, uint32_t *err, cudaStream_t st) {
    (void)lut;  // the trit5 LUT is built in each CTA's shared memory
    MvGeom M;
    const DevInfo di = dev_info();
    const int nw = J.w2 ? 2 : 1;
    if (!plan_matvec(J, nw, di.sms, di.reserved, M)) return TRX_ERR_UNSUPPORTED;
    // A tagged input, or a K-segment of a wider input, is read only by the staged prologue, one job at
    // a time.
    if (((J.tp.tag_points && J.tp.tag_in >= 0) || J.x_cols) && (!M.xfast || !J.x || J.njobs != 1))
        return TRX_ERR_UNSUPPORTED;
    MvMaps maps;
    const trx_status s = encode_maps(J, M, maps);
    if (s != TRX_OK) return s;
    if (J.kind == TRX_KIND_TERNARY5) {
        if (nw == 2) return launch_tmv<TRX_KIND_TERNARY5, 2, 1>(J, M, maps, err, st);
#if TRX_MV_R_T5 > 1
        if (M.R == 2) return launch_tmv<TRX_KIND_TERNARY5, 1, 2>(J, M, maps, err, st);
#endif
        return launch_tmv<TRX_KIND_TERNARY5, 1, 1>(J, M, maps, err, st);
    }
    if (nw == 2) return launch_tmv<TRX_KIND_TERNARY, 2, 1>(J, M, maps, err, st);
#if TRX_MV_R_2B > 1
    if (M.R == 2) return launch_tmv<TRX_KIND_TERNARY, 1, 2>(J, M, maps, err, st);
#endif
    return launch_tmv<TRX_KIND_TERNARY, 1, 1>(J, M, maps, err, st);
}

trx_status launch_matvec_fp(const MvJobs &J, uint32_t *err, cudaStream_t st) {
    const int G = J.cols / 128;
    const int TR = 16;
    // Rows of X per chunk: up to 4 while the chunk and the group partials fit shared memory.
    int TT = 4;
    auto bytes = [&](int tt) { return (size_t)tt * J.cols * 4 + (size_t)tt * TR * (G + 1) * 4; };
    while (TT > 1 && bytes(TT) > (size_t)kSmemMax) --TT;
    const size_t smem = bytes(TT);
    if (smem > (size_t)kSmemMax || J.njobs < 1) return TRX_ERR_UNSUPPORTED;
    int grid = (J.rows + TR - 1) / TR;
    if (grid > num_sms() * 4) grid = num_sms() * 4;
    cudaError_t e;
    if (J.kind == TRX_KIND_TERNARY5) {
        e = cudaFuncSetAttribute(tmv_fp_kernel<TRX_KIND_TERNARY5>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return note_cuda(e);
        e = launch_kernel(tmv_fp_kernel<TRX_KIND_TERNARY5>, dim3(grid), dim3(256), smem, st, J, TR, TT, err);
    } else {
        e = cudaFuncSetAttribute(tmv_fp_kernel<TRX_KIND_TERNARY>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return note_cuda(e);
        e = launch_kernel(tmv_fp_kernel<TRX_KIND_TERNARY>, dim3(grid), dim3(256), smem, st, J, TR, TT, err);
    }
    return note_cuda(e);
}

trx_status launch_quantize(const float *x, int n, int8_t *x8, int *e8, cudaStream_t st) {
    return note_cuda(launch_kernel(quantize_kernel, dim3(1), dim3(1024), 0, st, x, n, x8, e8));
}

// The quantiser over tagged words (a tensor-parallel gather point): every thread first polls its
// words until they carry the point's tag of this step (bounded; TRX_DEV_TIMEOUT and zeros when a
// wait runs out), then the max and the quantiser read the values (the low halves).  The words do
// not change until this launch's successors have run, so they are read again without a poll.
__global__ void __launch_bounds__(1024) quantize_tagged_kernel(const unsigned long long *xt, int n, int8_t *x8,
                                                               int *e8_out, TpXfer tp, uint32_t *err) {
    __shared__ uint32_t amax_s;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) amax_s = 0;
    const unsigned tag = tp_tag(tp, tp.tag_in);
    bool bad = false;
    unsigned long long t0 = 0ull;
    for (int k = threadIdx.x; k < n && !bad; k += blockDim.x) {
        unsigned long long w;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(xt + k) : "memory");
        while ((unsigned)(w >> 32) != tag) {
            if (!t0) {
                t0 = global_ns();
            } else if (global_ns() - t0 > kWaitNs) {
                atomicOr(err, TRX_DEV_TIMEOUT);
                bad = true;
                break;
            }
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(xt + k) : "memory");
        }
    }
    if (__syncthreads_or(bad ? 1 : 0)) {
        for (int k = threadIdx.x; k < n; k += blockDim.x) x8[k] = 0;
        if (threadIdx.x == 0) *e8_out = 0;
        return;
    }
    uint32_t m = 0;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        unsigned long long w;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(xt + k) : "memory");
        const uint32_t a = (uint32_t)w & 0x7fffffffu;  // |value| bits
        m = a > m ? a : m;
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) atomicMax(&amax_s, m);
    __syncthreads();
    const uint32_t amax = amax_s;
    const int e8 = amax ? frexp_exp(__uint_as_float(amax)) - 7 : 0;
    const float inv = pow2f(-e8);
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        unsigned long long w;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(xt + k) : "memory");
        x8[k] = amax ? quant_one(__uint_as_float((uint32_t)w), inv) : (int8_t)0;
    }
    if (threadIdx.x == 0) *e8_out = e8;
}

trx_status launch_quantize_tagged(const void *x, int n, int8_t *x8, int *e8, const TpXfer &tp, uint32_t *err,
                                  cudaStream_t st) {
    if (!tp.tag_points || tp.tag_in < 0 || !tp.step) return TRX_ERR_ARG;
    return note_cuda(launch_kernel(quantize_tagged_kernel, dim3(1), dim3(1024), 0, st,
                                   static_cast<const unsigned long long *>(x), n, x8, e8, tp, err));
}

trx_status launch_validate_t5(const uint8_t *w, int rows, int cols, uint32_t *err, cudaStream_t st) {
    const int G = cols / 128;
    const int sb = (G + 15) / 16 * 32;
    const int rb = sb + (26 * G + 31) / 32 * 32;
    long long total = (long long)rows * 26 * G;
    int grid = (int)((total + 255) / 256);
    if (grid > num_sms() * 8) grid = num_sms() * 8;
    if (grid < 1) grid = 1;
    return note_cuda(launch_kernel(validate_t5_kernel, dim3(grid), dim3(256), 0, st, w, rows, rb, sb, G, err));
}

trx_status launch_build_lut(uint32_t *lut, cudaStream_t st) {
    build_lut_kernel<<<kLutWords / 256, 256, 0, st>>>(lut);
    return note_cuda(cudaGetLastError());
}

size_t lut_bytes() { return kLutBytes; }

}  // namespace trx
