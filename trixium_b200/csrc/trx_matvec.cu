// Ternary matvec kernels for B200 (sm_100a): the TriXium engine's group-128 matvec over the
// converter's row packets (2-bit and 5-trit codes), bit-exact with model/bitexact.py:101-119,
// with the firmware's float wrapper (quantise -> engine -> scale, firmware/infer_float.c:398)
// fused in, and the fp-mode projection of model/fastref.py:103-125.
//
// Work decomposition (one launch = one "job list"; a job is one tensor against one input):
//  * A row tile of TR consecutive rows is one contiguous byte range of the packed tensor; one
//    elected thread moves it global -> shared with a 1-D TMA bulk copy (cp.async.bulk), double
//    buffered against the tile being decoded, completion tracked by an mbarrier.
//  * Thread (slot, g) owns group g of every row it touches (LS lanes per row-slot, RS slots).
//    The activation's permuted int8 words for its group live in registers for the whole job,
//    so the inner loop reads only codes and the trit5 LUT from shared memory.
//  * Group sums are exact int32 (dp4a / dp2a); the scale/shift contribution is int64; row
//    sums are reduced across the slot's lanes (warp shuffles, then a shared int64 atomic when a
//    slot spans warps) and finalised by one thread per row (>> R, overflow checks, epilogue).
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

// Shared-memory plan -------------------------------------------------------------------------------
constexpr int kLutWords = 256 * 64;              // 256 entries x 256-byte stride (32 replicas used)
constexpr int kLutBytes = kLutWords * 4;         // 64 KiB
constexpr int kXWordsT5 = 40;                    // 26 dp4a words + 14 dp2a words per group
constexpr int kXWords2b = 32;
constexpr int kStageBudget = 24 * 1024;          // bytes per stage buffer (all tensors of a tile)

struct __align__(16) SmemHead {
    uint64_t bar[2];
    uint32_t amax_bits;
    int e8;
    int pad[2];
};

// Geometry of one launch, derived on the host (trx_plan) and passed by value.
struct MvGeom {
    int G;        // groups per row
    int LS;       // lanes per row-slot (power of two <= 32, or a multiple of 32)
    int RS;       // row-slots per CTA
    int TR;       // rows per tile
    int rb;       // row packet bytes
    int sbytes;   // scale-region bytes
    int nw;       // tensors per tile (2 for SwiGLU)
    int xwords;   // permuted activation words per group
    int smem;     // dynamic shared bytes
    int tiles;    // tiles per job
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
// sequential fp32 partials in increasing index order, then the halving tree.  Threads 0..63
// compute the partials; warps 0 and 1 then run the tree through shared memory.
__device__ float block_sumsq64(const float *x, int n, float *red64) {
    const int t = threadIdx.x;
    if (t < 64) {
        float p = 0.f;
        for (int i = t; i < n; i += 64) {
            const float v = __ldg(x + i);
            p = __fadd_rn(p, __fmul_rn(v, v));
        }
        red64[t] = p;
    }
    __syncthreads();
    for (int w = 32; w >= 1; w >>= 1) {
        if (t < w) red64[t] = __fadd_rn(red64[t], red64[t + w]);
        __syncthreads();
    }
    const float ss = red64[0];
    __syncthreads();
    return ss;
}

// Build the permuted int8 activation for one job in shared memory.
// q8: K bytes (scratch), xp: G*xwords words, xsum: G ints.  Returns e8 (also in head->e8).
template <int KIND>
__device__ int build_activation(const float *x, const int8_t *x8g, const float *nw, float eps, int K,
                                int8_t *q8, uint32_t *xp, int *xsum, SmemHead *head, float *red64) {
    const int t = threadIdx.x, nt = blockDim.x;
    int e8 = 0;
    if (x8g) {
        for (int k = t; k < K; k += nt) q8[k] = x8g[k];
    } else {
        float r = 0.f;
        if (nw) {
            const float ss = block_sumsq64(x, K, red64);
            r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
        }
        if (t == 0) head->amax_bits = 0u;
        __syncthreads();
        uint32_t m = 0;
        for (int k = t; k < K; k += nt) {
            const uint32_t a = __float_as_uint(fabsf(prologue_value(x, nw, r, k)));
            m = a > m ? a : m;
        }
        for (int o = 16; o; o >>= 1) {
            const uint32_t o2 = __shfl_xor_sync(0xffffffffu, m, o);
            m = o2 > m ? o2 : m;
        }
        if ((t & 31) == 0) atomicMax(&head->amax_bits, m);
        __syncthreads();
        const uint32_t amax = head->amax_bits;
        if (amax == 0u) {
            e8 = 0;
            for (int k = t; k < K; k += nt) q8[k] = 0;
        } else {
            e8 = frexp_exp(__uint_as_float(amax)) - 7;
            const float inv = pow2f(-e8);
            for (int k = t; k < K; k += nt) q8[k] = quant_one(prologue_value(x, nw, r, k), inv);
        }
    }
    __syncthreads();
    const int G = K / 128;
    if (KIND == TRX_KIND_TERNARY5) {
        // Per group: words 0..25 = bytes (x[5i], x[5i+1], x[5i+2], x[5i+3]);
        // words 26..38 = 16-bit pairs (y[2j], y[2j+1]) with y[i] = x[5i+4] - 3*x[5i+3];
        // lanes 128/129 (digits 3/4 of byte 25) see x = 0.
        for (int idx = t; idx < G * kXWordsT5; idx += nt) {
            const int g = idx / kXWordsT5, j = idx % kXWordsT5;
            const int8_t *qg = q8 + g * 128;
            uint32_t w = 0;
            if (j < 26) {
                for (int k = 0; k < 4; ++k) {
                    const int l = 5 * j + k;
                    const uint32_t b = l < 128 ? (uint32_t)(uint8_t)qg[l] : 0u;
                    w |= b << (8 * k);
                }
            } else {
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
        for (int idx = t; idx < G * kXWords2b; idx += nt) {
            const int g = idx / kXWords2b, j = idx % kXWords2b;
            const int wq = j >> 2, p = j & 3;
            const int8_t *qg = q8 + g * 128;
            uint32_t w = 0;
            for (int b = 0; b < 4; ++b) w |= (uint32_t)(uint8_t)qg[16 * wq + 4 * b + p] << (8 * b);
            xp[idx] = w;
        }
    }
    for (int g = t; g < G; g += nt) {
        int s = 0;
        for (int k = 0; k < 128; ++k) s += q8[g * 128 + k];
        xsum[g] = s;
    }
    if (t == 0) head->e8 = e8;
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
    int acc = 0;
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
                acc = dp4a_ss(E[i], xa[4 * q + i], acc);
            }
        }
        if (nb == 4) {
            const uint32_t d01 = __byte_perm(E[0], E[1], 0x0073u);
            const uint32_t d23 = __byte_perm(E[2], E[3], 0x0073u);
            const uint32_t D = ((__byte_perm(d01, d23, 0x5410u) * 11u) >> 5) & 0x03030303u;
            acc = dp2a_lo(yy[2 * q], D, acc);
            acc = dp2a_hi(yy[2 * q + 1], D, acc);
        } else {
            const uint32_t D = ((__byte_perm(E[0], E[1], 0x0073u) * 11u) >> 5) & 0x03030303u;
            acc = dp2a_lo(yy[2 * q], D, acc);
        }
    }
    return acc;
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

// 64-bit sum over `width` consecutive lanes (width a power of two <= 32).
__device__ __forceinline__ long long slot_reduce(long long v, int width) {
    for (int o = width >> 1; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
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

// The matvec kernel ---------------------------------------------------------------------------------
template <int KIND>
__global__ void __launch_bounds__(512) tmv_kernel(MvJobs J, MvGeom M, const uint32_t *lut_g, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int G = M.G;

    // Carve shared memory.
    unsigned char *p = smem;
    char *lut = nullptr;
    if (KIND == TRX_KIND_TERNARY5) {
        lut = reinterpret_cast<char *>(p);
        p += kLutBytes;
    }
    unsigned char *const stage0 = p;  // two stage buffers, stage0 + buf * stage_bytes
    const int stage_bytes = M.TR * M.rb * M.nw;
    p += 2 * stage_bytes;
    uint32_t *xp = reinterpret_cast<uint32_t *>(p);
    p += G * M.xwords * 4;
    int *xsum = reinterpret_cast<int *>(p);
    p += ((G * 4 + 15) / 16) * 16;
    long long *red = reinterpret_cast<long long *>(p);
    p += (M.TR * M.nw * 8 + 15) / 16 * 16;
    float *red64 = reinterpret_cast<float *>(p);
    p += 64 * 4;
    SmemHead *head = reinterpret_cast<SmemHead *>(p);
    p += sizeof(SmemHead);
    int8_t *q8 = reinterpret_cast<int8_t *>(p);

    const int total = J.njobs * M.tiles;
    const int t_begin = (int)((long long)blockIdx.x * total / gridDim.x);
    const int t_end = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    if (t_begin >= t_end) return;

    if (tid == 0) {
        mbar_init(&head->bar[0], 1);
        mbar_init(&head->bar[1], 1);
        mbar_fence_init();
    }
    __syncthreads();

    auto issue = [&](int tile, int buf) {
        const int job = tile / M.tiles, tt = tile % M.tiles;
        const int r0 = tt * M.TR;
        const int nr = min(M.TR, J.rows - r0);
        const uint32_t bytes = (uint32_t)nr * (uint32_t)M.rb;
        fence_proxy_async();
        mbar_arrive_expect_tx(&head->bar[buf], bytes * M.nw);
        const uint8_t *src = J.w + (uint64_t)job * J.w_stride + (uint64_t)r0 * M.rb;
        bulk_g2s(stage0 + buf * stage_bytes, src, bytes, &head->bar[buf]);
        if (M.nw == 2) {
            const uint8_t *src2 = J.w2 + (uint64_t)job * J.w_stride + (uint64_t)r0 * M.rb;
            bulk_g2s(stage0 + buf * stage_bytes + (size_t)M.TR * M.rb, src2, bytes, &head->bar[buf]);
        }
    };

    if (tid == 0) issue(t_begin, 0);

    // The trit5 LUT: copied from the context's global table (replicated, 256-byte stride).
    if (KIND == TRX_KIND_TERNARY5) {
        const uint4 *src = reinterpret_cast<const uint4 *>(lut_g);
        uint4 *dst = reinterpret_cast<uint4 *>(lut);
        for (int i = tid; i < kLutBytes / 16; i += blockDim.x) dst[i] = src[i];
    }

    const int slot = tid / M.LS;
    const int g = tid % M.LS;
    const bool active = (slot < M.RS) && (g < G);
    const uint32_t lane4 = (uint32_t)lane * 4u;

    uint32_t xr[kXWordsT5 > kXWords2b ? kXWordsT5 : kXWords2b];
    int xs = 0;
    int e8 = 0;
    int cur_job = -1;
    bool ok = true;

    for (int tile = t_begin, it = 0; tile < t_end; ++tile, ++it) {
        const int buf = it & 1;
        const int job = tile / M.tiles, tt = tile % M.tiles;
        if (job != cur_job) {
            const float *xj = J.x ? J.x + (uint64_t)job * J.x_stride : nullptr;
            const int8_t *x8j = J.x8 ? J.x8 + (uint64_t)job * J.x_stride : nullptr;
            e8 = build_activation<KIND>(xj, x8j, J.norm_w, J.eps, J.cols, q8, xp, xsum, head, red64);
            if (active) {
#pragma unroll
                for (int i = 0; i < (KIND == TRX_KIND_TERNARY5 ? kXWordsT5 : kXWords2b); ++i)
                    xr[i] = xp[g * M.xwords + i];
                xs = xsum[g];
            }
            cur_job = job;
        }
        // Prefetch the next tile into the other buffer (consumed two iterations ago).
        if (tid == 0 && tile + 1 < t_end) issue(tile + 1, buf ^ 1);
        for (int i = tid; i < M.TR * M.nw; i += blockDim.x) red[i] = 0;
        __syncthreads();
        if (!mbar_wait_bounded(&head->bar[buf], (it >> 1) & 1, err)) {
            ok = false;
        }
        if (!__syncthreads_and(ok)) return;  // a copy never landed: give up on this CTA

        const int r0 = tt * M.TR;
        const int nr = min(M.TR, J.rows - r0);
        const unsigned char *sb = stage0 + buf * stage_bytes;
        for (int w = 0; w < M.nw; ++w) {
            const int B = w ? J.B2 : J.B;
            const int passes = (M.TR + M.RS - 1) / M.RS;
            for (int pass = 0; pass < passes; ++pass) {  // warp-uniform trip count
                const int rr = pass * M.RS + slot;
                long long c = 0;
                if (active && rr < nr) {
                    const unsigned char *row = sb + ((size_t)w * M.TR + rr) * M.rb;
                    const uint32_t sbits = reinterpret_cast<const uint16_t *>(row)[g];
                    int gs;
                    if (KIND == TRX_KIND_TERNARY5)
                        gs = gsum_t5(row + M.sbytes + 26 * g, g & 1, lut, lane4, xr, xr + 26) - xs;
                    else
                        gs = gsum_2b(row + M.sbytes + 32 * g, xr) - xs;
                    c = group_contrib(gs, sbits, B);
                }
                // Reduce across the slot's lanes.
                if (M.LS <= 32) {
                    c = slot_reduce(c, M.LS);
                    if (active && g == 0 && rr < nr) red[w * M.TR + rr] = c;
                } else {
                    c = slot_reduce(c, 32);
                    if (lane == 0 && slot < M.RS && rr < nr)
                        atomicAdd(reinterpret_cast<unsigned long long *>(&red[w * M.TR + rr]),
                                  (unsigned long long)c);
                }
            }
        }
        __syncthreads();
        // Finalise the tile's rows.
        for (int rr = tid; rr < nr; rr += blockDim.x) {
            const int row = r0 + rr;
            const long long a = red[rr];
            bool bad = (a >= (1ll << 47)) || (a <= -(1ll << 47)) || ((a >> J.R) >= (1ll << 31)) ||
                       ((a >> J.R) <= -(1ll << 31));
            if (J.out == OUT_I32) {
                reinterpret_cast<int *>(J.y)[(uint64_t)job * J.y_stride + row] = (int)(a >> J.R);
            } else if (J.out == OUT_F32) {
                float v = row_float(a, J.R, e8, J.B);
                if (J.resid) v = __fadd_rn(J.resid[row], v);
                reinterpret_cast<float *>(J.y)[(uint64_t)job * J.y_stride + row] = v;
            } else {  // OUT_SWIGLU
                const long long a2 = red[M.TR + rr];
                bad = bad || (a2 >= (1ll << 47)) || (a2 <= -(1ll << 47)) || ((a2 >> J.R2) >= (1ll << 31)) ||
                      ((a2 >> J.R2) <= -(1ll << 31));
                const float gv = row_float(a, J.R, e8, J.B);
                const float uv = row_float(a2, J.R2, e8, J.B2);
                reinterpret_cast<float *>(J.y)[(uint64_t)job * J.y_stride + row] = __fmul_rn(silu_f32(gv), uv);
            }
            if (bad) atomicOr(err, TRX_DEV_OVERFLOW);
        }
        __syncthreads();
    }
}

// fp-mode kernel (model/fastref.py:103-125): thread per (row, group); x fp32 in shared memory;
// per-group fp32 sums of (code-1)*x, times the fp32 scale, reduced over groups in group order.
template <int KIND>
__global__ void __launch_bounds__(256) tmv_fp_kernel(MvJobs J, MvGeom M, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);
    float *part = xs + J.cols;  // [TR][G+1]
    const int G = M.G, K = J.cols;
    for (int k = threadIdx.x; k < K; k += blockDim.x) xs[k] = J.x[k];
    __syncthreads();
    const int units = M.TR * G;
    for (int r0 = blockIdx.x * M.TR; r0 < J.rows; r0 += gridDim.x * M.TR) {
        const int nr = min(M.TR, J.rows - r0);
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
            const int rr = u / G, g = u % G;
            if (rr >= nr) continue;
            const uint8_t *row = J.w + (uint64_t)(r0 + rr) * M.rb;
            const float *xg = xs + g * 128;
            float s = 0.f;
            if (KIND == TRX_KIND_TERNARY5) {
                const uint8_t *cb = row + M.sbytes + 26 * g;
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
                const uint8_t *cb = row + M.sbytes + 32 * g;
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
            reinterpret_cast<float *>(J.y)[r0 + rr] = a;
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
static int round_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

bool plan_matvec(int rows, int cols, int kind, int nw, MvGeom &M) {
    M.G = cols / 128;
    if (M.G <= 32) {
        M.LS = round_pow2(M.G);
        M.RS = kThreads / M.LS;
    } else {
        M.LS = (M.G + 31) / 32 * 32;
        if (M.LS > 512) return false;
        M.RS = M.LS >= kThreads ? 1 : kThreads / M.LS;
    }
    M.sbytes = (M.G + 15) / 16 * 32;
    const int cb = kind == TRX_KIND_TERNARY5 ? 26 * M.G : 32 * M.G;
    M.rb = M.sbytes + (cb + 31) / 32 * 32;
    M.nw = nw;
    int per = kStageBudget / (M.rb * nw);
    if (per < 1) per = 1;
    int tr = per / M.RS * M.RS;
    if (tr < M.RS) tr = per < M.RS ? per : M.RS;
    if (tr > 64) tr = 64;
    if (tr > rows) tr = rows;
    M.TR = tr < 1 ? 1 : tr;
    M.tiles = (rows + M.TR - 1) / M.TR;
    M.xwords = kind == TRX_KIND_TERNARY5 ? kXWordsT5 : kXWords2b;
    int s = 0;
    if (kind == TRX_KIND_TERNARY5) s += kLutBytes;
    s += 2 * M.TR * M.rb * nw;
    s += M.G * M.xwords * 4;
    s += ((M.G * 4 + 15) / 16) * 16;
    s += (M.TR * nw * 8 + 15) / 16 * 16;
    s += 64 * 4;
    s += (int)sizeof(SmemHead);
    s += cols;
    M.smem = (s + 127) / 128 * 128;
    return M.smem <= 227 * 1024;
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

trx_status launch_matvec(const MvJobs &J, const uint32_t *lut, uint32_t *err, cudaStream_t st) {
    MvGeom M;
    if (!plan_matvec(J.rows, J.cols, J.kind, J.w2 ? 2 : 1, M)) return TRX_ERR_UNSUPPORTED;
    const int threads = M.LS * M.RS;
    int per_sm = (227 * 1024) / M.smem;
    if (per_sm > 2) per_sm = 2;
    if (per_sm < 1) per_sm = 1;
    const int total = J.njobs * M.tiles;
    int grid = num_sms() * per_sm;
    if (grid > total) grid = total;
    cudaError_t e;
    if (J.kind == TRX_KIND_TERNARY5) {
        e = cudaFuncSetAttribute(tmv_kernel<TRX_KIND_TERNARY5>, cudaFuncAttributeMaxDynamicSharedMemorySize, M.smem);
        if (e != cudaSuccess) return TRX_ERR_CUDA;
        tmv_kernel<TRX_KIND_TERNARY5><<<grid, threads, M.smem, st>>>(J, M, lut, err);
    } else {
        e = cudaFuncSetAttribute(tmv_kernel<TRX_KIND_TERNARY>, cudaFuncAttributeMaxDynamicSharedMemorySize, M.smem);
        if (e != cudaSuccess) return TRX_ERR_CUDA;
        tmv_kernel<TRX_KIND_TERNARY><<<grid, threads, M.smem, st>>>(J, M, lut, err);
    }
    return cudaGetLastError() == cudaSuccess ? TRX_OK : TRX_ERR_CUDA;
}

trx_status launch_matvec_fp(const MvJobs &J, uint32_t *err, cudaStream_t st) {
    MvGeom M;
    M.G = J.cols / 128;
    M.sbytes = (M.G + 15) / 16 * 32;
    const int cb = J.kind == TRX_KIND_TERNARY5 ? 26 * M.G : 32 * M.G;
    M.rb = M.sbytes + (cb + 31) / 32 * 32;
    M.TR = 16;
    const int smem = J.cols * 4 + M.TR * (M.G + 1) * 4;
    if (smem > 227 * 1024) return TRX_ERR_UNSUPPORTED;
    int grid = (J.rows + M.TR - 1) / M.TR;
    if (grid > num_sms() * 4) grid = num_sms() * 4;
    cudaError_t e;
    if (J.kind == TRX_KIND_TERNARY5) {
        e = cudaFuncSetAttribute(tmv_fp_kernel<TRX_KIND_TERNARY5>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return TRX_ERR_CUDA;
        tmv_fp_kernel<TRX_KIND_TERNARY5><<<grid, 256, smem, st>>>(J, M, err);
    } else {
        e = cudaFuncSetAttribute(tmv_fp_kernel<TRX_KIND_TERNARY>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return TRX_ERR_CUDA;
        tmv_fp_kernel<TRX_KIND_TERNARY><<<grid, 256, smem, st>>>(J, M, err);
    }
    return cudaGetLastError() == cudaSuccess ? TRX_OK : TRX_ERR_CUDA;
}

trx_status launch_quantize(const float *x, int n, int8_t *x8, int *e8, cudaStream_t st) {
    quantize_kernel<<<1, 1024, 0, st>>>(x, n, x8, e8);
    return cudaGetLastError() == cudaSuccess ? TRX_OK : TRX_ERR_CUDA;
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
    return cudaGetLastError() == cudaSuccess ? TRX_OK : TRX_ERR_CUDA;
}

trx_status launch_build_lut(uint32_t *lut, cudaStream_t st) {
    build_lut_kernel<<<kLutWords / 256, 256, 0, st>>>(lut);
    return cudaGetLastError() == cudaSuccess ? TRX_OK : TRX_ERR_CUDA;
}

size_t lut_bytes() { return kLutBytes; }

}  // namespace trx
