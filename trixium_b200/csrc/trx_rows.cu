// Batched ternary matvec on the B200's 5th-generation tensor cores (sm_100a tcgen05, kind::i8):
// nb independent int8 activation rows against one pass over a packed tensor, bit-exact with
// model/bitexact.py:121-125 (matvec_ternary_rows: every row is model/bitexact.py:101-119's
// matvec_ternary), and the float form (each row quantised with its own exponent, model/mirror.py
// :45-51 and :664-678).
//
// Per CTA: a tile of 128 output rows (the MMA's M) over a range of K chunks (4 groups of 128).
//  * Codes and scales arrive by TMA boxes {chunk bytes, 128 rows} into a two-slot ring.
//  * Each iteration handles a pair of groups: 256 threads, thread t decodes group (t >> 7) of the
//    pair for row t & 127 into that group's A tile: 128 rows x 128 int8 codes in {0, 1, 2}, K-major
//    with the 128-byte swizzle (a row's eight 16-byte pieces at piece ^ (row & 7)), written with
//    16-byte stores.  trit5: a per-lane replicated 256-entry LUT of 8-byte entries (digits d0..d3 |
//    d4), addressed with one PRMT per byte; 2-bit: the four bit planes of each code word.
//  * The codes' K order is permuted within each group (all five digits of a trit5 byte are not four
//    contiguous K slots); the activation is permuted the same way once per launch by the prep
//    kernel (x8p), whose tiles arrive by TMA with the same swizzle: B = x8p rows, K-major.
//  * One thread issues the pair's MMAs (M = 128, N = BN, K = 32; four per group) into the pair's
//    TMEM buffer (int32, one BN-column block per group; two buffers) and commits them to an
//    mbarrier; the MMAs of pair i overlap the epilogue of pair i - 1 and the decode of pair i + 1.
//  * Epilogue: warps w and w + 4 read TMEM lanes 32 (w % 4) .. (the tile's rows), w / 4 picks the
//    group; per (row, batch row) the exact group sum is the MMA's sum of codes * x8 minus sum(x8)
//    (codes are 0, 1, 2 for w + 1), and the scale contribution (gs * m11) shifted by e16 + B is
//    added in int64 (model/bitexact.py:111-115).
//  * K split over ks CTAs per row tile when the tiles alone would leave SMs idle: partial int64
//    sums added with 64-bit atomics (exact), the tile's last CTA applies >> R, the checks of
//    model/bitexact.py:116,118 and the output, and leaves the scratch at zero.
// Every wait (TMA, MMA completion) is bounded; on expiry TRX_DEV_TIMEOUT is recorded, the CTA
// stops issuing, waits (bounded) for what it issued, frees its TMEM and returns.
#include <atomic>
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {
namespace {

constexpr int kRowsM = 128;       // rows of a tile (the MMA's M)
constexpr int kRowsThreads = 256;
constexpr int kRowsCb5 = 112;     // trit5 codes box per row (the chunk's 104 bytes from the 16-byte boundary below)
constexpr int kRowsCb2 = 144;     // 2-bit codes box per row (the chunk's 128 bytes and the next 16)
constexpr int kRowsLut = 0x10000; // shared-window address of the LUT (64 KiB: 256 entries x 32 lanes x 8 bytes)

// Shared-memory plan (offsets from the dynamic base, which sits at window address `reserved`).
struct RowsPlan {
    int slot;        // one code-ring slot: codes box, then scales box
    int ring_off;    // 2 slots
    int bt_off[3];   // the activation tiles of a pair (2 groups x BN rows x 128 bytes), 3 buffers
    int misc_off;    // barriers, TMEM address, per-pair scales and activation sums
    int lut_off;     // window 0x10000
    int a_off;       // 2 buffers x 2 groups x 16 KiB, 1024-aligned
    int smem;
};

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major with the 128-byte swizzle: start address (>> 4), leading
// byte offset 1 (unused for this layout), stride byte offset 1024 >> 4 (8 rows x 128 bytes), the
// sm_100 descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor of kind::i8: D int32 (2), A unsigned 8-bit (0), B signed 8-bit (1), both
// K-major, N >> 3, M >> 4.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc_i8() {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kRowsM >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// TMEM loads, one lane per thread: 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 2-D TMA load (no multicast) at element coordinates (x, y).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// The 8-byte trit5 LUT entry of byte b: digits d0..d3 in the low word, d4 in byte 0 of the high
// word (model/bons.py:125-130).
__host__ __device__ __forceinline__ uint2 t5_entry8(uint32_t b) {
    return make_uint2((b % 3) | ((b / 3) % 3) << 8 | ((b / 9) % 3) << 16 | ((b / 27) % 3) << 24, (b / 81) % 3);
}

// The K slot order of a group's 128 codes as the decoders write them (the prep kernel permutes the
// activation to match): the lane (weight index within the group) held in slot s.
//  trit5: slots 4i..4i+3 = digits 0..3 of byte i (i < 25); slots 100..102 = digits 0..2 of byte 25
//         (lanes 125..127); slot 103 = digit 4 of byte 24 (lane 124); slots 104 + i = digit 4 of
//         byte i (i < 24).  (Byte 25's digits 3 and 4 are the group's padding lanes 128, 129.)
//  2-bit: slot 16w + 4p + i = bit pair p of byte 4w + i (lane 16w + 4i + p).
__host__ __device__ __forceinline__ int slot_lane(int kind, int s) {
    if (kind == TRX_KIND_TERNARY5) {
        if (s < 100) return 5 * (s >> 2) + (s & 3);
        if (s < 103) return 125 + (s - 100);
        if (s == 103) return 124;
        return 5 * (s - 104) + 4;
    }
    return 16 * (s >> 4) + 4 * (s & 3) + ((s >> 2) & 3);
}

// Per batch row: the quantised activation (fp32 rows: the power-of-two quantiser with its own
// exponent, model/mirror.py:45-51; int8 rows: as given), permuted per group to the decoders' K
// order (x8p [nb][K]), and each group's activation sum (xsum [nb][G]).  One CTA per batch row.
__global__ void __launch_bounds__(256) rows_prep_kernel(const float *x, const int8_t *x8, int K, int kind,
                                                        int8_t *x8p, int *xsum, int *e8_out) {
    extern __shared__ int8_t q[];  // K bytes
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, t = threadIdx.x;
    __shared__ uint32_t amax_s;
    if (x) {
        const float *xr = x + (size_t)b * K;
        if (t == 0) amax_s = 0;
        __syncthreads();
        uint32_t m = 0;
        for (int k = t; k < K; k += blockDim.x) {
            const uint32_t a = __float_as_uint(fabsf(xr[k]));
            m = a > m ? a : m;
        }
        m = __reduce_max_sync(0xffffffffu, m);
        if ((t & 31) == 0) atomicMax(&amax_s, m);
        __syncthreads();
        const uint32_t amax = amax_s;
        const int e8 = amax ? frexp_exp(__uint_as_float(amax)) - 7 : 0;
        const float inv = amax ? pow2f(-e8) : 0.f;
        for (int k = t; k < K; k += blockDim.x) {
            // The mirror's rounding: floor(|x| 2^-e8 + 0.5) in fp32, clamped to 127, signed.
            const float v = __fmul_rn(xr[k], inv);
            const float a = __fadd_rn(fabsf(v), 0.5f);
            const int mm = a < 128.0f ? (int)floorf(a) : 127;
            q[k] = (int8_t)(v < 0.f ? -mm : mm);
        }
        if (t == 0) e8_out[b] = e8;
    } else {
        for (int k = t; k < K; k += blockDim.x) q[k] = x8[(size_t)b * K + k];
        if (t == 0) e8_out[b] = 0;
    }
    __syncthreads();
    const int G = K / 128;
    for (int i = t; i < K; i += blockDim.x) {
        const int g = i >> 7, s = i & 127;
        x8p[(size_t)b * K + i] = q[g * 128 + slot_lane(kind, s)];
    }
    for (int g = t >> 5; g < G; g += blockDim.x >> 5) {
        const int lane = t & 31;
        int s = 0;
        for (int j = lane; j < 128; j += 32) s += q[g * 128 + j];
        s = __reduce_add_sync(0xffffffffu, s);
        if (lane == 0) xsum[(size_t)b * G + g] = s;
    }
}

}  // namespace

// One batched launch (host-built, by value).
struct RowsArgs {
    int N, K, G, nch, sbytes, rb, kind, nb;
    int B, R;
    int ks, cps;              // K splits per tile, chunks per split
    const int *xsum;          // [nb][G]
    const int *e8;            // [nb] (float outputs)
    int32_t *out_i;           // [nb][N] int32, or
    float *out_f;             // [nb][N] fp32
    const float *resid;       // [nb][N] added to the fp32 results, or nullptr
    unsigned long long *acc;  // [nb][N] int64 partial sums (ks > 1), zero between launches
    unsigned *cnt;            // [tiles] arrival counts (ks > 1), zero between launches
    RowsPlan P;
    int base;                 // window address of the dynamic shared memory the plan assumes
};

struct RowsMaps {
    CUtensorMap codes, scales, xp;
};

namespace {

// Decode one trit5 group (its 26 bytes from byte OFF of the row's 112-byte window) into 32 words
// of codes in the slot order above, and store them as the row's 128-byte A row (swizzled).
template <int OFF>
__device__ __forceinline__ void decode_t5(const unsigned char *win, uint32_t lane8x, unsigned char *arow, int r) {
    constexpr int p0 = OFF / 16, p1 = (OFF + 25) / 16;  // 16-byte pieces holding the group
    uint32_t w[12];
#pragma unroll
    for (int p = p0; p <= p1; ++p) {
        const uint4 v = reinterpret_cast<const uint4 *>(win)[p];
        w[4 * (p - p0)] = v.x;
        w[4 * (p - p0) + 1] = v.y;
        w[4 * (p - p0) + 2] = v.z;
        w[4 * (p - p0) + 3] = v.w;
    }
    uint32_t E[26], F[26];
#pragma unroll
    for (int i = 0; i < 26; ++i) {
        const int pb = OFF - 16 * p0 + i;  // byte of w (compile time)
        // 0x10000 + byte * 256 + lane * 8: this lane's replica of the 8-byte entry.
        const uint32_t a = __byte_perm(w[pb >> 2], lane8x, 0x7604u | ((pb & 3) << 4));
        asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(E[i]), "=r"(F[i]) : "r"(a));
    }
    uint32_t o[32];
#pragma unroll
    for (int i = 0; i < 25; ++i) o[i] = E[i];
    o[25] = __byte_perm(E[25], F[24], 0x4210u);  // digits 0..2 of byte 25, digit 4 of byte 24
#pragma unroll
    for (int j = 0; j < 6; ++j)
        o[26 + j] = __byte_perm(__byte_perm(F[4 * j], F[4 * j + 1], 0x0040u), __byte_perm(F[4 * j + 2], F[4 * j + 3], 0x0040u),
                                0x5410u);
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4 *>(arow + ((c ^ (r & 7)) << 4)) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}

// One 2-bit group (32 code bytes at cp): bit plane p of word w is slot block 16w + 4p.
__device__ __forceinline__ void decode_2b(const unsigned char *cp, unsigned char *arow, int r) {
    const uint4 c0 = reinterpret_cast<const uint4 *>(cp)[0], c1 = reinterpret_cast<const uint4 *>(cp)[1];
    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {  // 16-byte piece c = word c's four planes
        const uint32_t v = cw[c];
        const uint4 o = make_uint4(v & 0x03030303u, (v >> 2) & 0x03030303u, (v >> 4) & 0x03030303u,
                                   (v >> 6) & 0x03030303u);
        *reinterpret_cast<uint4 *>(arow + ((c ^ (r & 7)) << 4)) = o;
    }
}

template <int BN>
__device__ __forceinline__ void tmem_ld_bn(uint32_t taddr, int (&v)[BN]) {
    if constexpr (BN == 16) {
        tmem_ld16(taddr, v);
    } else {
        int a[16], b2[16];
        tmem_ld16(taddr, a);
        tmem_ld16(taddr + 16, b2);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            v[i] = a[i];
            v[16 + i] = b2[i];
        }
    }
}

template <int KIND, int BN>
__global__ void __launch_bounds__(kRowsThreads, 1)
    rows_kernel(const __grid_constant__ RowsMaps maps, RowsArgs A, uint32_t *err) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = tid & 127, h = tid >> 7;  // decode: row r, group h of the pair
    pdl_trigger();
    const int tile = blockIdx.x / A.ks, split = blockIdx.x - tile * A.ks;
    const int c0 = split * A.cps, c1 = min(A.nch, c0 + A.cps);
    const RowsPlan &P = A.P;
    if (smem_u32(smem) != (uint32_t)A.base) {  // the plan's window layout does not hold
        pdl_wait();
        if (tid == 0) atomicOr(err, TRX_DEV_INTERNAL);
        return;
    }
    unsigned char *const misc = smem + P.misc_off;
    const uint32_t bar_code = smem_u32(misc);          // [2] code-ring slots
    const uint32_t bar_bt = bar_code + 16;             // [3] activation tiles
    const uint32_t bar_mma = bar_code + 40;            // [2] MMA completion per TMEM/A buffer
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(misc + 64);
    uint32_t *const flag = tmem_slot + 1;              // a wait ran out somewhere in the CTA
    uint16_t *const scur = reinterpret_cast<uint16_t *>(misc + 128);  // [2 buf][2 grp][128 rows]
    int *const xcur = reinterpret_cast<int *>(misc + 128 + 2 * 2 * 128 * 2);  // [2 buf][2 grp][BN]
    const int G = A.G;
    const int np = 2 * (c1 - c0);  // pairs (the last ones may hold fewer groups)
    const uint32_t lane8x = (uint32_t)kRowsLut | ((uint32_t)lane << 3);

    if (KIND == TRX_KIND_TERNARY5) {  // the LUT: entry b at 0x10000 + b*256, one 8-byte replica per lane
        uint2 *lw = reinterpret_cast<uint2 *>(smem + P.lut_off);
        for (int i = tid; i < 256 * 32; i += kRowsThreads) lw[i] = t5_entry8((uint32_t)(i >> 5));
    }
    if (tid == 0) {
        for (int i = 0; i < 7; ++i) mbar_init_s(bar_code + 8u * i, 1);
        *flag = 0u;
        mbar_fence_init();
        tma_prefetch_map(&maps.codes);
        tma_prefetch_map(&maps.scales);
        tma_prefetch_map(&maps.xp);
    }
    if (warp == 0) {  // TMEM: 2 buffers x 2 groups x BN int32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(4 * BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t slot_bytes = (uint32_t)P.slot;
    const int cb = KIND == TRX_KIND_TERNARY5 ? kRowsCb5 : kRowsCb2;
    const int y0 = tile * kRowsM;

    // Issue (thread 0): chunk k's codes and scales into ring slot k % 2; pair p's activation tiles
    // into buffer p % 3.  Weights are written by no kernel, so both code slots go before the
    // dependency wait; the activation is the prep kernel's, after it.
    auto issue_chunk = [&](int k) {
        const int c = c0 + k;
        const uint32_t dst = smem_u32(smem + P.ring_off) + (uint32_t)(k & 1) * slot_bytes;
        const uint32_t bar = bar_code + 8u * (k & 1);
        mbar_expect_tx_s(bar, slot_bytes);
        const int xc = KIND == TRX_KIND_TERNARY5 ? A.sbytes + 104 * c - 8 * (c & 1) : A.sbytes + 128 * c;
        tma_load_3d(dst, &maps.codes, xc, y0, 0, bar);
        tma_load_3d(dst + (uint32_t)(cb * kRowsM), &maps.scales, 16 * (c >> 1), y0, 0, bar);
    };
    auto issue_bt = [&](int p) {
        const int g = 4 * c0 + 2 * p;  // first group of the pair
        const int ng = min(2, G - g);
        const uint32_t dst = smem_u32(smem + P.bt_off[p % 3]);
        const uint32_t bar = bar_bt + 8u * (p % 3);
        mbar_expect_tx_s(bar, (uint32_t)(ng * BN * 128));
        for (int j = 0; j < ng; ++j) tma_load_2d(dst + (uint32_t)(j * BN * 128), &maps.xp, 128 * (g + j), 0, bar);
    };
    // Arms per barrier (thread 0's count; the last armed phase of barrier j is (uses[j] - 1) & 1):
    // code slots 0, 1; activation tiles 2..4; MMA buffers 5, 6.
    int uses[7] = {0, 0, 0, 0, 0, 0, 0};
    if (tid == 0) {
        fence_proxy_async();
        for (int k = 0; k < min(2, c1 - c0); ++k) {
            issue_chunk(k);
            ++uses[k];
        }
    }
    pdl_wait();
    if (tid == 0 && np > 0) {
        issue_bt(0);
        ++uses[2];
    }

    // Per-row sums of this CTA's groups, per batch row (two threads per row: h = 0, 1).
    long long acc[BN];
#pragma unroll
    for (int b = 0; b < BN; ++b) acc[b] = 0;
    const ScaleFast F = scale_fast(A.B);
    const uint32_t idesc = umma_idesc_i8<BN>();

    // A warp-uniform bounded wait: lane 0 waits, the lanes learn the outcome, and each lane then
    // observes the completed phase itself (its own acquire of the data).
    auto warp_wait = [&](uint32_t bar, uint32_t parity) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded_s(bar, parity, err);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok) mbar_try_wait_s(bar, parity);
        return ok;
    };
    auto epilogue = [&](int i) {  // pair i: warps w and w + 4 read TMEM lanes 32 (w % 4) .., group w / 4
        const int eh = warp >> 2, er = 32 * (warp & 3) + lane;
        const int g = 4 * c0 + 2 * i + eh;
        if (g >= G) return;
        tc_fence_after();
        int v[BN];
        tmem_ld_bn<BN>(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)((i & 1) * 2 * BN + eh * BN), v);
        tmem_wait_ld();
        const uint32_t sb = scur[((i & 1) * 2 + eh) * 128 + er];
        const int *xs = xcur + ((i & 1) * 2 + eh) * BN;
#pragma unroll
        for (int b = 0; b < BN; ++b)
            if (b < A.nb) acc[b] += contrib(v[b] - xs[b], sb, A.B, F);
    };

    int done = -1;  // the last pair whose MMAs were committed
    for (int i = 0; i < np; ++i) {
        const int k = i >> 1;                  // chunk (local)
        const int c = c0 + k;
        const int g0 = 4 * c + 2 * (i & 1);    // the pair's first group
        if (g0 >= G) break;                    // (uniform)
        const int ng = min(2, G - g0);
        // MMA(i - 2) read A[i & 1] and the tiles of pair i - 2; the chunk's codes must be in.
        bool ok = i < 2 || warp_wait(bar_mma + 8u * (i & 1), ((i - 2) >> 1) & 1u);
        ok = ok && warp_wait(bar_code + 8u * (k & 1), (k >> 1) & 1u);
        if (!ok && lane == 0) atomicOr(flag, 1u);
        __syncthreads();
        if (*flag) break;                      // (uniform)
        // Decode: row r, group g0 + h of the pair, into A[i & 1][h].
        const unsigned char *slot = smem + P.ring_off + (size_t)(k & 1) * slot_bytes;
        unsigned char *arow = smem + P.a_off + (size_t)((i & 1) * 2 + h) * 16384 + (size_t)r * 128;
        const int q = 2 * (i & 1) + h;         // group within the chunk
        if (h < ng) {
            if (KIND == TRX_KIND_TERNARY5) {
                const unsigned char *win = slot + (size_t)r * kRowsCb5;
                switch (q + 4 * (c & 1)) {  // window offset 8 (c & 1) + 26 q
                    case 0: decode_t5<0>(win, lane8x, arow, r); break;
                    case 1: decode_t5<26>(win, lane8x, arow, r); break;
                    case 2: decode_t5<52>(win, lane8x, arow, r); break;
                    case 3: decode_t5<78>(win, lane8x, arow, r); break;
                    case 4: decode_t5<8>(win, lane8x, arow, r); break;
                    case 5: decode_t5<34>(win, lane8x, arow, r); break;
                    case 6: decode_t5<60>(win, lane8x, arow, r); break;
                    default: decode_t5<86>(win, lane8x, arow, r); break;
                }
            } else {
                decode_2b(slot + (size_t)r * kRowsCb2 + 32 * q, arow, r);
            }
            const uint16_t *sc = reinterpret_cast<const uint16_t *>(slot + cb * kRowsM + (size_t)r * 16 + 8 * (c & 1));
            scur[((i & 1) * 2 + h) * 128 + r] = sc[q];
        }
        if (tid < 2 * BN) {  // the pair's activation sums
            const int gh = tid / BN, b = tid - gh * BN;
            xcur[((i & 1) * 2 + gh) * BN + b] = (gh < ng && b < A.nb) ? A.xsum[(size_t)b * G + g0 + gh] : 0;
        }
        fence_proxy_async();  // the A rows (generic stores) before the tensor cores read them
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            // The chunk's slot is free once both its pairs are decoded: chunk k + 2 goes in.
            if ((i & 1) && k + 2 < c1 - c0) {
                issue_chunk(k + 2);
                ++uses[k & 1];
            }
            // Pair i + 1's activation tiles: its buffer's last reader, MMA(i - 2), is complete.
            if (i + 1 < np && 4 * c0 + 2 * (i + 1) < G) {
                issue_bt(i + 1);
                ++uses[2 + (i + 1) % 3];
            }
            if (mbar_wait_bounded_s(bar_bt + 8u * (i % 3), (uint32_t)(i / 3) & 1u, err)) {
                tc_fence_after();
                const uint32_t abase = smem_u32(smem + P.a_off) + (uint32_t)((i & 1) * 2) * 16384u;
                const uint32_t bbase = smem_u32(smem + P.bt_off[i % 3]);
                for (int j = 0; j < ng; ++j)
#pragma unroll
                    for (int s2 = 0; s2 < 4; ++s2)
                        umma_i8(tmem + (uint32_t)((i & 1) * 2 * BN + j * BN),
                                umma_desc_sw128(abase + (uint32_t)j * 16384u + 32u * s2),
                                umma_desc_sw128(bbase + (uint32_t)(j * BN * 128) + 32u * s2), idesc, s2);
                umma_commit(bar_mma + 8u * (i & 1));
                ++uses[5 + (i & 1)];
            } else {
                *flag = 1u;
            }
        }
        __syncthreads();
        if (*flag) break;                      // (uniform)
        done = i;
        if (i >= 1) {  // epilogue of pair i - 1 (its MMAs were committed an iteration ago)
            if (warp_wait(bar_mma + 8u * ((i - 1) & 1), ((i - 1) >> 1) & 1u))
                epilogue(i - 1);
            else if (lane == 0)
                atomicOr(flag, 1u);
            tc_fence_before();
        }
    }
    __syncthreads();
    if (!*flag && done >= 0) {  // the last pair's epilogue
        if (warp_wait(bar_mma + 8u * (done & 1), (done >> 1) & 1u))
            epilogue(done);
        else if (lane == 0)
            atomicOr(flag, 1u);
        tc_fence_before();
    }
    __syncthreads();
    const bool dead = *flag != 0u;
    if (dead && tid == 0) {  // wait (bounded) for every copy and MMA this CTA armed, then leave
        for (int j = 0; j < 7; ++j)
            if (uses[j]) mbar_wait_bounded_s(bar_code + 8u * j, (uint32_t)(uses[j] - 1) & 1u, nullptr);
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(4 * BN) : "memory");
    }
    if (dead) return;

    // Two threads per row: h = 1 hands its sums to h = 0 through shared memory (the A tiles are idle).
    long long *xch = reinterpret_cast<long long *>(smem + P.a_off);
    if (h == 1)
#pragma unroll
        for (int b = 0; b < BN; ++b) xch[b * 128 + r] = acc[b];
    __syncthreads();
    const int n = y0 + r;
    if (h == 0) {
#pragma unroll
        for (int b = 0; b < BN; ++b) acc[b] += xch[b * 128 + r];
    }
    auto finish = [&](int b, long long a) {
        if (acc_bad(a, A.R)) atomicOr(err, TRX_DEV_OVERFLOW);
        const int res = (int)(a >> A.R);
        if (A.out_f) {
            float v = __fmul_rn((float)res, pow2f(A.e8[b] + A.R - A.B));
            if (A.resid) v = __fadd_rn(A.resid[(size_t)b * A.N + n], v);
            A.out_f[(size_t)b * A.N + n] = v;
        } else
            A.out_i[(size_t)b * A.N + n] = res;
    };
    if (A.ks == 1) {
        if (h == 0 && n < A.N)
#pragma unroll
            for (int b = 0; b < BN; ++b)
                if (b < A.nb) finish(b, acc[b]);
        return;
    }
    // K split: exact int64 partial sums, then the tile's last CTA finishes and clears.
    if (h == 0 && n < A.N)
#pragma unroll
        for (int b = 0; b < BN; ++b)
            if (b < A.nb) atomicAdd(A.acc + (size_t)b * A.N + n, (unsigned long long)acc[b]);
    __threadfence();
    __syncthreads();
    if (tid == 0) *flag = atomicAdd(A.cnt + tile, 1u) == (unsigned)(A.ks - 1) ? 2u : 0u;
    __syncthreads();
    if (*flag != 2u) return;
    __threadfence();
    if (h == 0 && n < A.N)
        for (int b = 0; b < A.nb; ++b) {
            unsigned long long *p = A.acc + (size_t)b * A.N + n;
            finish(b, (long long)__ldcg(p));
            *p = 0ull;
        }
    if (tid == 0) A.cnt[tile] = 0u;
}

}  // namespace

// Host ---------------------------------------------------------------------------------------------
using EncodeTiledFn2 = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
    static std::atomic<EncodeTiledFn2> fn{nullptr};
    EncodeTiledFn2 f = fn.load(std::memory_order_acquire);
    if (!f) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f = reinterpret_cast<EncodeTiledFn2>(p);
        fn.store(f, std::memory_order_release);
    }
    return f;
}

static bool encode(CUtensorMap *m, const void *base, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
                   const cuuint32_t *box, CUtensorMapSwizzle sw) {
    const EncodeTiledFn2 f = encode_fn();
    if (!f) return false;
    const cuuint32_t es[3] = {1, 1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void *>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

static bool rows_plan(int kind, int BN, int reserved, RowsPlan &P) {
    const int cb = kind == TRX_KIND_TERNARY5 ? kRowsCb5 : kRowsCb2;
    P.slot = (cb + 16) * kRowsM;
    P.ring_off = 0;
    const int bt = 2 * BN * 128;
    P.bt_off[0] = (2 * P.slot + 1023) / 1024 * 1024;
    P.bt_off[1] = P.bt_off[0] + bt;
    P.misc_off = P.bt_off[1] + bt;
    const int misc = 128 + 2 * 2 * 128 * 2 + 2 * 2 * BN * 4;
    P.lut_off = kRowsLut - reserved;
    if (P.misc_off + misc > P.lut_off) return false;
    P.a_off = P.lut_off + 65536;                 // window 0x20000: 1024-aligned
    P.bt_off[2] = P.a_off + 4 * 16384;
    P.smem = P.bt_off[2] + bt;
    return (reserved % 1024) == 0 && P.smem <= 227 * 1024;
}

template <int KIND, int BN>
static trx_status launch_rows_t(const RowsMaps &maps, const RowsArgs &A, int grid, uint32_t *err, cudaStream_t st) {
    static DevBits configured{0};
    const cudaError_t e = once_per_device(configured, [] {
        return cudaFuncSetAttribute(rows_kernel<KIND, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    });
    if (e != cudaSuccess) return note_cuda(e);
    return note_cuda(launch_kernel(rows_kernel<KIND, BN>, dim3(grid), dim3(kRowsThreads), A.P.smem, st, maps, A, err));
}

trx_status launch_matvec_rows(const uint8_t *w, int N, int K, int kind, int B, int R, const float *x, const int8_t *x8,
                              int nb, int8_t *x8p, int *xsum, int *e8, unsigned long long *acc_scratch,
                              size_t acc_cap, unsigned *cnt, int cnt_cap, int32_t *out_i, float *out_f,
                              const float *resid, uint32_t *err, int sms, int reserved, cudaStream_t st) {
    const int BN = nb <= 16 ? 16 : 32;
    RowsArgs A{};
    A.N = N;
    A.K = K;
    A.G = K / 128;
    A.nch = (A.G + 3) / 4;
    A.sbytes = (A.G + 15) / 16 * 32;
    A.rb = A.sbytes + ((kind == TRX_KIND_TERNARY5 ? 26 : 32) * A.G + 31) / 32 * 32;
    A.kind = kind;
    A.nb = nb;
    A.B = B;
    A.R = R;
    const int tiles = (N + kRowsM - 1) / kRowsM;
    A.ks = tiles >= sms ? 1 : std::min(A.nch, std::max(1, sms / tiles));
    A.cps = (A.nch + A.ks - 1) / A.ks;
    A.ks = (A.nch + A.cps - 1) / A.cps;  // no empty splits
    if (A.ks > 1 && ((size_t)nb * N > acc_cap || tiles > cnt_cap)) {
        A.ks = 1;
        A.cps = A.nch;
    }
    A.xsum = xsum;
    A.e8 = e8;
    A.out_i = out_i;
    A.out_f = out_f;
    A.resid = resid;
    A.acc = acc_scratch;
    A.cnt = cnt;
    A.base = reserved;
    if (!rows_plan(kind, BN, reserved, A.P)) return TRX_ERR_UNSUPPORTED;
    RowsMaps maps;
    memset(&maps, 0, sizeof(maps));
    const cuuint64_t wd[3] = {(cuuint64_t)A.rb, (cuuint64_t)N, 1}, ws[2] = {(cuuint64_t)A.rb, (cuuint64_t)N * A.rb};
    const cuuint32_t cbox[3] = {(cuuint32_t)(kind == TRX_KIND_TERNARY5 ? kRowsCb5 : kRowsCb2), (cuuint32_t)kRowsM, 1};
    const cuuint32_t sbox[3] = {16, (cuuint32_t)kRowsM, 1};
    const cuuint64_t xd[2] = {(cuuint64_t)K, (cuuint64_t)nb}, xs[1] = {(cuuint64_t)K};
    const cuuint32_t xbox[2] = {128, (cuuint32_t)BN};
    if (!encode(&maps.codes, w, 3, wd, ws, cbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(&maps.scales, w, 3, wd, ws, sbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(&maps.xp, x8p, 2, xd, xs, xbox, CU_TENSOR_MAP_SWIZZLE_128B))
        return TRX_ERR_CUDA;
    // The permuted activation, its group sums and exponents (one CTA per batch row).
    cudaError_t e = launch_kernel(rows_prep_kernel, dim3(nb), dim3(256), (size_t)K, st, x, x8, K, kind, x8p, xsum, e8);
    if (e != cudaSuccess) return note_cuda(e);
    const int grid = tiles * A.ks;
    if (kind == TRX_KIND_TERNARY5)
        return BN == 16 ? launch_rows_t<TRX_KIND_TERNARY5, 16>(maps, A, grid, err, st)
                        : launch_rows_t<TRX_KIND_TERNARY5, 32>(maps, A, grid, err, st);
    return BN == 16 ? launch_rows_t<TRX_KIND_TERNARY, 16>(maps, A, grid, err, st)
                    : launch_rows_t<TRX_KIND_TERNARY, 32>(maps, A, grid, err, st);
}

}  // namespace trx
