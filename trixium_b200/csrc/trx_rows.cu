// Batched ternary matvec on the B200's 5th-generation tensor cores (sm_100a tcgen05, kind::i8):
// nb <= 32 independent int8 activation rows against one pass over a packed tensor, bit-exact with
// model/bitexact.py:121-125 (matvec_ternary_rows: every row is model/bitexact.py:101-119's
// matvec_ternary), and the float form (each row quantised with its own exponent, model/mirror.py
// :45-51 and :664-678).
//
// Work: a unit is (a tile of 128 output rows, a range of K chunks of 4 groups).  A persistent CTA
// takes a contiguous range of units; its three decoder warpgroups take its units in turn, so each
// warpgroup owns the 128 rows of its unit (one row per thread, the MMA's M = 128 TMEM lanes) and no
// sums are exchanged between them.  Warp roles:
//  * the last warp, one thread: the producer.  It streams each warpgroup's chunks, in one order all
//    roles follow, through that warpgroup's ring of D / 3 shared-memory slots (TMA boxes: the chunk's
//    codes and scales for the 128 rows, and the activation tiles of its groups, B = BN batch rows x
//    128 int8, 128-byte swizzled), and refills a slot once the MMAs that read it are complete.
//  * the decoder warpgroups.  Thread r decodes its row's group into the 128 int8 codes {0, 1, 2}
//    (trit5: a per-lane replicated 256-entry LUT of 8-byte entries, digits d0..d3 | d4, addressed by
//    one PRMT per byte; 2-bit: the four bit planes of each code word) and writes them straight into
//    its warpgroup's A buffer in tensor memory (tcgen05.st, its own lane): the unpacked codes never
//    touch shared memory.  Two A/D buffer pairs per warpgroup: the MMAs of a group run while the
//    next one is decoded.  One warp of the warpgroup per chunk (in turn) issues, from one elected
//    lane of the converged warp, the four MMAs of each of the chunk's groups (M = 128, N = BN,
//    K = 32, A from tensor memory) once all four warps' rows are in, and commits them; a tcgen05.mma
//    from a thread in a divergent branch issued at about 0.4x that rate (measured on B200).
//  * The same threads read each group's result back (tcgen05.ld, BN int32 per row), subtract the
//    group's activation sum (staged in shared memory; the codes are w + 1) and add the exact scale
//    contribution (gs * m11) shifted by e16 + B in int64 (model/bitexact.py:111-115).
//  * The codes' K order is permuted within each group (a trit5 byte's five digits are not four
//    contiguous K slots); the prep kernel permutes the activation the same way (x8p) and writes the
//    group sums.
//  * A unit covering part of K adds its int64 partial sums with 64-bit atomics (exact in any order);
//    each row's last unit (a per-row arrival count) applies >> R, the checks of
//    model/bitexact.py:116,118 and the output, and leaves the scratch at zero.
// Every wait (TMA, MMA completion, decoded buffer) is bounded; on expiry TRX_DEV_TIMEOUT is
// recorded, every role stops, the producer waits (bounded) for what it armed, the tensor memory is
// freed and the CTA returns.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {
namespace {

constexpr int kRowsM = 128;                       // rows of a tile (the MMA's M, the TMEM lanes)
constexpr int kRowsCb5 = 112;  // trit5 codes box per row (the chunk's 104 bytes from the 16-byte boundary below)
constexpr int kRowsCb2 = 144;  // 2-bit codes box per row (the chunk's 128 bytes and the next 16)
constexpr int kRowsLut = 0x10000;  // shared-window address of the LUT (64 KiB: 256 entries x 32 lanes x 8 bytes)
constexpr int kRowsMaxD = 8;       // ring slots at most
constexpr int kRowsTmemCols = 512; // per warpgroup A 2 x 32 and D 2 x BN columns

// Shared-memory plan (offsets from the dynamic base, which sits at window address `reserved`).
struct RowsPlan {
    int D;                    // ring slots
    int slot_off[kRowsMaxD];  // each slot: [activation tiles 4 x BN x 128][codes 128 x cb][scales 128 x 16]
    int codes_off, scales_off;  // within a slot
    int lut_off;              // trit5: window 0x10000
    int xs_off;               // the activation's group sums [G][BN] int32
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

// Instruction descriptor of kind::i8: D int32 (2), A unsigned 8-bit (0: the codes 0, 1, 2), B signed
// 8-bit (1), both K-major, N >> 3, M >> 4.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc_i8() {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kRowsM >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, A in tensor memory (lane = row, 4 int8 K elements per column),
// issued by one elected lane of a converged warp (all lanes execute it; warp-uniform operands):
// measured on B200 about 2.5x the issue rate of a thread in a divergent branch.
__device__ __forceinline__ void umma_i8_ta_elect(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                 int acc) {
    asm volatile(
        "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
        " @e tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// Commit this warp's MMAs issued so far to an mbarrier (one arrival once they are complete).
__device__ __forceinline__ void umma_commit_elect(uint32_t bar) {
    asm volatile(
        "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
        " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar)
        : "memory");
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

// TMEM store, one lane per thread: 32 consecutive 32-bit columns (a row's 128 int8 codes).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&o)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3]), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7]), "r"(o[8]), "r"(o[9]),
        "r"(o[10]), "r"(o[11]), "r"(o[12]), "r"(o[13]), "r"(o[14]), "r"(o[15]), "r"(o[16]), "r"(o[17]), "r"(o[18]),
        "r"(o[19]), "r"(o[20]), "r"(o[21]), "r"(o[22]), "r"(o[23]), "r"(o[24]), "r"(o[25]), "r"(o[26]), "r"(o[27]),
        "r"(o[28]), "r"(o[29]), "r"(o[30]), "r"(o[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2-D TMA load (no multicast) at element coordinates (x, y).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Non-blocking test of a phase (mbarrier.try_wait may suspend the thread for a while before it
// reports an incomplete phase; a thread polling several barriers must not be held on one).
__device__ __forceinline__ bool mbar_test_wait_s(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void mbar_arrive_s(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// Per batch row: the quantised activation (fp32 rows: optionally RMS-normalised first, y = (x * r) * w
// with the canonical 64-partial sum of squares, model/mirror.py:576-591,697-700; then the
// power-of-two quantiser with its own exponent, model/mirror.py:45-51; int8 rows: as given), permuted
// per group to the decoders' K order (x8p [nb][K]), and each group's activation sum (xsum [G][32],
// batch row minor).  One CTA of 256 threads per batch row; K floats (norm) + K bytes of shared memory.
__global__ void __launch_bounds__(256) rows_prep_kernel(const float *x, const int8_t *x8, const float *nw, float eps,
                                                        int K, int kind, int8_t *x8p, int *xsum, int *e8_out) {
    extern __shared__ __align__(16) unsigned char prep_smem[];
    int8_t *const q = reinterpret_cast<int8_t *>(prep_smem);  // K bytes
    float *const v = reinterpret_cast<float *>(prep_smem + (K + 15) / 16 * 16);  // K floats (norm only)
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, t = threadIdx.x;
    __shared__ uint32_t amax_s;
    __shared__ float part[64];
    if (x) {
        const float *xr = x + (size_t)b * K;
        if (t == 0) amax_s = 0;
        if (nw) {
            if (t < 64) {
                float p = 0.f;
                for (int i = t; i < K; i += 64) p = __fadd_rn(p, __fmul_rn(xr[i], xr[i]));
                part[t] = p;
            }
            __syncthreads();
            for (int h = 32; h >= 1; h >>= 1) {
                if (t < h) part[t] = __fadd_rn(part[t], part[t + h]);
                __syncthreads();
            }
            const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(part[0], (float)K), eps)));
            for (int i = t; i < K; i += blockDim.x) v[i] = __fmul_rn(__fmul_rn(xr[i], r), nw[i]);
            xr = v;
        }
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
            const float vv = __fmul_rn(xr[k], inv);
            const float a = __fadd_rn(fabsf(vv), 0.5f);
            const int mm = a < 128.0f ? (int)floorf(a) : 127;
            q[k] = (int8_t)(vv < 0.f ? -mm : mm);
        }
        if (t == 0) e8_out[b] = e8;
    } else {
        for (int k = t; k < K; k += blockDim.x) q[k] = x8[(size_t)b * K + k];
        if (t == 0) e8_out[b] = 0;
    }
    __syncthreads();
    for (int i = t; i < K; i += blockDim.x) {
        const int g = i >> 7, s = i & 127;
        x8p[(size_t)b * K + i] = q[g * 128 + slot_lane(kind, s)];
    }
    for (int g = t >> 5; g < K / 128; g += blockDim.x >> 5) {
        const int lane = t & 31;
        int s = 0;
        for (int j = lane; j < 128; j += 32) s += q[g * 128 + j];
        s = __reduce_add_sync(0xffffffffu, s);
        if (lane == 0) xsum[(size_t)g * 32 + b] = s;
    }
}

}  // namespace

// One batched launch (host-built, by value).
struct RowsArgs {
    int N, K, G, nch, sbytes, rb, kind, nb;
    int tiles, ks, cps;       // row tiles, K splits per tile, chunks per split (unit u: tile u / ks, split u % ks)
    const int *xsum;          // [G][32]
    const int *e8;            // [nb] (float outputs)
    int nseg;                 // segments (tensors packed back to back): rows [start, end) of the launch
    int seg_end[kRowsMaxSegs];
    RowsSeg seg[kRowsMaxSegs];  // B, R, output [nb][rows] (int32 or fp32), residual of each
    unsigned long long *acc;  // [nb][N] int64 partial sums (ks > 1), zero between launches
    unsigned *cnt;            // [tiles] arrival counts (ks > 1), zero between launches
    RowsPlan P;
    int base;                 // window address of the dynamic shared memory the plan assumes
};

struct RowsMaps {
    CUtensorMap codes, scales, xp;
};

namespace {

// Decode one trit5 group (its 26 bytes from byte OFF of the row's 112-byte window) into 32 words of
// codes in the slot order above.
template <int OFF>
__device__ __forceinline__ void decode_t5(const unsigned char *win, uint32_t lane8x, uint32_t (&o)[32]) {
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
    uint32_t F[26];
#pragma unroll
    for (int i = 0; i < 26; ++i) {
        const int pb = OFF - 16 * p0 + i;  // byte of w (compile time)
        // 0x10000 + byte * 256 + lane * 8: this lane's replica of the 8-byte entry.
        const uint32_t a = __byte_perm(w[pb >> 2], lane8x, 0x7604u | ((pb & 3) << 4));
        uint32_t e;
        asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(e), "=r"(F[i]) : "r"(a));
        if (i < 25)
            o[i] = e;
        else
            o[25] = __byte_perm(e, F[24], 0x4210u);  // digits 0..2 of byte 25, digit 4 of byte 24
    }
#pragma unroll
    for (int j = 0; j < 6; ++j)
        o[26 + j] = __byte_perm(__byte_perm(F[4 * j], F[4 * j + 1], 0x0040u), __byte_perm(F[4 * j + 2], F[4 * j + 3], 0x0040u),
                                0x5410u);
}

// One 2-bit group (32 code bytes at cp): bit plane p of word w is slot block 16w + 4p.
__device__ __forceinline__ void decode_2b(const unsigned char *cp, uint32_t (&o)[32]) {
    const uint4 c0 = reinterpret_cast<const uint4 *>(cp)[0], c1 = reinterpret_cast<const uint4 *>(cp)[1];
    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint32_t v = cw[c];
        o[4 * c] = v & 0x03030303u;
        o[4 * c + 1] = (v >> 2) & 0x03030303u;
        o[4 * c + 2] = (v >> 4) & 0x03030303u;
        o[4 * c + 3] = (v >> 6) & 0x03030303u;
    }
}

// The order every role follows: the CTA's units [u0, u1) in rounds of NWG (warpgroup w takes the
// w-th unit of a round), each round's chunks interleaved between its units.
struct RowsSeq {
    int u0, u1, ks, cps, nch, nwg;
    int p, i, w;
};

__device__ __forceinline__ int unit_chunks(int u, int ks, int cps, int nch, int &c0) {
    c0 = (u % ks) * cps;
    return max(0, min(nch, c0 + cps) - c0);
}

// The next item of the sequence: false at its end.  unit, chunk (global chunk index), the
// warpgroup, and whether it is the last chunk of its unit.
__device__ __forceinline__ bool seq_next(RowsSeq &S, int &unit, int &chunk, int &wg, bool &last) {
    for (;;) {
        const int ur = S.u0 + S.nwg * S.p;  // the round's first unit
        if (ur >= S.u1) return false;
        int mx = 0;
        for (int w = 0; w < S.nwg && ur + w < S.u1; ++w) {
            int c0;
            mx = max(mx, unit_chunks(ur + w, S.ks, S.cps, S.nch, c0));
        }
        if (S.i >= mx) {
            ++S.p;
            S.i = 0;
            S.w = 0;
            continue;
        }
        const int w = S.w, i = S.i;
        if (++S.w == S.nwg) {
            S.w = 0;
            ++S.i;
        }
        if (ur + w >= S.u1) continue;
        int c0;
        const int n = unit_chunks(ur + w, S.ks, S.cps, S.nch, c0);
        if (i >= n) continue;
        unit = ur + w;
        chunk = c0 + i;
        wg = w;
        last = i == n - 1;
        return true;
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

constexpr int kRowsMaxWg = 4;
// Decoder warpgroups: three, with the producer warp 13 warps, so that no SM sub-partition holds more
// than 4 warps of 128 registers (its 16 K registers; the tensor memory holds per warpgroup two A
// buffers of 32 columns and two D buffers of BN, after the shared 32 columns of minus ones).
template <int BN>
constexpr int rows_nwg() { return 3; }

// Barriers and flags at the start of the dynamic shared memory.
struct RowsBars {
    uint64_t full[kRowsMaxD];           // slot loaded (codes, scales, activation tiles)
    uint64_t freed[kRowsMaxD];          // the MMAs that read the slot are complete
    uint64_t afull[kRowsMaxWg][2];      // warpgroup w's A buffer s holds a decoded group (4 warp arrivals)
    uint64_t mdone[kRowsMaxWg][2];      // the MMAs of that group are complete
    uint64_t fin[4 * kRowsMaxWg];       // per decoder warp: every MMA it issued is complete (the exit)
    uint32_t slot[kRowsMaxD];           // window addresses of the ring slots
    uint32_t tmem;                      // tensor-memory base address
    volatile uint32_t dead;             // a wait ran out somewhere in the CTA
};

}  // namespace

namespace {

// Registers per thread: 4 warps of 128 fill a sub-partition's 16 K.
template <int KIND, int BN>
__global__ void __maxnreg__(128)
    rows_kernel(const __grid_constant__ RowsMaps maps, RowsArgs A, uint32_t *err) {
    extern __shared__ __align__(1024) unsigned char smem[];
    constexpr int NWG = rows_nwg<BN>();
    constexpr int NDW = 4 * NWG;  // decoder warps; warp NDW is the producer
    static_assert(NWG <= kRowsMaxWg, "barrier arrays hold every warpgroup");
    constexpr bool T5 = KIND == TRX_KIND_TERNARY5;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    const RowsPlan &P = A.P;
    if (smem_u32(smem) != (uint32_t)A.base) {  // the plan's window layout does not hold
        pdl_wait();
        if (tid == 0) atomicOr(err, TRX_DEV_INTERNAL);
        return;
    }
    RowsBars *const bars = reinterpret_cast<RowsBars *>(smem);
    const uint32_t bfull = smem_u32(bars->full), bfreed = smem_u32(bars->freed);
    const uint32_t bafull = smem_u32(&bars->afull[0][0]), bmdone = smem_u32(&bars->mdone[0][0]);
    int *const xs_s = reinterpret_cast<int *>(smem + P.xs_off);  // [G][BN] group sums of the activation
    const int units = A.tiles * A.ks;
    RowsSeq S0;
    S0.u0 = (int)((long long)blockIdx.x * units / gridDim.x);
    S0.u1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
    S0.ks = A.ks;
    S0.cps = A.cps;
    S0.nch = A.nch;
    S0.nwg = NWG;
    S0.p = S0.i = S0.w = 0;
    const int D = P.D, G = A.G;
    const int tid_prod = 32 * NDW;
    const int cb = T5 ? kRowsCb5 : kRowsCb2;
    const uint32_t codes_bytes = (uint32_t)(cb * kRowsM), tile_bytes = (uint32_t)(BN * 128);

    if (T5 && warp < 8) {  // the LUT: entry b at 0x10000 + b*256 + lane*8; warp w writes entries 32w..32w+31
        uint2 *lw = reinterpret_cast<uint2 *>(smem + P.lut_off);
        const uint2 mine = t5_entry8((uint32_t)(32 * warp + lane));
        for (int i = 0; i < 32; ++i)
            lw[(32 * warp + i) * 32 + lane] =
                make_uint2(__shfl_sync(0xffffffffu, mine.x, i), __shfl_sync(0xffffffffu, mine.y, i));
    }
    if (tid == tid_prod) {
        for (int d = 0; d < D; ++d) {
            mbar_init_s(bfull + 8u * d, 1);
            mbar_init_s(bfreed + 8u * d, 1);
            bars->slot[d] = smem_u32(smem + P.slot_off[d]);
        }
        for (int i = 0; i < 2 * NWG; ++i) {
            mbar_init_s(bafull + 8u * i, 4);
            mbar_init_s(bmdone + 8u * i, 1);
        }
        for (int i = 0; i < NDW; ++i) mbar_init_s(smem_u32(&bars->fin[i]), 1);
        bars->dead = 0u;
        mbar_fence_init();
        tma_prefetch_map(&maps.codes);
        tma_prefetch_map(&maps.scales);
        tma_prefetch_map(&maps.xp);
    }
    if (warp == NDW) {  // tensor memory: per warpgroup A 2 x 32 columns, D 2 x BN
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem)),
                     "r"(kRowsTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem;
    constexpr uint32_t kWgCols = 64 + 2 * BN;

    // Per-warpgroup rings: warpgroup w's i-th position (chunk of one of its units) lives in slot
    // w * Dw + i % Dw, so a slow warpgroup never holds up another's refills.
    const int Dw = D / NWG;
    // Producer: the codes and scales of each warpgroup's first Dw positions (written by no kernel)
    // before the dependency wait, their activation tiles after it.
    auto issue_w = [&](int slot, int unit, int chunk) {
        const uint32_t dst = bars->slot[slot], bar = bfull + 8u * slot;
        const int ng = min(4, G - 4 * chunk);
        mbar_expect_tx_s(bar, codes_bytes + 2048u + (uint32_t)ng * tile_bytes);
        const int y0 = (unit / A.ks) * kRowsM;
        const int xc = T5 ? A.sbytes + 104 * chunk - 8 * (chunk & 1) : A.sbytes + 128 * chunk;
        tma_load_2d(dst + (uint32_t)P.codes_off, &maps.codes, xc, y0, bar);
        tma_load_2d(dst + (uint32_t)P.scales_off, &maps.scales, 16 * (chunk >> 1), y0, bar);
    };
    auto issue_x = [&](int slot, int chunk) {
        const uint32_t dst = bars->slot[slot], bar = bfull + 8u * slot;
        const int ng = min(4, G - 4 * chunk);
        for (int q = 0; q < ng; ++q) tma_load_2d(dst + (uint32_t)q * tile_bytes, &maps.xp, 128 * (4 * chunk + q), 0, bar);
    };
    // The next position of warpgroup w in the sequence (its unit and chunk): false at its end.
    auto next_of = [&](RowsSeq &S, int w, int &unit, int &chunk) {
        int g;
        bool l;
        while (seq_next(S, unit, chunk, g, l))
            if (g == w) return true;
        return false;
    };
    RowsSeq Sp[NWG];
    int issued_w[NWG], pre_chunk[kRowsMaxD];
#pragma unroll
    for (int w = 0; w < NWG; ++w) {
        Sp[w] = S0;
        issued_w[w] = 0;
    }
    if (tid == tid_prod) {
        fence_proxy_async();
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
            int unit, chunk;
            while (issued_w[w] < Dw && next_of(Sp[w], w, unit, chunk)) {
                const int slot = w * Dw + issued_w[w]++;
                issue_w(slot, unit, chunk);
                pre_chunk[slot] = chunk;
            }
        }
    }
    pdl_wait();
    // The activation's group sums (the prep kernel's), staged once for every role.
    for (int i = tid; i < G * BN; i += blockDim.x) xs_s[i] = A.xsum[(i / BN) * 32 + (i % BN)];
    __syncthreads();

    if (tid == tid_prod) {
        // Producer: a warpgroup's positions retire in its order once the MMAs that read their slot
        // are complete; the freed slot takes the warpgroup's position i + Dw.
#pragma unroll
        for (int w = 0; w < NWG; ++w)
            for (int i = 0; i < issued_w[w]; ++i) issue_x(w * Dw + i, pre_chunk[w * Dw + i]);
        int retired_w[NWG];
#pragma unroll
        for (int w = 0; w < NWG; ++w) retired_w[w] = 0;
        unsigned long long t_last = global_ns();
        bool ok = true, more = true;
        while (more) {
            if (bars->dead) break;
            more = false;
            bool progress = false;
#pragma unroll
            for (int w = 0; w < NWG; ++w) {
                const int rw = retired_w[w];
                if (rw >= issued_w[w]) continue;
                more = true;
                const int slot = w * Dw + rw % Dw;
                if (!mbar_test_wait_s(bfreed + 8u * slot, (uint32_t)(rw / Dw) & 1u)) continue;
                int unit, chunk;
                if (next_of(Sp[w], w, unit, chunk)) {
                    fence_proxy_async();  // the decoders' reads of the slot (ordered by their arrivals) first
                    issue_w(slot, unit, chunk);
                    issue_x(slot, chunk);
                    ++issued_w[w];
                }
                retired_w[w] = rw + 1;
                progress = true;
            }
            if (progress) {
                t_last = global_ns();
            } else if (more && global_ns() - t_last > kWaitNs) {
                atomicOr(err, TRX_DEV_TIMEOUT);
                ok = false;
                break;
            }
        }
        if (!ok) bars->dead = 1u;
        // Every copy issued is complete before the CTA leaves (bounded; an expired wait was recorded).
#pragma unroll
        for (int w = 0; w < NWG; ++w)
            for (int d = 0; d < Dw && d < issued_w[w]; ++d) {
                const int plast = d + (issued_w[w] - 1 - d) / Dw * Dw;  // the last position issued into slot d
                mbar_wait_bounded_s(bfull + 8u * (w * Dw + d), (uint32_t)(plast / Dw) & 1u, nullptr);
            }
    } else if (warp < NDW) {
        // Decoders: warpgroup W, row r of its units' tiles (TMEM lane r).  The warp (position count
        // mod 4) of the warpgroup issues the MMAs of all groups of that position.
        const int W = warp >> 2, r = tid & 127;
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t lane8x = (uint32_t)kRowsLut | ((uint32_t)lane << 3);
        const uint32_t tA0 = tmem + (uint32_t)W * kWgCols, tD0 = tA0 + 64u;  // MMA operand addresses (lane 0)
        const uint32_t tA = tA0 + lane_base, tD = tD0 + lane_base;          // this warp's lanes
        const uint32_t idesc = umma_idesc_i8<BN>();
        // This thread's row of the current unit: its segment (tensor) gives B and the fast range.
        int Brow = A.seg[0].B;
        ScaleFast F = scale_fast(Brow);
        int cur_unit = -1;
        long long acc[BN];
#pragma unroll
        for (int b = 0; b < BN; ++b) acc[b] = 0;
        uint32_t sb0 = 0u, sb1 = 0u;  // the scale bits of the items in buffers 0 and 1
        int g0 = 0, g1 = 0;           // and their groups
        // Warp-uniform bounded wait: lane 0 waits, the lanes learn the outcome, and each lane then
        // observes the completed phase itself (its own acquire).
        auto warp_wait = [&](uint32_t bar, uint32_t parity) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait_bounded_s(bar, parity, err);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (ok) mbar_try_wait_s(bar, parity);
            return ok;
        };
        // Item e's group sums: D buffer e & 1 (sum(code * x8)) minus the group's sum(x8), read once
        // the item's MMAs are complete; its scale contribution in int64.
        auto epilogue = [&](int e) {
            const int s = e & 1;
            if (!warp_wait(bmdone + 8u * (2 * W + s), (uint32_t)(e >> 1) & 1u)) return false;
            tc_fence_after();
            int v[BN];
            tmem_ld_bn<BN>(tD + (uint32_t)(s * BN), v);
            tmem_wait_ld();
            const uint32_t sb = s ? sb1 : sb0;
            const int4 *xs4 = reinterpret_cast<const int4 *>(xs_s + (s ? g1 : g0) * BN);
#pragma unroll
            for (int i = 0; i < BN / 4; ++i) {
                const int4 t = xs4[i];
                v[4 * i] -= t.x;
                v[4 * i + 1] -= t.y;
                v[4 * i + 2] -= t.z;
                v[4 * i + 3] -= t.w;
            }
            const int E = (int)((sb >> 10) & 31u);
            if ((unsigned)(E - F.lo) <= (unsigned)F.span) {  // one 32 x 32 -> 64 multiply-add per batch row
                const int f = (int)(((sb & 0x3ffu) | 0x400u) << (E + F.sh));
                const long long fs = (sb & 0x8000u) ? -(long long)f : (long long)f;
#pragma unroll
                for (int b = 0; b < BN; ++b) acc[b] += (long long)v[b] * fs;
            } else {
#pragma unroll
                for (int b = 0; b < BN; ++b) acc[b] += group_contrib(v[b], sb, Brow);
            }
            return true;
        };
        auto finish = [&](int b, int n, long long a) {
            int sg = 0;
#pragma unroll
            for (int i = 0; i < kRowsMaxSegs - 1; ++i) sg += (i < A.nseg - 1 && n >= A.seg_end[i]) ? 1 : 0;
            const RowsSeg &S = A.seg[sg];
            const int sn = n - (sg ? A.seg_end[sg - 1] : 0);  // the row within its tensor
            if (acc_bad(a, S.R)) atomicOr(err, TRX_DEV_OVERFLOW);
            const size_t o = (size_t)b * S.rows + sn;
            // With earlier K-segments: their int32 sum plus this one's, wrapped to int32 (the mirror's
            // int64 sum of the segments' results).
            const int res = S.part_in ? (int)(uint32_t)(unsigned long long)((long long)S.part_in[o] + (a >> S.R))
                                      : (int)(a >> S.R);
            if (S.out_f) {
                float y = __fmul_rn((float)res, pow2f(A.e8[b] + S.R - S.B));
                if (S.resid) y = __fadd_rn(S.resid[o], y);
                S.out_f[o] = y;
            } else {
                S.out_i[o] = res;
            }
        };
        // A unit's rows are done: output them (whole K), or add the partial sums and let the row's
        // last unit (a per-row arrival count, so no barrier between the warps) finish it.
        auto flush = [&](int unit) {
            const int n = (unit / A.ks) * kRowsM + r;
            if (n < A.N) {
                if (A.ks == 1) {
#pragma unroll
                    for (int b = 0; b < BN; ++b)
                        if (b < A.nb) finish(b, n, acc[b]);
                } else {
#pragma unroll
                    for (int b = 0; b < BN; ++b)
                        if (b < A.nb) atomicAdd(A.acc + (size_t)b * A.N + n, (unsigned long long)acc[b]);
                    __threadfence();
                    if (atomicAdd(A.cnt + n, 1u) == (unsigned)(A.ks - 1)) {
                        __threadfence();
                        for (int b = 0; b < A.nb; ++b) {
                            unsigned long long *p = A.acc + (size_t)b * A.N + n;
                            finish(b, n, (long long)__ldcg(p));
                            *p = 0ull;
                        }
                        A.cnt[n] = 0u;
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < BN; ++b) acc[b] = 0;
        };
        RowsSeq Sd = S0;
        int unit, chunk, wg, j = 0, ep = 0, wpos = 0;
        bool last, alive = true, issued = false;
        while (alive && seq_next(Sd, unit, chunk, wg, last)) {
            if (wg != W) continue;
            if (bars->dead) {
                alive = false;
                break;
            }
            if (unit != cur_unit) {  // a new unit: this thread's row, its tensor's B
                cur_unit = unit;
                const int n = (unit / A.ks) * kRowsM + r;
                int sg = 0;
#pragma unroll
                for (int i = 0; i < kRowsMaxSegs - 1; ++i) sg += (i < A.nseg - 1 && n >= A.seg_end[i]) ? 1 : 0;
                Brow = A.seg[sg].B;
                F = scale_fast(Brow);
            }
            const int slot = W * Dw + wpos % Dw;
            if (!warp_wait(bfull + 8u * slot, (uint32_t)(wpos / Dw) & 1u)) {
                alive = false;
                break;
            }
            const bool issuer = (warp & 3) == (wpos & 3);
            ++wpos;
            const int ng = min(4, G - 4 * chunk);
            const uint32_t sbase = bars->slot[slot];
            const unsigned char *sp = smem + (sbase - (uint32_t)A.base);
            for (int q = 0; q < ng; ++q) {
                const int s = j & 1;
                uint32_t o[32];
                if (T5) {
                    const unsigned char *win = sp + P.codes_off + r * kRowsCb5;
                    switch (q + 4 * (chunk & 1)) {  // window offset 8 (chunk & 1) + 26 q
                        case 0: decode_t5<0>(win, lane8x, o); break;
                        case 1: decode_t5<26>(win, lane8x, o); break;
                        case 2: decode_t5<52>(win, lane8x, o); break;
                        case 3: decode_t5<78>(win, lane8x, o); break;
                        case 4: decode_t5<8>(win, lane8x, o); break;
                        case 5: decode_t5<34>(win, lane8x, o); break;
                        case 6: decode_t5<60>(win, lane8x, o); break;
                        default: decode_t5<86>(win, lane8x, o); break;
                    }
                } else {
                    decode_2b(sp + P.codes_off + r * kRowsCb2 + 32 * q, o);
                }
                const uint32_t sb = *reinterpret_cast<const uint16_t *>(sp + P.scales_off + r * 16 + 8 * (chunk & 1) + 2 * q);
                if (ep < j - 1) {  // item j - 2 (buffers s) read back before they are reused
                    if (!epilogue(ep)) {
                        alive = false;
                        break;
                    }
                    ++ep;
                }
                if (s) {
                    sb1 = sb;
                    g1 = 4 * chunk + q;
                } else {
                    sb0 = sb;
                    g0 = 4 * chunk + q;
                }
                tmem_st32(tA + (uint32_t)(s * 32), o);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_s(bafull + 8u * (2 * W + s));
                if (issuer) {  // every warp's A rows are in: the group's four MMAs, from one elected lane
                    if (!warp_wait(bafull + 8u * (2 * W + s), (uint32_t)(j >> 1) & 1u)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ta = tA0 + (uint32_t)(s * 32), td = tD0 + (uint32_t)(s * BN);
                    const uint32_t sbq = sbase + (uint32_t)q * tile_bytes;
#pragma unroll
                    for (int s2 = 0; s2 < 4; ++s2) umma_i8_ta_elect(td, ta + 8u * s2, umma_desc_sw128(sbq + 32u * s2), idesc, s2);
                    umma_commit_elect(bmdone + 8u * (2 * W + s));
                    if (q == ng - 1) umma_commit_elect(bfreed + 8u * slot);  // the position's slot: free once done
                    issued = true;
                }
                ++j;
            }
            if (!alive) break;
            if (last) {  // the unit's last chunk: read back its last groups, then output its rows
                while (ep < j) {
                    if (!epilogue(ep)) {
                        alive = false;
                        break;
                    }
                    ++ep;
                }
                if (!alive) break;
                flush(unit);
            }
        }
        if (!alive && lane == 0) bars->dead = 1u;
        if (issued) {  // this warp's MMAs are complete before the tensor memory is freed (bounded)
            umma_commit_elect(smem_u32(&bars->fin[warp]));
            if (lane == 0) mbar_wait_bounded_s(smem_u32(&bars->fin[warp]), 0u, nullptr);
            __syncwarp();
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == NDW) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kRowsTmemCols) : "memory");
    }
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

static bool encode(CUtensorMap *m, const void *base, const cuuint64_t *dims, const cuuint64_t *strides,
                   const cuuint32_t *box, CUtensorMapSwizzle sw) {
    const EncodeTiledFn2 f = encode_fn();
    if (!f) return false;
    const cuuint32_t es[2] = {1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// Slots of [activation tiles][codes][scales] (1024-byte multiples, 1024-aligned in the window) after
// the barriers; trit5: around the LUT at window 0x10000.
static bool rows_plan(int kind, int BN, int G, int reserved, RowsPlan &P) {
    if (reserved % 1024) return false;
    const bool t5 = kind == TRX_KIND_TERNARY5;
    const int cb = t5 ? kRowsCb5 : kRowsCb2;
    const int bt = 4 * BN * 128;
    P.codes_off = bt;
    P.scales_off = bt + cb * kRowsM;
    const int slot = (P.scales_off + 16 * kRowsM + 1023) / 1024 * 1024;
    const int top = 227 * 1024;
    static_assert(sizeof(RowsBars) <= 1024, "barriers fit the first KiB");
    P.xs_off = 1024;
    const int first = 1024 + (G * BN * 4 + 1023) / 1024 * 1024;  // after the group sums
    P.D = 0;
    auto region = [&](int lo, int hi) {
        for (int o = lo; o + slot <= hi && P.D < kRowsMaxD; o += slot) P.slot_off[P.D++] = o;
    };
    if (t5) {
        P.lut_off = kRowsLut - reserved;
        if (first > P.lut_off) return false;
        region(first, P.lut_off);
        region(P.lut_off + 65536, top);
    } else {
        P.lut_off = 0;
        region(first, top);
    }
    if (P.D < 2) return false;
    P.smem = std::max(P.slot_off[P.D - 1] + slot, t5 ? P.lut_off + 65536 : 0);
    return P.smem <= top;
}

template <int KIND, int BN>
static trx_status launch_rows_t(const RowsMaps &maps, const RowsArgs &A, int grid, uint32_t *err, cudaStream_t st) {
    static DevBits configured{0};
    const cudaError_t e = once_per_device(configured, [] {
        return cudaFuncSetAttribute(rows_kernel<KIND, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    });
    if (e != cudaSuccess) return note_cuda(e);
    return note_cuda(launch_kernel(rows_kernel<KIND, BN>, dim3(grid), dim3(32 * (4 * rows_nwg<BN>() + 1)), A.P.smem, st,
                                   maps, A, err));
}

trx_status launch_matvec_rows(const uint8_t *w, int K, int kind, const RowsSeg *segs, int nseg, const float *x,
                              const int8_t *x8, int nb, const float *norm_w, float eps, int8_t *x8p, int *xsum,
                              int *e8, unsigned long long *acc_scratch, size_t acc_cap, unsigned *cnt, int cnt_cap,
                              uint32_t *err, int sms, int reserved, cudaStream_t st, int K_full, int k_off,
                              bool prep) {
    if (nseg < 1 || nseg > kRowsMaxSegs) return TRX_ERR_ARG;
    if (!K_full) K_full = K;
    if (k_off < 0 || k_off % 128 || k_off + K > K_full || (!prep && !x8p)) return TRX_ERR_ARG;
    int N = 0;
    const int BN = nb <= 16 ? 16 : 32;
    RowsArgs A{};
    A.nseg = nseg;
    for (int i = 0; i < nseg; ++i) {
        A.seg[i] = segs[i];
        N += segs[i].rows;
        A.seg_end[i] = N;
    }
    A.N = N;
    A.K = K;
    A.G = K / 128;
    A.nch = (A.G + 3) / 4;
    A.sbytes = (A.G + 15) / 16 * 32;
    A.rb = A.sbytes + ((kind == TRX_KIND_TERNARY5 ? 26 : 32) * A.G + 31) / 32 * 32;
    A.kind = kind;
    A.nb = nb;
    // Units: (128-row tile, K range).  Split K when the tiles alone give fewer units than the SMs'
    // decoder warpgroups, within the scratch the partial sums and per-row counts need.
    const int nwg = BN == 16 ? rows_nwg<16>() : rows_nwg<32>();
    A.tiles = (N + kRowsM - 1) / kRowsM;
    A.ks = A.tiles >= nwg * sms ? 1 : std::min(A.nch, (nwg * sms + A.tiles - 1) / A.tiles);
    A.cps = (A.nch + A.ks - 1) / A.ks;
    A.ks = (A.nch + A.cps - 1) / A.cps;  // no empty splits
    if (A.ks > 1 && ((size_t)nb * N > acc_cap || N > cnt_cap)) {
        A.ks = 1;
        A.cps = A.nch;
    }
    A.xsum = xsum + (size_t)(k_off / 128) * 32;  // this segment's groups
    A.e8 = e8;
    A.acc = acc_scratch;
    A.cnt = cnt;
    A.base = reserved;
    if (!rows_plan(kind, BN, A.G, reserved, A.P) || A.P.D < nwg) return TRX_ERR_UNSUPPORTED;
    RowsMaps maps;
    memset(&maps, 0, sizeof(maps));
    const cuuint64_t wd[2] = {(cuuint64_t)A.rb, (cuuint64_t)N}, ws[1] = {(cuuint64_t)A.rb};
    const cuuint32_t cbox[2] = {(cuuint32_t)(kind == TRX_KIND_TERNARY5 ? kRowsCb5 : kRowsCb2), (cuuint32_t)kRowsM};
    const cuuint32_t sbox[2] = {16, (cuuint32_t)kRowsM};
    const cuuint64_t xd[2] = {(cuuint64_t)K, (cuuint64_t)nb}, xs[1] = {(cuuint64_t)K_full};
    const cuuint32_t xbox[2] = {128, (cuuint32_t)BN};
    if (!encode(&maps.codes, w, wd, ws, cbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(&maps.scales, w, wd, ws, sbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(&maps.xp, x8p + k_off, xd, xs, xbox, CU_TENSOR_MAP_SWIZZLE_128B))
        return TRX_ERR_CUDA;
    // The permuted activation, its group sums and exponents (one CTA per batch row).
    const size_t prep_smem = (size_t)(K_full + 15) / 16 * 16 + (norm_w ? (size_t)K_full * 4 : 0);
    constexpr int kPrepSmemMax = 192 * 1024;  // K <= 32768: 32 KiB of q8 and 128 KiB of normalised x
    if (prep_smem > (size_t)kPrepSmemMax) return TRX_ERR_UNSUPPORTED;
    static DevBits prep_configured{0};
    cudaError_t e = once_per_device(prep_configured, [] {
        return cudaFuncSetAttribute(rows_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmemMax);
    });
    if (e != cudaSuccess) return note_cuda(e);
    if (prep) {
        e = launch_kernel(rows_prep_kernel, dim3(nb), dim3(256), prep_smem, st, x, x8, norm_w, eps, K_full, kind, x8p,
                          xsum, e8);
        if (e != cudaSuccess) return note_cuda(e);
    }
    const int units = A.tiles * A.ks;
    const int grid = std::max(1, std::min(sms, (units + nwg - 1) / nwg));
    if (kind == TRX_KIND_TERNARY5)
        return BN == 16 ? launch_rows_t<TRX_KIND_TERNARY5, 16>(maps, A, grid, err, st)
                        : launch_rows_t<TRX_KIND_TERNARY5, 32>(maps, A, grid, err, st);
    return BN == 16 ? launch_rows_t<TRX_KIND_TERNARY, 16>(maps, A, grid, err, st)
                    : launch_rows_t<TRX_KIND_TERNARY, 32>(maps, A, grid, err, st);
}

}  // namespace trx
