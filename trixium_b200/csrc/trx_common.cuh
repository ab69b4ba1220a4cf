// Device helpers shared by the B200 ternary decode kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/trixium_b200.h"

namespace trx {

// Launch shape -----------------------------------------------------------------------------------
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Bounded waits: an mbarrier wait gives up after kWaitNs nanoseconds of %globaltimer, records
// TRX_DEV_TIMEOUT in the error word and returns (the caller then leaves the kernel).
constexpr unsigned long long kWaitNs = 200ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Shared-memory addresses and the TMA bulk-copy / mbarrier wrappers -------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D TMA bulk copy global -> shared, completing `bytes` of transaction on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16 (checked by the callers' geometry).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Shared-window address forms of the above (barrier given by its shared address).
__device__ __forceinline__ void mbar_init_s(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx_s(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 3-D tiled TMA load (no multicast): the box of `map` at element coordinates (x, y, z) into shared
// address dst, completing its bytes on barrier `bar`.  x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void *map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const void *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_s(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait by shared address: false (timeout bit set by lane 0 of the caller) if the phase did
// not complete within kWaitNs.
__device__ __forceinline__ bool mbar_wait_bounded_s(uint32_t bar, uint32_t parity, uint32_t *err) {
    if (mbar_try_wait_s(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait_s(bar, parity)) {
        if (global_ns() - t0 > kWaitNs) {
            if (err && (threadIdx.x & 31) == 0) atomicOr(err, TRX_DEV_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar`, bounded: returns false (and sets the timeout bit) if the
// phase did not complete within kWaitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kWaitNs) {
            if (err) atomicOr(err, TRX_DEV_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Tensor-parallel waits and signals (TpXfer, trx_internal.h) ---------------------------------------
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread: wait until *wait >= (*step + 1) * world (peers' completions of the gather point),
// bounded by kWaitNs (then TRX_DEV_TIMEOUT is recorded and the caller goes on).  The fence orders
// the peers' stores before later bulk (async-proxy) reads of the same bytes.
template <typename T>
__device__ __forceinline__ void tp_wait(const T &X, uint32_t *err) {
    if (!X.wait) return;
    const unsigned target = (unsigned)(*X.step + 1) * (unsigned)X.world;
    if ((int)(ld_acquire_sys(X.wait) - target) < 0) {
        const unsigned long long t0 = global_ns();
        while ((int)(ld_acquire_sys(X.wait) - target) < 0) {
            if (global_ns() - t0 > kWaitNs) {
                atomicOr(err, TRX_DEV_TIMEOUT);
                break;
            }
        }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Every thread of an arriving CTA (after its stores): the last of `arrivals` CTAs adds 1 to every
// rank's counter.  One system-scope fence per CTA, by the thread that arrives, after the block
// barrier that orders the other threads' stores before it.
template <typename T>
__device__ __forceinline__ void tp_signal(const T &X, unsigned arrivals) {
    if (!X.signal[0]) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(X.arrive, 1u) == arrivals - 1) {
            *X.arrive = 0u;
            __threadfence_system();
            for (int r = 0; r < X.world; ++r) atomicAdd_system(X.signal[r], 1u);
        }
    }
}

// Tagged words (TpXfer::tag_points > 0): value bits | tag << 32 in one 64-bit store.
template <typename T>
__device__ __forceinline__ unsigned tp_tag(const T &X, int point) {
    return (unsigned)(*X.step) * X.tag_points + (unsigned)point + 1u;
}

__device__ __forceinline__ void st_tagged(void *base, size_t i, float v, unsigned tag) {
    const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(reinterpret_cast<unsigned long long *>(base) + i), "l"(w)
                 : "memory");
}

__device__ __forceinline__ ulonglong2 ld_tagged2(const ulonglong2 *p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}

// Result i of a producing launch into the exchange: tagged words into every rank's copy, or plain
// floats into the other ranks' copies (the counter protocol; this rank's own copy is the launch's
// output).
template <typename T>
__device__ __forceinline__ void tp_push_all(const T &X, size_t i, float v) {
    if (X.tag_out >= 0 && X.tag_points) {
        const unsigned tag = tp_tag(X, X.tag_out);
        for (int r = 0; r < X.world; ++r) st_tagged(X.dst[r], X.offset + i, v, tag);
    } else {
        for (int r = 0; r < X.world; ++r)
            if (r != X.rank && X.dst[r]) reinterpret_cast<float *>(X.dst[r])[X.offset + i] = v;
    }
}

// Integer dot products ---------------------------------------------------------------------------
// acc + sum_k a.byte[k] * b.byte[k], a's bytes unsigned, b's signed (PTX dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int acc) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(acc));
    return d;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int acc) {
    return __dp4a(static_cast<int>(a), static_cast<int>(b), acc);
}

// acc + a.h0*b.b0 + a.h1*b.b1 (lo) / b.b2, b.b3 (hi): 16-bit signed pairs times signed bytes.
__device__ __forceinline__ int dp2a_lo(uint32_t a16, uint32_t b8, int acc) {
    return __dp2a_lo(static_cast<int>(a16), static_cast<int>(b8), acc);
}
__device__ __forceinline__ int dp2a_hi(uint32_t a16, uint32_t b8, int acc) {
    return __dp2a_hi(static_cast<int>(a16), static_cast<int>(b8), acc);
}

// fp16 scale -> (m11, e16), value = m11 * 2^e16 exactly (model/bitexact.py:56-68).
__device__ __forceinline__ void fp16_split(uint32_t bits, int &m11, int &e16) {
    const int E = (bits >> 10) & 31;
    const int mag = E ? (int)((bits & 1023u) | 1024u) : (int)(bits & 1023u);
    m11 = (bits & 0x8000u) ? -mag : mag;
    e16 = E ? E - 25 : -24;
}

// One group's contribution (gs*m11) shifted by e16+B: left if >= 0, arithmetic (floor) right
// otherwise (model/bitexact.py:111-115).  Shifts are clamped to [0, 63]; any left shift that
// large overflows the int48 accumulator check anyway.
__device__ __forceinline__ long long group_contrib(int gs, uint32_t scale_bits, int B) {
    int m11, e16;
    fp16_split(scale_bits, m11, e16);
    const long long prod = (long long)gs * (long long)m11;
    const int sh = e16 + B;
    if (sh >= 0) return prod << (sh > 63 ? 63 : sh);
    const int rs = -sh;
    return prod >> (rs > 63 ? 63 : rs);
}

// The trit5 byte LUT entry: digits d_k = (b / 3^k) % 3 (the reference reader's decode,
// model/bons.py:125-130), packed as bytes (d0, d1, d2, d3 + 3*d4).  The last byte is the
// byte's value / 27 for every valid byte; d4 = that / 3 is recovered in registers.
__host__ __device__ __forceinline__ uint32_t trit5_lut_entry(uint32_t b) {
    const uint32_t d0 = b % 3, d1 = (b / 3) % 3, d2 = (b / 9) % 3, d3 = (b / 27) % 3, d4 = (b / 81) % 3;
    return d0 | (d1 << 8) | (d2 << 16) | ((d3 + 3 * d4) << 24);
}

// frexp exponent of a positive finite float (the e in x = m * 2^e, m in [0.5, 1)).
__device__ __forceinline__ int frexp_exp(float a) {
    int e;
    frexpf(a, &e);
    return e;
}

// Programmatic dependent launch (sm_90+): every kernel of the library releases its successor as
// soon as it starts (the successor's CTAs take SMs as this kernel's CTAs leave) and waits for its
// predecessor's completion before it reads anything a kernel may have written.  Both are no-ops
// for a launch without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// (gs*m11) shifted by e16+B as int64 (model/bitexact.py:111-115).  Fast range: a normal fp16
// scale (biased exponent E in [1, 30]) with 0 <= e16+B = E-25+B <= 19, where m11 << (e16+B) is
// below 2^30: the contribution is (+-gs) * (m11 << (E-25+B)), one 32x32->64 multiply.  Other
// scales (tiny or subnormal ones, far below the tensor's largest) take the general floor/left
// shift.
struct ScaleFast {
    int lo, span;  // fast iff E - lo in [0, span]
    int sh;        // B - 25: the left shift is E + sh
};

__device__ __forceinline__ ScaleFast scale_fast(int B) {
    ScaleFast f;
    const int lo = max(1, 25 - B), hi = min(30, 44 - B);
    f.lo = hi >= lo ? lo : 64;  // an empty range: E - 64 < 0 fails the unsigned test below
    f.span = hi >= lo ? hi - lo : 0;
    f.sh = B - 25;
    return f;
}

__device__ __forceinline__ long long contrib(int gs, uint32_t sb, int B, const ScaleFast &F) {
    const int E = (int)((sb >> 10) & 31u);
    if ((unsigned)(E - F.lo) <= (unsigned)F.span)
        return (long long)(sb & 0x8000u ? -gs : gs) * (long long)(int)(((sb & 0x3ffu) | 0x400u) << (E + F.sh));
    return group_contrib(gs, sb, B);
}

// The checks of model/bitexact.py:116,118 (and :141,:143): the int48 accumulator and the int32
// result after >> R.
__device__ __forceinline__ bool acc_bad(long long a, int R) {
    const long long r = a >> R;
    return a >= (1ll << 47) || a <= -(1ll << 47) || r >= (1ll << 31) || r <= -(1ll << 31);
}

// 2^k as an fp32, exact for k in [-149, 127] (the scale of the power-of-two quantiser).
__device__ __forceinline__ float pow2f(int k) {
    if (k >= -126) return __int_as_float((min(k, 128) + 127) << 23);  // k = 128 gives inf
    return k >= -149 ? __int_as_float(1 << (k + 149)) : 0.f;           // subnormal powers
}

}  // namespace trx
