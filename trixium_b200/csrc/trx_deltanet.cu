// Gated-DeltaNet decode step for B200 (sm_100a): model/mirror.py:892-943 (mathematical profile),
// model/golden.py:400-434, after the layer's projections (qkv, z, beta, alpha: one segmented
// matvec launch).
//
// CTA (s, h) owns rows [s*rows, (s+1)*rows) of value head h's state (hv x hk fp32; rows are
// independent given the head's q, k, decay and beta):
//  * causal conv (K taps, the previous K-1 inputs in a K-slot ring indexed by the step's position,
//    so this step's writes never touch a slot another CTA reads) + SiLU for the q and k channels
//    of key head h % nk (recomputed per CTA: 2*hk channels) and the CTA's value channels;
//    L2-normalised q, k (canonical sum of squares; x * 1/max(|x|, eps), mirror.py:702-705);
//  * decay = exp(softplus(alpha + dt_bias) * a), beta = sigmoid(beta_raw);
//  * per row j, one warp: M_j *= decay; delta_j = (v_j - M_j.k) * beta; M_j += delta_j k;
//    o_j = M_j.q / sqrt(hk); M_j written back.  The state is streamed once: 2*4*hk bytes per row;
//  * the last CTA of the head to arrive (atomic count, reset by it) applies RMSNorm over o
//    (canonical) times silu(z) and writes the head at its grouped position (h % nk)*(nv/nk) + h/nk.
// The ring slot each channel writes is written by exactly one CTA.
#include <cstdint>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

constexpr int kDnThreads = 256;
constexpr int kDnWarps = kDnThreads / 32;
constexpr int kDnMaxPerLane = 8;  // hk <= 256

// Canonical sum of squares of v[0..n) (64 sequential partials, halving tree) by one warp; the
// result in every lane.
__device__ float warp_sumsq64(const float *v, int n, int lane) {
    float p0 = 0.f, p1 = 0.f;
    for (int i = lane; i < n; i += 64) p0 = __fadd_rn(p0, __fmul_rn(v[i], v[i]));
    for (int i = lane + 32; i < n; i += 64) p1 = __fadd_rn(p1, __fmul_rn(v[i], v[i]));
    float a = __fadd_rn(p0, p1);
    for (int o = 16; o; o >>= 1) a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, o));
    return __shfl_sync(0xffffffffu, a, 0);
}

__device__ __forceinline__ float silu_dn(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// Causal conv of channel c (taps w[c*K ..]; ring slots of the previous K-1 inputs, oldest first)
// then SiLU; sequential fp32 sum in tap order.
__device__ __forceinline__ float conv_silu(const DnArgs &A, int c, int pos) {
    const float *w = A.conv_w + (size_t)c * A.K;
    float acc = 0.f;
    for (int i = 0; i < A.K - 1; ++i) {
        const int slot = (pos + 1 + i) % A.K;  // = (pos - (K-1) + i) mod K
        acc = __fadd_rn(acc, __fmul_rn(__ldg(w + i), A.win[(size_t)slot * A.C + c]));
    }
    acc = __fadd_rn(acc, __fmul_rn(__ldg(w + A.K - 1), __ldg(A.qkv + c)));
    return silu_dn(acc);
}

__global__ void __launch_bounds__(kDnThreads) deltanet_kernel(DnArgs A, uint32_t *err) {
    extern __shared__ __align__(16) float dsm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x, h = blockIdx.y;
    if (blockIdx.z) {  // sequence z of a batch
        const long long z = blockIdx.z, vh = (long long)A.nv * A.hv;
        A.qkv += z * A.C;
        A.z += z * vh;
        A.beta += z * A.nv;
        A.alpha += z * A.nv;
        A.pos += z;
        A.win += z * (long long)A.K * A.C;
        A.S += z * vh * A.hk;
        A.out += z * vh;
        A.part += z * vh;
        A.cnt += z * A.nv;
    }
    const int hk = A.hk, hv = A.hv, nk = A.nk, nq = A.nk * A.hk;
    pdl_trigger();
    pdl_wait();
    const int pos = *A.pos;
    if (pos < 0) {
        if (tid == 0 && s == 0 && h == 0) atomicOr(err, TRX_DEV_RANGE);
        return;
    }
    float *qv = dsm;            // [hk]
    float *kv = qv + hk;        // [hk]
    float *vv = kv + hk;        // [rows]
    __shared__ float sh_decay, sh_beta;
    __shared__ int last_s;
    const int kh = h % nk;
    const int j0 = s * A.rows, j1 = min(hv, j0 + A.rows);
    const int wslot = pos % A.K;
    const bool owner_qk = s == 0 && h == kh;  // writes the ring slot of key head kh's channels

    // Conv + SiLU: q, k of key head kh; this CTA's value channels.
    for (int i = tid; i < 2 * hk; i += kDnThreads) {
        const int c = i < hk ? kh * hk + i : nq + kh * hk + (i - hk);
        const float y = conv_silu(A, c, pos);
        (i < hk ? qv : kv)[i < hk ? i : i - hk] = y;
    }
    for (int j = j0 + tid; j < j1; j += kDnThreads) vv[j - j0] = conv_silu(A, 2 * nq + h * hv + j, pos);
    if (tid == 0) {
        const float x = __fadd_rn(__ldg(A.alpha + h), __ldg(A.dt_bias + h));
        const float sp = x > 20.f ? x : log1pf(expf(x));
        sh_decay = expf(__fmul_rn(sp, __ldg(A.ssm_a + h)));
        sh_beta = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-__ldg(A.beta + h))));
    }
    __syncthreads();
    // This step's ring slot (after every conv above has read the older slots of this CTA; other
    // CTAs read only the older slots).
    if (owner_qk)
        for (int i = tid; i < 2 * hk; i += kDnThreads) {
            const int c = i < hk ? kh * hk + i : nq + kh * hk + (i - hk);
            A.win[(size_t)wslot * A.C + c] = __ldg(A.qkv + c);
        }
    for (int j = j0 + tid; j < j1; j += kDnThreads) {
        const int c = 2 * nq + h * hv + j;
        A.win[(size_t)wslot * A.C + c] = __ldg(A.qkv + c);
    }
    // L2 norms of q (warp 0) and k (warp 1).
    if (warp < 2) {
        float *v = warp ? kv : qv;
        float nrm = __fsqrt_rn(warp_sumsq64(v, hk, lane));
        nrm = fmaxf(nrm, A.eps);
        const float r = __fdiv_rn(1.0f, nrm);
        __syncwarp();
        for (int i = lane; i < hk; i += 32) v[i] = __fmul_rn(v[i], r);
    }
    __syncthreads();
    // The recurrence, one warp per row.
    const int per = hk / 32;
    float kr[kDnMaxPerLane], qr[kDnMaxPerLane];
#pragma unroll
    for (int e = 0; e < kDnMaxPerLane; ++e) {
        kr[e] = e < per ? kv[lane + 32 * e] : 0.f;
        qr[e] = e < per ? qv[lane + 32 * e] : 0.f;
    }
    const float decay = sh_decay, beta = sh_beta;
    for (int j = j0 + warp; j < j1; j += kDnWarps) {
        float *Mj = A.S + ((size_t)h * hv + j) * hk;
        float m[kDnMaxPerLane];
        float dk = 0.f;
#pragma unroll
        for (int e = 0; e < kDnMaxPerLane; ++e)
            if (e < per) {
                m[e] = __fmul_rn(Mj[lane + 32 * e], decay);
                dk = fmaf(m[e], kr[e], dk);
            }
        for (int o = 16; o; o >>= 1) dk += __shfl_xor_sync(0xffffffffu, dk, o);
        const float delta = __fmul_rn(__fsub_rn(vv[j - j0], dk), beta);
        float dq = 0.f;
#pragma unroll
        for (int e = 0; e < kDnMaxPerLane; ++e)
            if (e < per) {
                m[e] = __fadd_rn(m[e], __fmul_rn(delta, kr[e]));
                Mj[lane + 32 * e] = m[e];
                dq = fmaf(m[e], qr[e], dq);
            }
        for (int o = 16; o; o >>= 1) dq += __shfl_xor_sync(0xffffffffu, dq, o);
        if (lane == 0) A.part[(size_t)h * hv + j] = __fmul_rn(dq, A.scale);
    }
    // Arrive; the head's last CTA normalises, gates and writes the head.
    __threadfence();
    __syncthreads();
    if (tid == 0) last_s = atomicAdd(A.cnt + h, 1u) == (unsigned)(A.nsplit - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    float *o = dsm;  // reuse: [hv]
    for (int j = tid; j < hv; j += kDnThreads) o[j] = __ldcg(A.part + (size_t)h * hv + j);
    __syncthreads();
    if (warp == 0) {
        const float ss = warp_sumsq64(o, hv, lane);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hv), A.eps)));
        if (lane == 0) sh_decay = r;
    }
    __syncthreads();
    const float r = sh_decay;
    const int gpos = kh * (A.nv / nk) + h / nk;
    for (int j = tid; j < hv; j += kDnThreads) {
        const float nv_ = __fmul_rn(__fmul_rn(o[j], r), __ldg(A.norm_w + j));
        const float v = __fmul_rn(nv_, silu_dn(__ldg(A.z + (size_t)h * hv + j)));
        A.out[(size_t)gpos * hv + j] = v;
        if (A.tp.world) tp_push_all(A.tp, (size_t)gpos * hv + j, v);  // tensor-parallel gather
    }
    if (tid == 0) A.cnt[h] = 0u;
}

trx_status launch_deltanet(const DnArgs &A, uint32_t *err, cudaStream_t st) {
    const size_t smem = (size_t)(2 * A.hk + (A.rows > A.hv ? A.rows : A.hv)) * 4;
    return note_cuda(launch_kernel(deltanet_kernel, dim3(A.nsplit, A.nv, A.nseq > 1 ? A.nseq : 1), dim3(kDnThreads),
                                   smem, st, A, err));
}

}  // namespace trx
