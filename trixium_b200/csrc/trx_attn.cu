// GQA decode attention for B200 (sm_100a): one new token against the fp16 KV cache, the decode
// step of model/mirror.py:945-996 (model/golden.py:361-398).
//
// One launch does the whole step:
//  * per query head: RMSNorm with the canonical 64-partial sum of squares (mirror.py:576-591,
//    :697-700), then neox RoPE over the first rope_n dims with cos/sin of fp32(pos * freq)
//    (mirror.py:954-961);
//  * the new key (normalised, rotated) and value are rounded to fp16 and written to the cache at
//    position pos by the CTA whose chunk holds pos;
//  * split-K over the cache: CTA (s, kv head) owns positions [s*chunk, (s+1)*chunk) and every query
//    head of its group (GQA: head h reads kv head h / (H/Hkv)).  It stages the K and V rows of its
//    chunk in shared memory with cp.async, forms the scores q.k * 1/sqrt(hd), the chunk's max and
//    exp-sum and the exp-weighted sum of V rows, and writes (max, sum, o) to a scratch partial;
//  * the last CTA of a kv head to arrive (an atomic count, reset by that CTA) merges the partials:
//    o = sum_s e^(m_s-M) o_s * 1/(sum_s e^(m_s-M) l_s) (one reciprocal per head, as mirror.py:984
//    and ggml), times sigmoid(gate) for gated heads (mirror.py:992-993).
// The position is read from device memory, so a captured CUDA graph replays every step.  CTAs
// past the position only arrive at the count.  Memory-bound on the KV stream: 4*hd bytes per
// (position, kv head) read once.
#include <cstdint>
#include <cstring>
#include <mutex>
#include <cuda_fp16.h>
#include <cooperative_groups.h>
#include <cstdlib>
#include <cuda_runtime.h>

#include "trx_common.cuh"
#include "trx_internal.h"

namespace trx {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;

// Canonical RMSNorm of one head vector in shared memory, by one warp: partial j (j < 64) sums
// v[i]^2 over i = j, j+64, ... in order, then the halving tree; r = 1/sqrt(ss/n + eps) in fp32;
// v = (v*r)*w.
__device__ void head_rmsnorm(float *v, int hd, const float *w, float eps, int lane) {
    float p0 = 0.f, p1 = 0.f;
    for (int i = lane; i < hd; i += 64) p0 = __fadd_rn(p0, __fmul_rn(v[i], v[i]));
    for (int i = lane + 32; i < hd; i += 64) p1 = __fadd_rn(p1, __fmul_rn(v[i], v[i]));
    float a = __fadd_rn(p0, p1);
    for (int o = 16; o; o >>= 1) a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, o));
    const float ss = __shfl_sync(0xffffffffu, a, 0);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
    __syncwarp();
    for (int i = lane; i < hd; i += 32) v[i] = __fmul_rn(__fmul_rn(v[i], r), w ? __ldg(w + i) : 1.0f);
    __syncwarp();
}

// neox RoPE over dims [0, 2*half): pairs (d, d + half), angle fp32(pos * freq[d]).
__device__ void head_rope(float *v, int half, const float *freq, int pos, int lane) {
    for (int d = lane; d < half; d += 32) {
        const float ang = __fmul_rn((float)pos, __ldg(freq + d));
        const float c = cosf(ang), s = sinf(ang);
        const float x0 = v[d], x1 = v[d + half];
        v[d] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        v[d + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    __syncwarp();
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return __half22float2(h);
}

__device__ __forceinline__ void cp16_attn(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// CT: the cache element type, __half (the build's fp16 KV cache) or float (the fp32 cache of the
// reference mirror, model/mirror.py:966, for parity runs).
template <typename CT>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(AttnArgs A, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x, kh = blockIdx.y;
    if (blockIdx.z) {  // sequence z of a batch: its own inputs, cache, position, output and scratch
        const long long z = blockIdx.z;
        A.q += z * A.q_bs;
        A.k += z * A.kv_bs;
        A.v += z * A.kv_bs;
        A.kc = reinterpret_cast<__half *>(reinterpret_cast<CT *>(A.kc) + z * A.cache_bs);
        A.vc = reinterpret_cast<__half *>(reinterpret_cast<CT *>(A.vc) + z * A.cache_bs);
        A.pos += z;
        A.out += z * A.out_bs;
        A.part += z * A.part_bs;
        A.cnt += z * A.Hkv;
    }
    const int hd = A.hd, rep = A.H / A.Hkv, chunk = A.chunk;
    pdl_trigger();
    pdl_wait();
    const int pos = *A.pos;
    if (pos < 0 || pos >= A.max_pos) {  // every CTA reads the same position: all leave together
        if (tid == 0 && s == 0 && kh == 0) atomicOr(err, TRX_DEV_RANGE);
        return;
    }
    constexpr int EPP = 16 / (int)sizeof(CT);  // cache elements per 16-byte piece
    const int rowh = hd + EPP;  // elements per staged row (16 bytes of padding: conflict-free rows)
    CT *kt = reinterpret_cast<CT *>(smem);
    CT *vt = kt + chunk * rowh;
    float *qs = reinterpret_cast<float *>(vt + chunk * rowh);  // [rep][hd]
    float *knew = qs + rep * hd;                                // [hd]
    float *sc = knew + hd;                                      // [rep][chunk]
    float *mrow = sc + rep * chunk;                             // [rep]
    float *lrow = mrow + rep;                                   // [rep]
    __shared__ int last_s;

    const int t0 = s * chunk;
    const int n = min(chunk, pos + 1 - t0);  // positions of this chunk in use (<= 0: none)
    const int stride_t = A.Hkv * hd;         // elements between positions in the cache
    CT *const kcache = reinterpret_cast<CT *>(A.kc);
    CT *const vcache = reinterpret_cast<CT *>(A.vc);
    float *part = A.part + (size_t)(kh * A.nsplit + s) * rep * (hd + 2);
    if (n > 0) {
        // Query heads of this group: RMSNorm + RoPE, one warp per head.
        for (int r = warp; r < rep; r += kAttnWarps) {
            const float *qh = A.q + (size_t)(kh * rep + r) * A.qstride;
            float *v = qs + r * hd;
            for (int i = lane; i < hd; i += 32) v[i] = __ldg(qh + i);
            __syncwarp();
            head_rmsnorm(v, hd, A.qn, A.eps, lane);
            head_rope(v, A.rope_half, A.freq, pos, lane);
        }
        // The new key and value: into the cache, by the CTA whose chunk holds pos.
        if (pos >= t0 && pos < t0 + chunk && warp == kAttnWarps - 1) {
            const float *kg = A.k + (size_t)kh * hd;
            for (int i = lane; i < hd; i += 32) knew[i] = __ldg(kg + i);
            __syncwarp();
            head_rmsnorm(knew, hd, A.kn, A.eps, lane);
            head_rope(knew, A.rope_half, A.freq, pos, lane);
            CT *kc = kcache + (size_t)pos * stride_t + (size_t)kh * hd;
            CT *vc = vcache + (size_t)pos * stride_t + (size_t)kh * hd;
            const float *vg = A.v + (size_t)kh * hd;
            for (int i = lane; i < hd; i += 32) {
                if constexpr (sizeof(CT) == 2) {
                    kc[i] = __float2half_rn(knew[i]);
                    vc[i] = __float2half_rn(__ldg(vg + i));
                } else {
                    kc[i] = knew[i];
                    vc[i] = __ldg(vg + i);
                }
            }
        }
        __syncthreads();  // queries ready; the new cache row is visible to this CTA's copies
        // Stage K and V rows [t0, t0 + n).
        const int pieces = hd / EPP;  // 16-byte pieces per row
        for (int i = tid; i < n * pieces; i += kAttnThreads) {
            const int t = i / pieces, j = i - t * pieces;
            const size_t g = (size_t)(t0 + t) * stride_t + (size_t)kh * hd + EPP * j;
            cp16_attn(kt + t * rowh + EPP * j, kcache + g);
            cp16_attn(vt + t * rowh + EPP * j, vcache + g);
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // Scores.
        for (int i = tid; i < rep * n; i += kAttnThreads) {
            const int r = i / n, t = i - r * n;
            const float *qv = qs + r * hd;
            float acc = 0.f;
            const float4 *q4 = reinterpret_cast<const float4 *>(qv);
            if constexpr (sizeof(CT) == 2) {
                const uint4 *kr = reinterpret_cast<const uint4 *>(kt + t * rowh);
                for (int j = 0; j < pieces; ++j) {
                    const uint4 w = kr[j];
                    const float4 qa = q4[2 * j], qb = q4[2 * j + 1];
                    const float2 f0 = h2_to_f2(w.x), f1 = h2_to_f2(w.y), f2 = h2_to_f2(w.z), f3 = h2_to_f2(w.w);
                    acc = fmaf(qa.x, f0.x, acc);
                    acc = fmaf(qa.y, f0.y, acc);
                    acc = fmaf(qa.z, f1.x, acc);
                    acc = fmaf(qa.w, f1.y, acc);
                    acc = fmaf(qb.x, f2.x, acc);
                    acc = fmaf(qb.y, f2.y, acc);
                    acc = fmaf(qb.z, f3.x, acc);
                    acc = fmaf(qb.w, f3.y, acc);
                }
            } else {
                const float4 *kr = reinterpret_cast<const float4 *>(kt + t * rowh);
                for (int j = 0; j < pieces; ++j) {
                    const float4 w = kr[j], qa = q4[j];
                    acc = fmaf(qa.x, w.x, acc);
                    acc = fmaf(qa.y, w.y, acc);
                    acc = fmaf(qa.z, w.z, acc);
                    acc = fmaf(qa.w, w.w, acc);
                }
            }
            sc[r * chunk + t] = __fmul_rn(acc, A.scale);
        }
        __syncthreads();
        // Chunk max and exp-sum per head, one warp per head.
        for (int r = warp; r < rep; r += kAttnWarps) {
            float m = -INFINITY;
            for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[r * chunk + t]);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float l = 0.f;
            for (int t = lane; t < n; t += 32) {
                const float e = expf(__fsub_rn(sc[r * chunk + t], m));
                sc[r * chunk + t] = e;
                l += e;
            }
            for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) {
                mrow[r] = m;
                lrow[r] = l;
            }
        }
        __syncthreads();
        // Exp-weighted sum of V rows, two dims per thread.
        const int hp = hd / 2;
        for (int i = tid; i < rep * hp; i += kAttnThreads) {
            const int r = i / hp, dp = i - r * hp;
            const float *e = sc + r * chunk;
            float ax = 0.f, ay = 0.f;
            for (int t = 0; t < n; ++t) {
                float2 f;
                if constexpr (sizeof(CT) == 2)
                    f = __half22float2(reinterpret_cast<const __half2 *>(vt + t * rowh)[dp]);
                else
                    f = reinterpret_cast<const float2 *>(vt + t * rowh)[dp];
                ax = fmaf(e[t], f.x, ax);
                ay = fmaf(e[t], f.y, ay);
            }
            reinterpret_cast<float2 *>(part + r * (hd + 2) + 2)[dp] = make_float2(ax, ay);
        }
        if (tid < rep) {
            part[tid * (hd + 2)] = mrow[tid];
            part[tid * (hd + 2) + 1] = lrow[tid];
        }
    }
    // Arrive; the last CTA of this kv head merges the active chunks.
    __threadfence();
    __syncthreads();
    if (tid == 0) last_s = atomicAdd(A.cnt + kh, 1u) == (unsigned)(A.nsplit - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    const int ns = pos / chunk + 1;
    const float *pk = A.part + (size_t)kh * A.nsplit * rep * (hd + 2);
    // Chunk maxima and sums of every head, staged in shared memory with all their loads in flight
    // at once (the K and V tiles are no longer needed): wm[rep][ns], wl[rep][ns].
    float *wm = reinterpret_cast<float *>(smem);
    float *wl = wm + rep * ns;
    for (int i = tid; i < rep * ns; i += kAttnThreads) {
        const int r = i / ns, j = i - r * ns;
        const float *pj = pk + (size_t)(j * rep + r) * (hd + 2);
        wm[i] = __ldcg(pj);
        wl[i] = __ldcg(pj + 1);
    }
    __syncthreads();
    // Weights per head: w_j = e^(m_j - M) / sum_j e^(m_j - M) l_j (one reciprocal per head).
    for (int r = warp; r < rep; r += kAttnWarps) {
        float M = -INFINITY;
        for (int j = lane; j < ns; j += 32) M = fmaxf(M, wm[r * ns + j]);
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
        for (int j = lane; j < ns; j += 32) {
            const float w = expf(__fsub_rn(wm[r * ns + j], M));
            wm[r * ns + j] = w;
            L = fmaf(w, wl[r * ns + j], L);
        }
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float inv = __fdiv_rn(1.0f, L);
        __syncwarp();
        for (int j = lane; j < ns; j += 32) wm[r * ns + j] = __fmul_rn(wm[r * ns + j], inv);
    }
    __syncthreads();
    for (int i = tid; i < rep * hd; i += kAttnThreads) {
        const int r = i / hd, d = i - r * hd;
        const float *w = wm + r * ns;
        const float *pd = pk + (size_t)r * (hd + 2) + 2 + d;
        const size_t step = (size_t)rep * (hd + 2);
        float O0 = 0.f, O1 = 0.f, O2 = 0.f, O3 = 0.f;
        int j = 0;
        for (; j + 16 <= ns; j += 16) {  // sixteen independent L2 loads in flight
            float a[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) a[u] = __ldcg(pd + (j + u) * step);
#pragma unroll
            for (int u = 0; u < 16; u += 4) {
                O0 = fmaf(w[j + u], a[u], O0);
                O1 = fmaf(w[j + u + 1], a[u + 1], O1);
                O2 = fmaf(w[j + u + 2], a[u + 2], O2);
                O3 = fmaf(w[j + u + 3], a[u + 3], O3);
            }
        }
        {
            float a[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) a[u] = j + u < ns ? __ldcg(pd + (j + u) * step) : 0.f;
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (j + u < ns) O0 = fmaf(w[j + u], a[u], O0);
        }
        float o = (O0 + O1) + (O2 + O3);
        const int h = kh * rep + r;
        if (A.gated) {
            const float g = __ldg(A.q + (size_t)h * A.qstride + hd + d);
            o = __fmul_rn(o, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
        }
        A.out[(size_t)h * hd + d] = o;
        if (A.tp.world) tp_push_all(A.tp, (size_t)h * hd + d, o);  // tensor-parallel gather (tagged words)
    }
    if (tid == 0) A.cnt[kh] = 0u;
}

// Cluster decode attention -------------------------------------------------------------------
// The same step with the splits of a kv head in one thread-block cluster (at most 16 CTAs): the
// partials are merged through distributed shared memory instead of global scratch and an arrival
// count.  Per CTA (split s of kv head kh, 256 threads):
//  * before the dependency wait: the q/k norm weights and the RoPE frequencies into shared memory;
//  * after it: the position, then the K and V rows [t0, min(t0 + chunk, pos + 1)) staged with
//    cp.async while warps 0..REP-1 normalise and rotate their query heads; the CTA whose chunk
//    holds pos normalises and rotates the new key and writes the new K/V row (fp16) to the cache
//    and into its own tiles;
//  * scores: hd/DPL lanes per position, each holding DPL dims of every query head in registers,
//    the dot products finished by shuffles; softmax per head (one warp each);
//  * P.V: hd/4 threads per position group, each 4 dims of every head, the groups' partial sums
//    added in a fixed order;
//  * merge: after a cluster barrier, every CTA forms the per-head weights
//    w_j = e^(m_j - M) * (1 / sum_j e^(m_j - M) l_j) from all splits' (m, l), and writes its share
//    of the outputs sum_j w_j o_j (times sigmoid(gate) for gated heads); a second barrier keeps
//    every CTA's shared memory alive until all reads are done.
namespace {
namespace cg = cooperative_groups;

constexpr int kClThreads = 256;

__device__ __forceinline__ void cp4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// head_rmsnorm / head_rope with the weights in shared memory.
__device__ void head_rmsnorm_s(float *v, int hd, const float *w, float eps, int lane) {
    float p0 = 0.f, p1 = 0.f;
    for (int i = lane; i < hd; i += 64) p0 = __fadd_rn(p0, __fmul_rn(v[i], v[i]));
    for (int i = lane + 32; i < hd; i += 64) p1 = __fadd_rn(p1, __fmul_rn(v[i], v[i]));
    float a = __fadd_rn(p0, p1);
    for (int o = 16; o; o >>= 1) a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, o));
    const float ss = __shfl_sync(0xffffffffu, a, 0);
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)hd), eps));
    __syncwarp();
    for (int i = lane; i < hd; i += 32) v[i] = __fmul_rn(__fmul_rn(v[i], r), w[i]);
    __syncwarp();
}

__device__ void head_rope_s(float *v, int half, const float *freq, int pos, int lane) {
    for (int d = lane; d < half; d += 32) {
        const float ang = __fmul_rn((float)pos, freq[d]);
        float sn, c;
        sincosf(ang, &sn, &c);
        const float x0 = v[d], x1 = v[d + half];
        v[d] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        v[d + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    __syncwarp();
}

struct ClLayout {  // float offsets after the K and V tiles
    int qs, cq, ck, cf, knew, sc, et, pp, om, ml, wt, mg, total;
};

__host__ __device__ inline ClLayout cl_layout(int hd, int rep, int repp, int chunk) {
    ClLayout L;
    int o = 0;
    L.qs = o; o += rep * hd;
    L.cq = o; o += hd;
    L.ck = o; o += hd;
    L.cf = o; o += hd / 2;
    L.knew = o; o += hd;
    L.sc = o; o += rep * chunk;
    L.et = o; o += chunk * repp;
    L.pp = o; o += 4 * kClThreads * rep;  // (threads / (hd/4)) position groups x rep x hd
    L.om = o; o += rep * hd;
    L.ml = o; o += 2 * rep;
    L.wt = o; o += 16 * rep;
    L.mg = o;  // the merge area (16 slots), when it gets its own region
    L.total = o;
    return L;
}

__host__ __device__ inline size_t cl_smem_bytes(int hd, int rep, int chunk, int merge_slots) {
    const int repp = rep <= 4 ? 4 : 8;
    const size_t tiles = (size_t)chunk * (hd + 8) * 2 + (size_t)chunk * hd * 2;
    return tiles + ((size_t)cl_layout(hd, rep, repp, chunk).total + (size_t)merge_slots * rep * (hd + 2)) * 4;
}

template <int REP, int DPL>
__global__ void __launch_bounds__(kClThreads) attn_cluster_kernel(AttnArgs A, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int REPP = REP <= 4 ? 4 : 8;
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x, kh = blockIdx.y, ns = A.nsplit;
    const int hd = A.hd, chunk = A.chunk, rowk = hd + 8;
    __half *const kt = reinterpret_cast<__half *>(smem);  // [chunk][hd + 8]
    __half *const vt = kt + (size_t)chunk * rowk;         // [chunk][hd]
    float *const fb = reinterpret_cast<float *>(vt + (size_t)chunk * hd);
    const ClLayout Ly = cl_layout(hd, REP, REPP, chunk);
    float *const qs = fb + Ly.qs, *const cq = fb + Ly.cq, *const ck = fb + Ly.ck, *const cf = fb + Ly.cf;
    float *const knew = fb + Ly.knew, *const sc = fb + Ly.sc, *const et = fb + Ly.et, *const pp = fb + Ly.pp;
    float *const om = fb + Ly.om, *const mrow = fb + Ly.ml, *const lrow = mrow + REP, *const wt = fb + Ly.wt;

    pdl_trigger();
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");  // waited on before the merge
    // Weights written by no kernel: requested before the wait.
    for (int i = tid; i < hd; i += kClThreads) {
        cp4(cq + i, A.qn + i);
        cp4(ck + i, A.kn + i);
    }
    for (int i = tid; i < A.rope_half; i += kClThreads) cp4(cf + i, A.freq + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
    pdl_wait();
    const int pos = *A.pos;
    if (pos < 0 || pos >= A.max_pos) {  // every CTA reads the same position: all leave together
        if (tid == 0 && s == 0 && kh == 0) atomicOr(err, TRX_DEV_RANGE);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        return;
    }
    const int t0 = s * chunk;
    const int n = max(0, min(chunk, pos + 1 - t0));
    const bool owner = pos >= t0 && pos < t0 + chunk;
    const int stride_t = A.Hkv * hd;
    {
        const int lp = __ffs(hd) - 4;  // log2(hd / 8): 16-byte pieces per row
        for (int i = tid; i < (n << lp); i += kClThreads) {
            const int t = i >> lp, j = i & ((1 << lp) - 1);
            if (t0 + t == pos) continue;  // written below by this CTA
            const size_t g = (size_t)(t0 + t) * stride_t + (size_t)kh * hd + 8 * j;
            cp16_attn(kt + t * rowk + 8 * j, A.kc + g);
            cp16_attn(vt + t * hd + 8 * j, A.vc + g);
        }
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 1;" ::: "memory");
    __syncthreads();  // the norm weights and frequencies are visible
    if (n > 0) {
        for (int r = warp; r < REP; r += kClThreads / 32) {
            const float *qh = A.q + (size_t)(kh * REP + r) * A.qstride;
            float *v = qs + r * hd;
            for (int i = lane; i < hd; i += 32) v[i] = qh[i];
            __syncwarp();
            head_rmsnorm_s(v, hd, cq, A.eps, lane);
            head_rope_s(v, A.rope_half, cf, pos, lane);
        }
        if (owner && warp == kClThreads / 32 - 1) {
            const float *kg = A.k + (size_t)kh * hd;
            for (int i = lane; i < hd; i += 32) knew[i] = kg[i];
            __syncwarp();
            head_rmsnorm_s(knew, hd, ck, A.eps, lane);
            head_rope_s(knew, A.rope_half, cf, pos, lane);
            const int tp = pos - t0;
            __half *kc = A.kc + (size_t)pos * stride_t + (size_t)kh * hd;
            __half *vc = A.vc + (size_t)pos * stride_t + (size_t)kh * hd;
            const float *vg = A.v + (size_t)kh * hd;
            for (int i = lane; i < hd; i += 32) {
                const __half kh16 = __float2half_rn(knew[i]), vh16 = __float2half_rn(vg[i]);
                kc[i] = kh16;
                vc[i] = vh16;
                kt[tp * rowk + i] = kh16;
                vt[tp * hd + i] = vh16;
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // K/V tiles and queries ready

    if (n > 0) {
        // Scores: lpp lanes per position, DPL dims each: pieces of 8 dims at 8*(sub + lpp*c), so
        // the lanes of a quarter warp read 128 contiguous bytes of a K row.  Two positions per
        // step (independent chains).
        const int lpp = hd / DPL, ppw = 32 / lpp;
        const int sub = lane % lpp, pl = lane / lpp;
        constexpr int NP = DPL / 8;  // 8-dim pieces per lane
        float qr[REP][DPL];
#pragma unroll
        for (int r = 0; r < REP; ++r)
#pragma unroll
            for (int c = 0; c < NP; ++c) {
                const float *qp = qs + r * hd + 8 * (sub + lpp * c);
                const float4 a = *reinterpret_cast<const float4 *>(qp), b = *reinterpret_cast<const float4 *>(qp + 4);
                qr[r][8 * c] = a.x; qr[r][8 * c + 1] = a.y; qr[r][8 * c + 2] = a.z; qr[r][8 * c + 3] = a.w;
                qr[r][8 * c + 4] = b.x; qr[r][8 * c + 5] = b.y; qr[r][8 * c + 6] = b.z; qr[r][8 * c + 7] = b.w;
            }
        const int step = (kClThreads / 32) * ppw;
        for (int tb = warp * ppw; tb < n; tb += 2 * step) {
            float acc[2][REP];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int t = tb + h * step + pl;
                float kv[DPL];
#pragma unroll
                for (int c = 0; c < NP; ++c) {
                    uint4 w = make_uint4(0u, 0u, 0u, 0u);
                    if (t < n) w = *reinterpret_cast<const uint4 *>(kt + t * rowk + 8 * (sub + lpp * c));
                    const float2 f0 = h2_to_f2(w.x), f1 = h2_to_f2(w.y), f2 = h2_to_f2(w.z), f3 = h2_to_f2(w.w);
                    kv[8 * c] = f0.x; kv[8 * c + 1] = f0.y; kv[8 * c + 2] = f1.x; kv[8 * c + 3] = f1.y;
                    kv[8 * c + 4] = f2.x; kv[8 * c + 5] = f2.y; kv[8 * c + 6] = f3.x; kv[8 * c + 7] = f3.y;
                }
#pragma unroll
                for (int r = 0; r < REP; ++r) {
                    float a0 = 0.f, a1 = 0.f;
#pragma unroll
                    for (int i = 0; i < DPL; i += 2) {
                        a0 = fmaf(qr[r][i], kv[i], a0);
                        a1 = fmaf(qr[r][i + 1], kv[i + 1], a1);
                    }
                    acc[h][r] = a0 + a1;
                }
            }
            for (int o = lpp >> 1; o; o >>= 1)
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int r = 0; r < REP; ++r) acc[h][r] += __shfl_xor_sync(0xffffffffu, acc[h][r], o);
            if (sub == 0)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int t = tb + h * step + pl;
                    if (t < n)
#pragma unroll
                        for (int r = 0; r < REP; ++r) sc[r * chunk + t] = __fmul_rn(acc[h][r], A.scale);
                }
        }
        __syncthreads();
        // Softmax per head: e = exp(s - m) into et[t][REPP], chunk max and sum.
        for (int r = warp; r < REP; r += kClThreads / 32) {
            float m = -INFINITY;
            for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[r * chunk + t]);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float l = 0.f;
            for (int t = lane; t < n; t += 32) {
                const float e = expf(__fsub_rn(sc[r * chunk + t], m));
                et[t * REPP + r] = e;
                l += e;
            }
            for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) {
                mrow[r] = m;
                lrow[r] = l;
            }
        }
        __syncthreads();
        // P.V: position group grp (positions grp, grp + ngrp, ...), 4 dims per thread.
        const int tpg = hd / 4, ngrp = kClThreads / tpg;
        const int grp = tid / tpg, dq = tid - grp * tpg;
        float acc[REP][4];
#pragma unroll
        for (int r = 0; r < REP; ++r) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.f;
        for (int t = grp; t < n; t += ngrp) {
            const uint2 vv = *reinterpret_cast<const uint2 *>(vt + t * hd + 4 * dq);
            const float2 v01 = h2_to_f2(vv.x), v23 = h2_to_f2(vv.y);
            float e[REPP];
#pragma unroll
            for (int i = 0; i < REPP; i += 4) {
                const float4 e4 = *reinterpret_cast<const float4 *>(et + t * REPP + i);
                e[i] = e4.x;
                e[i + 1] = e4.y;
                e[i + 2] = e4.z;
                e[i + 3] = e4.w;
            }
#pragma unroll
            for (int r = 0; r < REP; ++r) {
                acc[r][0] = fmaf(e[r], v01.x, acc[r][0]);
                acc[r][1] = fmaf(e[r], v01.y, acc[r][1]);
                acc[r][2] = fmaf(e[r], v23.x, acc[r][2]);
                acc[r][3] = fmaf(e[r], v23.y, acc[r][3]);
            }
        }
#pragma unroll
        for (int r = 0; r < REP; ++r)
            *reinterpret_cast<float4 *>(pp + ((size_t)grp * REP + r) * hd + 4 * dq) =
                make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        __syncthreads();
        for (int i = tid; i < REP * hd; i += kClThreads) {
            float o = 0.f;
            for (int g = 0; g < ngrp; ++g) o += pp[(size_t)g * REP * hd + i];
            om[i] = o;
        }
    } else {
        for (int i = tid; i < REP * hd; i += kClThreads) om[i] = 0.f;
        if (tid < REP) {
            mrow[tid] = -INFINITY;
            lrow[tid] = 0.f;
        }
    }
    // Merge at rank 0: every CTA stores its (m, l, o) into slot s of rank 0's merge area (its own
    // region when the plan found room, else rank 0's K/V tiles once every CTA is done with them),
    // one cluster barrier, then rank 0 merges from its own shared memory.
    const int slot = REP * (hd + 2);
    float *mg = A.merge_own ? fb + Ly.mg : reinterpret_cast<float *>(smem);
    // Every CTA of the cluster has started (arrival at entry) before any shared memory of another
    // is written; this CTA's (m, l, o) are complete.
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (!A.merge_own)
        cluster.sync();  // also: every CTA is done with its K/V tiles
    else
        __syncthreads();
    {
        float *dst = cluster.map_shared_rank(mg, 0) + (size_t)s * slot;
        for (int i = tid; i < slot; i += kClThreads) {
            const int r = i / (hd + 2), j = i - r * (hd + 2);
            dst[i] = j == 0 ? mrow[r] : (j == 1 ? lrow[r] : om[r * hd + j - 2]);
        }
    }
    cluster.sync();  // every split's (m, l, o) is in rank 0's merge area
    if (s != 0) return;
    for (int r = warp; r < REP; r += kClThreads / 32) {
        const float mj = lane < ns ? mg[lane * slot + r * (hd + 2)] : -INFINITY;
        const float lj = lane < ns ? mg[lane * slot + r * (hd + 2) + 1] : 0.f;
        float M = mj;
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = lane < ns ? expf(__fsub_rn(mj, M)) : 0.f;
        float L = w * lj;
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float inv = __fdiv_rn(1.0f, L);
        if (lane < ns) wt[r * 16 + lane] = __fmul_rn(w, inv);
    }
    __syncthreads();
    for (int i = tid; i < REP * hd; i += kClThreads) {
        const int r = i / hd, d = i - r * hd;
        const float *src = mg + r * (hd + 2) + 2 + d;
        float o = 0.f;
        for (int j = 0; j < ns; ++j) o = fmaf(wt[r * 16 + j], src[(size_t)j * slot], o);
        const int h = kh * REP + r;
        if (A.gated) {
            const float g = A.q[(size_t)h * A.qstride + hd + d];
            o = __fmul_rn(o, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
        }
        A.out[(size_t)h * hd + d] = o;
        if (A.tp.world) tp_push_all(A.tp, (size_t)h * hd + d, o);  // tensor-parallel gather (tagged words)
    }
}

// Tensor-core variant (head dim 64 or 128, at most 8 query heads per kv head): the same
// prologue and merge, with scores and P.V on mma.sync m16n8k16 (f16 in, f32 accumulate).  Per
// warp, 16-position blocks: S = Q K^T with the heads as the 16 rows (rows >= REP zero) and the
// fp32 queries split into two fp16 parts (q = hi + lo, both products accumulated), then an online
// softmax per head within the warp, then O^T += V^T P^T with V^T fragments from ldmatrix.trans and
// P^T fragments taken straight from the score accumulators (p split the same way).  K and V are
// fp16 already, so every product is exact up to the f32 accumulation.  The warps' (m, l, O) are
// combined in shared memory in a fixed order.
struct MmaLayout {  // float offsets after the K and V tiles
    int qs, cq, ck, cf, knew, wp, om, ml, wt, mg, total;
};

__host__ __device__ inline MmaLayout mma_layout(int hd, int rep) {
    MmaLayout L;
    int o = 0;
    L.qs = o; o += rep * hd;
    L.cq = o; o += hd;
    L.ck = o; o += hd;
    L.cf = o; o += hd / 2;
    L.knew = o; o += hd;
    L.wp = o; o += (kClThreads / 32) * rep * (hd + 2);  // per-warp (m, l, o)
    L.om = o; o += rep * hd;
    L.ml = o; o += 2 * rep;
    L.wt = o; o += 16 * rep;
    L.mg = o;
    L.total = o;
    return L;
}

__host__ __device__ inline size_t mma_smem_bytes(int hd, int rep, int chunk, int merge_slots) {
    return (size_t)2 * chunk * (hd + 8) * 2 + ((size_t)mma_layout(hd, rep).total + (size_t)merge_slots * rep * (hd + 2)) * 4;
}

// x = hi + lo with hi = fp16(x), lo = fp16(x - hi), for a pair: (hi word, lo word).
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
    const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
    const __half2 H = __halves2half2(h0, h1), Lo = __halves2half2(l0, l1);
    memcpy(&hi, &H, 4);
    memcpy(&lo, &Lo, 4);
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

template <int HD>
__global__ void __launch_bounds__(kClThreads, 2) attn_mma_kernel(AttnArgs A, uint32_t *err) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int KS = HD / 16;  // 16-dim steps
    constexpr int NWARP = kClThreads / 32;
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const int s = blockIdx.x, kh = blockIdx.y, ns = A.nsplit;
    const int chunk = A.chunk, rowk = HD + 8, rep = A.H / A.Hkv;
    __half *const kt = reinterpret_cast<__half *>(smem);  // [chunk][HD + 8]
    __half *const vt = kt + (size_t)chunk * rowk;         // [chunk][HD + 8]
    float *const fb = reinterpret_cast<float *>(vt + (size_t)chunk * rowk);
    const MmaLayout Ly = mma_layout(HD, rep);
    float *const qs = fb + Ly.qs, *const cq = fb + Ly.cq, *const ck = fb + Ly.ck, *const cf = fb + Ly.cf;
    float *const knew = fb + Ly.knew, *const wp = fb + Ly.wp, *const om = fb + Ly.om;
    float *const mrow = fb + Ly.ml, *const lrow = mrow + rep, *const wt = fb + Ly.wt;

    pdl_trigger();
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");  // waited on before the merge
    for (int i = tid; i < HD; i += kClThreads) {
        cp4(cq + i, A.qn + i);
        cp4(ck + i, A.kn + i);
    }
    for (int i = tid; i < A.rope_half; i += kClThreads) cp4(cf + i, A.freq + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
    // The K/V rows of the whole chunk (within the cache) are staged before the dependency wait: the
    // rows before the current position were written by earlier decode steps, which completed before
    // any kernel of this step started; row pos (this step's) and the rows after it are replaced or
    // masked below.  The copies overlap the predecessor's tail.
    const int t0 = s * chunk;
    const int stride_t = A.Hkv * HD;
    constexpr int lp = HD == 64 ? 3 : 4;  // log2(HD / 8)
    {
        const int nmax = max(0, min(chunk, A.max_pos - t0));
        for (int i = tid; i < (nmax << lp); i += kClThreads) {
            const int t = i >> lp, j = i & ((1 << lp) - 1);
            const size_t gix = (size_t)(t0 + t) * stride_t + (size_t)kh * HD + 8 * j;
            cp16_attn(kt + t * rowk + 8 * j, A.kc + gix);
            cp16_attn(vt + t * rowk + 8 * j, A.vc + gix);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    pdl_wait();
    const int pos = *A.pos;
    if (pos < 0 || pos >= A.max_pos) {  // every CTA reads the same position: all leave together
        if (tid == 0 && s == 0 && kh == 0) atomicOr(err, TRX_DEV_RANGE);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        return;
    }
    const int n = max(0, min(chunk, pos + 1 - t0));
    const int nb16 = (n + 15) >> 4;  // 16-position blocks in use
    const bool owner = pos >= t0 && pos < t0 + chunk;
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();  // the norm weights and frequencies are visible
    if (n > 0) {
        for (int r = warp; r < rep; r += NWARP) {
            const float *qh = A.q + (size_t)(kh * rep + r) * A.qstride;
            float *v = qs + r * HD;
            for (int i = lane; i < HD; i += 32) v[i] = qh[i];
            __syncwarp();
            head_rmsnorm_s(v, HD, cq, A.eps, lane);
            head_rope_s(v, A.rope_half, cf, pos, lane);
        }
        if (owner && warp == NWARP - 1) {
            const float *kg = A.k + (size_t)kh * HD;
            for (int i = lane; i < HD; i += 32) knew[i] = kg[i];
            __syncwarp();
            head_rmsnorm_s(knew, HD, ck, A.eps, lane);
            head_rope_s(knew, A.rope_half, cf, pos, lane);
            __half *kc = A.kc + (size_t)pos * stride_t + (size_t)kh * HD;
            __half *vc = A.vc + (size_t)pos * stride_t + (size_t)kh * HD;
            const float *vg = A.v + (size_t)kh * HD;
            for (int i = lane; i < HD; i += 32) {
                kc[i] = __float2half_rn(knew[i]);
                vc[i] = __float2half_rn(vg[i]);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // the staged rows have landed
    // Rows [n, 16*nb16) of the last block: zero (their scores are masked; P.V must see 0).  The
    // owner puts the new row into its tiles.
    for (int i = tid; i < ((16 * nb16 - n) << lp); i += kClThreads) {
        const int t = n + (i >> lp), j = i & ((1 << lp) - 1);
        *reinterpret_cast<uint4 *>(kt + t * rowk + 8 * j) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4 *>(vt + t * rowk + 8 * j) = make_uint4(0u, 0u, 0u, 0u);
    }
    if (n > 0 && owner && warp == NWARP - 1) {
        const int tp = pos - t0;
        const float *vg = A.v + (size_t)kh * HD;
        for (int i = lane; i < HD; i += 32) {
            kt[tp * rowk + i] = __float2half_rn(knew[i]);
            vt[tp * rowk + i] = __float2half_rn(vg[i]);
        }
    }
    __syncthreads();  // K/V tiles and queries ready

    // Per warp: blocks warp, warp + NWARP, ...  Lane (g, c): head row g; the running max and sum of
    // head g; O^T columns 2c, 2c+1 (heads) of every 16-dim tile.
    float m_run = -INFINITY, l_run = 0.f;
    float ot[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) ot[i][0] = ot[i][1] = ot[i][2] = ot[i][3] = 0.f;
    if (warp < nb16) {
        const float *qg = qs + (g < rep ? g : 0) * HD + 2 * c;  // rows g >= rep use zeros below
        const uint32_t vbase = smem_u32(vt);
        for (int b = warp; b < nb16; b += NWARP) {
            const int tb = 16 * b;
            float sh[2][4], sl[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                sh[nt][0] = sh[nt][1] = sh[nt][2] = sh[nt][3] = 0.f;
                sl[nt][0] = sl[nt][1] = sl[nt][2] = sl[nt][3] = 0.f;
                const __half *kr = kt + (tb + 8 * nt + g) * rowk + 2 * c;
#pragma unroll 2
                for (int k = 0; k < KS; ++k) {
                    // A fragments a0 (row g, dims 16k + 2c, +1) and a2 (dims + 8, + 9), split in two
                    // fp16 parts; a1 = a3 = 0 (rows g + 8).
                    const float2 xa = *reinterpret_cast<const float2 *>(qg + 16 * k);
                    const float2 xb = *reinterpret_cast<const float2 *>(qg + 16 * k + 8);
                    const bool on = g < rep;
                    uint32_t qh0, ql0, qh2, ql2;
                    split_h2(on ? xa.x : 0.f, on ? xa.y : 0.f, qh0, ql0);
                    split_h2(on ? xb.x : 0.f, on ? xb.y : 0.f, qh2, ql2);
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kr + 16 * k);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t *>(kr + 16 * k + 8);
                    mma16816(sh[nt], qh0, 0u, qh2, 0u, b0, b1);
                    mma16816(sl[nt], ql0, 0u, ql2, 0u, b0, b1);
                }
            }
            // Scores of head g at positions tb + 2c, +1 (tile 0) and tb + 8 + 2c, +1 (tile 1).
            float sv[4];
            sv[0] = (sh[0][0] + sl[0][0]) * A.scale;
            sv[1] = (sh[0][1] + sl[0][1]) * A.scale;
            sv[2] = (sh[1][0] + sl[1][0]) * A.scale;
            sv[3] = (sh[1][1] + sl[1][1]) * A.scale;
            const int tq[4] = {tb + 2 * c, tb + 2 * c + 1, tb + 8 + 2 * c, tb + 9 + 2 * c};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (tq[i] >= n) sv[i] = -INFINITY;
            float bm = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
            const float m_new = fmaxf(m_run, bm);  // finite: every block holds a position < n
            const float alpha = expf(m_run - m_new);
            float pv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pv[i] = g < rep ? expf(sv[i] - m_new) : 0.f;
            l_run = l_run * alpha + ((pv[0] + pv[1]) + (pv[2] + pv[3]));
            m_run = m_new;
            // Rescale O^T columns (heads 2c, 2c+1) by their heads' alpha.
            const float a0 = __shfl_sync(0xffffffffu, alpha, 8 * c), a1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);
#pragma unroll
            for (int i = 0; i < KS; ++i) {
                ot[i][0] *= a0;
                ot[i][1] *= a1;
                ot[i][2] *= a0;
                ot[i][3] *= a1;
            }
            uint32_t ph0, pl0, ph1, pl1;
            split_h2(pv[0], pv[1], ph0, pl0);
            split_h2(pv[2], pv[3], ph1, pl1);
            const uint32_t arow = (uint32_t)(tb + (lane & 7) + ((lane >> 4) & 1) * 8);
            const uint32_t acol = (uint32_t)(((lane >> 3) & 1) * 8);
#pragma unroll
            for (int i = 0; i < KS; ++i) {
                uint32_t v0, v1, v2, v3;
                ldsm_x4_trans(vbase + (arow * rowk + 16 * i + acol) * 2, v0, v1, v2, v3);
                mma16816(ot[i], v0, v1, v2, v3, ph0, ph1);
                mma16816(ot[i], v0, v1, v2, v3, pl0, pl1);
            }
        }
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    }
    // This warp's partial: (m, l) of head g (lanes 4g), O of heads 2c, 2c+1 at dims 16i + g, + 8.
    {
        float *w = wp + (size_t)warp * rep * (HD + 2);
        if (c == 0 && g < rep) {
            w[g * (HD + 2)] = m_run;
            w[g * (HD + 2) + 1] = l_run;
        }
#pragma unroll
        for (int i = 0; i < KS; ++i) {
            const int d = 16 * i + g;
            if (2 * c < rep) {
                w[(2 * c) * (HD + 2) + 2 + d] = ot[i][0];
                w[(2 * c) * (HD + 2) + 2 + d + 8] = ot[i][2];
            }
            if (2 * c + 1 < rep) {
                w[(2 * c + 1) * (HD + 2) + 2 + d] = ot[i][1];
                w[(2 * c + 1) * (HD + 2) + 2 + d + 8] = ot[i][3];
            }
        }
    }
    __syncthreads();
    // Combine the warps in order: M = max m_w, o = sum e^(m_w - M) o_w, l = sum e^(m_w - M) l_w.
    const int nwu = min(NWARP, max(nb16, 1));  // warps that held a block (warp 0 at least, possibly empty)
    // Warps 0-1, one lane per (row r, warp w): M_r by a shuffle over the row's 8 lanes, then the
    // warp's scale e^(m_w - M_r) into wt[8 r + w] (free until the rank-0 merge), and l_r summed in
    // warp order by the row's first lane.  rep <= 8, so 64 lanes cover every (r, w).
    if (tid < 64) {
        const int r = tid >> 3, w = tid & 7;
        const bool live = r < rep && w < nwu;
        const float mw = live ? wp[(w * rep + r) * (HD + 2)] : -INFINITY;
        float M = mw;
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 4));
        const float e = (live && M != -INFINITY) ? expf(mw - M) : 0.f;
        const float lw = live ? wp[(w * rep + r) * (HD + 2) + 1] : 0.f;
        if (r < rep) wt[r * 8 + w] = e;
        float L = 0.f;
        for (int j = 0; j < NWARP; ++j) {
            const float ej = __shfl_sync(0xffffffffu, e, (lane & ~7) + j), lj = __shfl_sync(0xffffffffu, lw, (lane & ~7) + j);
            if (j < nwu && M != -INFINITY) L = fmaf(ej, lj, L);
        }
        if (w == 0 && r < rep) {
            mrow[r] = M;
            lrow[r] = L;
        }
    }
    __syncthreads();
    // o = sum e^(m_w - M) o_w in warp order.
    for (int i = tid; i < rep * HD; i += kClThreads) {
        const int r = i / HD, d = i - r * HD;
        float o = 0.f;
        if (mrow[r] != -INFINITY)
            for (int w = 0; w < nwu; ++w) o = fmaf(wt[r * 8 + w], wp[(w * rep + r) * (HD + 2) + 2 + d], o);
        om[i] = o;
    }
    // Merge at rank 0, as in attn_cluster_kernel.
    const int slot = rep * (HD + 2);
    float *mg = A.merge_own ? fb + Ly.mg : reinterpret_cast<float *>(smem);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (!A.merge_own)
        cluster.sync();
    else
        __syncthreads();
    {
        float *dst = cluster.map_shared_rank(mg, 0) + (size_t)s * slot;
        for (int i = tid; i < slot; i += kClThreads) {
            const int r = i / (HD + 2), j = i - r * (HD + 2);
            dst[i] = j == 0 ? mrow[r] : (j == 1 ? lrow[r] : om[r * HD + j - 2]);
        }
    }
    cluster.sync();  // every split's (m, l, o) is in rank 0's merge area
    if (s != 0) return;
    for (int r = warp; r < rep; r += NWARP) {
        const float mj = lane < ns ? mg[lane * slot + r * (HD + 2)] : -INFINITY;
        const float lj = lane < ns ? mg[lane * slot + r * (HD + 2) + 1] : 0.f;
        float M = mj;
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = lane < ns ? expf(__fsub_rn(mj, M)) : 0.f;
        float L = w * lj;
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float inv = __fdiv_rn(1.0f, L);
        if (lane < ns) wt[r * 16 + lane] = __fmul_rn(w, inv);
    }
    __syncthreads();
    for (int i = tid; i < rep * HD; i += kClThreads) {
        const int r = i / HD, d = i - r * HD;
        const float *src = mg + r * (HD + 2) + 2 + d;
        float o = 0.f;
        for (int j = 0; j < ns; ++j) o = fmaf(wt[r * 16 + j], src[(size_t)j * slot], o);
        const int h = kh * rep + r;
        if (A.gated) {
            const float gg = A.q[(size_t)h * A.qstride + HD + d];
            o = __fmul_rn(o, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gg))));
        }
        A.out[(size_t)h * HD + d] = o;
        if (A.tp.world) tp_push_all(A.tp, (size_t)h * HD + d, o);  // the ranks' copies (tensor-parallel gather)
    }
    tp_signal(A.tp, gridDim.y);  // the rank-0 CTAs of the clusters arrive
}

// Launch a cluster attention kernel: one cluster of nsplit CTAs per kv head.
template <typename K>
cudaError_t launch_cluster(K k, DevBits &configured, const AttnArgs &A, uint32_t *err, size_t smem,
                           cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e0 = once_per_device(configured, [&] {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    });
    if (e0 != cudaSuccess) return e0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(A.nsplit, A.Hkv);
    cfg.blockDim = dim3(kClThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = A.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // A cluster this wide must fit on one GPC at this shared-memory size (asked once per shape).
    static struct {
        const void *k;
        int dev, ns;
        size_t smem;
        int ok;
    } seen[64];
    static int nseen = 0;
    static std::mutex seen_mu;
    int ok = -1;
    {
        std::lock_guard<std::mutex> lock(seen_mu);
        for (int i = 0; i < nseen; ++i)
            if (seen[i].k == (const void *)k && seen[i].dev == dev && seen[i].ns == A.nsplit && seen[i].smem == smem)
                ok = seen[i].ok;
    }
    if (ok < 0) {
        int nc = 0;
        ok = cudaOccupancyMaxActiveClusters(&nc, k, &cfg) == cudaSuccess && nc > 0 ? 1 : 0;
        cudaGetLastError();
        std::lock_guard<std::mutex> lock(seen_mu);
        if (nseen < 64) seen[nseen++] = {(const void *)k, dev, A.nsplit, smem, ok};
    }
    if (!ok) return cudaErrorNotSupported;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k, A, err);
}

template <int REP, int DPL>
cudaError_t launch_cl(const AttnArgs &A, uint32_t *err, size_t smem, cudaStream_t st) {
    static DevBits configured{0};
    return launch_cluster(attn_cluster_kernel<REP, DPL>, configured, A, err, smem, st);
}

template <int HD>
cudaError_t launch_mma(const AttnArgs &A, uint32_t *err, size_t smem, cudaStream_t st) {
    static DevBits configured{0};
    return launch_cluster(attn_mma_kernel<HD>, configured, A, err, smem, st);
}

// The tensor-core plan: the cluster chunking, head dim 64 or 128, at most 8 query heads per kv
// head.
bool mma_plan(const AttnArgs &A, int &chunk, int &nsplit, size_t &smem, int &merge_own) {
    const int rep = A.H / A.Hkv;
    if (rep < 1 || rep > 8 || !(A.hd == 64 || A.hd == 128)) return false;
    chunk = ((A.max_pos + 15) / 16 + 31) / 32 * 32;
    nsplit = (A.max_pos + chunk - 1) / chunk;
    if (nsplit > 16) return false;
    const size_t own = mma_smem_bytes(A.hd, rep, chunk, nsplit), tiles_only = mma_smem_bytes(A.hd, rep, chunk, 0);
    merge_own = own <= 113 * 1024 ? 1 : 0;
    smem = merge_own ? own : tiles_only;
    if (!merge_own && (size_t)chunk * (2 * A.hd + 16) * 2 < (size_t)nsplit * rep * (A.hd + 2) * 4) return false;
    return smem <= 227 * 1024;
}

// The cluster plan: chunk a multiple of 32 with at most 16 splits, in shared memory.  false: the
// shape takes the scratch-merge kernel.
bool cl_plan(const AttnArgs &A, int &chunk, int &nsplit, size_t &smem, int &merge_own) {
    const int rep = A.H / A.Hkv;
    if (!(rep == 1 || rep == 2 || rep == 4 || rep == 6 || rep == 8)) return false;
    if (!(A.hd == 64 || A.hd == 128 || A.hd == 256)) return false;
    chunk = ((A.max_pos + 15) / 16 + 31) / 32 * 32;
    nsplit = (A.max_pos + chunk - 1) / chunk;
    if (nsplit > 16) return false;
    // The merge area in its own region when two CTAs still fit an SM with it, else in rank 0's
    // K/V tiles (which must then hold it).
    const size_t own = cl_smem_bytes(A.hd, rep, chunk, nsplit), tiles_only = cl_smem_bytes(A.hd, rep, chunk, 0);
    merge_own = own <= 113 * 1024 ? 1 : 0;
    smem = merge_own ? own : tiles_only;
    if (!merge_own && (size_t)chunk * (2 * A.hd + 8) * 2 < (size_t)nsplit * rep * (A.hd + 2) * 4) return false;
    return smem <= 227 * 1024;
}

}  // namespace

// Positions per CTA: the smallest of 64, 128, 256 that keeps the splits per kv head at 16 or fewer
// (fewer partials to merge), capped so two staged tiles of esize-byte cache elements fit in shared
// memory.
int attn_chunk(int max_pos, int hd, int esize) {
    const int cap = (hd <= 128 ? 256 : 128) / (esize / 2);
    int chunk = 64;
    while (chunk < cap && (max_pos + chunk - 1) / chunk > 16) chunk *= 2;
    return chunk;
}

size_t attn_smem_bytes(int hd, int rep, int chunk, int esize) {
    return (size_t)2 * chunk * (hd + 16 / esize) * esize +
           ((size_t)rep * hd + hd + (size_t)rep * chunk + 2 * rep) * 4;
}

trx_status launch_attn_decode(const AttnArgs &A0, uint32_t *err, cudaStream_t st) {
    if (!A0.scratch_merge) {
        AttnArgs C = A0;
        size_t csmem = 0;
        if (mma_plan(A0, C.chunk, C.nsplit, csmem, C.merge_own)) {
            const cudaError_t e = A0.hd == 64 ? launch_mma<64>(C, err, csmem, st) : launch_mma<128>(C, err, csmem, st);
            if (e != cudaErrorNotSupported) return note_cuda(e);
        }
        // The other kernels exchange their output as tagged words only (no completion counters).
        if (A0.tp.world && !(A0.tp.tag_points && A0.tp.tag_out >= 0)) return TRX_ERR_UNSUPPORTED;
        if (cl_plan(A0, C.chunk, C.nsplit, csmem, C.merge_own)) {
            // 16 dims per lane up to 4 heads, 8 beyond: rep * DPL query values in registers <= 64.
            cudaError_t e;
            switch (A0.H / A0.Hkv) {
                case 1: e = launch_cl<1, 16>(C, err, csmem, st); break;
                case 2: e = launch_cl<2, 16>(C, err, csmem, st); break;
                case 4: e = launch_cl<4, 16>(C, err, csmem, st); break;
                case 6: e = launch_cl<6, 8>(C, err, csmem, st); break;
                default: e = launch_cl<8, 8>(C, err, csmem, st); break;
            }
            if (e != cudaErrorNotSupported) return note_cuda(e);  // not supported: no cluster that wide fits
        }
    }
    const AttnArgs &A = A0;
    const size_t smem = attn_smem_bytes(A.hd, A.H / A.Hkv, A.chunk, A.f32cache ? 4 : 2);
    if (A.f32cache) {
        static DevBits configured{0};
        const cudaError_t e = once_per_device(configured, [] {
            return cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        226 * 1024);
        });
        if (e != cudaSuccess) return note_cuda(e);
        return note_cuda(launch_kernel(attn_decode_kernel<float>, dim3(A.nsplit, A.Hkv, A.nseq > 0 ? A.nseq : 1),
                                       dim3(kAttnThreads), smem, st, A, err));
    }
    static DevBits configured{0};
    const cudaError_t e = once_per_device(configured, [] {
        return cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    226 * 1024);
    });
    if (e != cudaSuccess) return note_cuda(e);
    return note_cuda(launch_kernel(attn_decode_kernel<__half>, dim3(A.nsplit, A.Hkv, A.nseq > 0 ? A.nseq : 1),
                                   dim3(kAttnThreads), smem, st, A, err));
}

}  // namespace trx

// Context-free decode attention ---------------------------------------------------------------
// For callers that cannot allocate device memory while they run: a serving loop that reserved
// all of the device's memory before it started, or a host runtime whose device allocator belongs
// to another framework.  The partials and arrival counts live in this file's static device arrays
// instead of a trx_ctx's scratch; the library allocates nothing.  The arrays are zero when the
// module loads on a device (the counts must start at zero; every launch leaves them at zero
// again).  Their device addresses are looked up on every call (host-side, allocation-free), so a
// context torn down and recreated on the device (cudaDeviceReset) gets the new module's arrays.
// Calls that overlap in time race on the one array per device.
namespace trx {
namespace {

constexpr size_t kStaticPartFloats = size_t(1) << 20;  // 4 MiB: [n_kv][splits][H/n_kv][hd + 2]
constexpr uint32_t kStaticMaxKv = 64;
__device__ __align__(256) float g_static_part[kStaticPartFloats];
__device__ __align__(256) unsigned g_static_cnt[kStaticMaxKv];  // zero at module load and between launches

struct StaticScratch {
    float *part;
    unsigned *cnt;
};

// The static arrays' device addresses in the current device's context (host code cannot use the
// arrays' names as device addresses).
trx_status static_scratch(StaticScratch &out) {
    void *p = nullptr, *c = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_part);
    if (e != cudaSuccess) return note_cuda(e);
    e = cudaGetSymbolAddress(&c, g_static_cnt);
    if (e != cudaSuccess) return note_cuda(e);
    out.part = static_cast<float *>(p);
    out.cnt = static_cast<unsigned *>(c);
    return TRX_OK;
}

}  // namespace
}  // namespace trx

extern "C" trx_status trx_attn_decode_static(const trx_attn_shape *sh, const float *d_q, const float *d_k,
                                             const float *d_v, const float *d_qnorm_w, const float *d_knorm_w,
                                             const float *d_rope_freq, void *d_kcache, void *d_vcache,
                                             const int32_t *d_pos, float *d_out, uint32_t *d_err,
                                             cudaStream_t stream) {
    if (!sh) return TRX_ERR_ARG;
    const uint32_t H = sh->n_head, Hkv = sh->n_kv, hd = sh->head_dim;
    if (H == 0 || Hkv == 0 || H % Hkv || hd == 0 || hd % 8 || hd > 512) return TRX_ERR_ARG;
    if (sh->rope_dims % 2 || sh->rope_dims > hd || sh->max_pos == 0 || sh->max_pos > (1u << 24)) return TRX_ERR_ARG;
    if (!(sh->eps >= 0.f)) return TRX_ERR_ARG;
    if (!d_q || !d_k || !d_v || !d_qnorm_w || !d_knorm_w || !d_kcache || !d_vcache || !d_pos || !d_out || !d_err)
        return TRX_ERR_ARG;
    if ((sh->rope_dims && !d_rope_freq) || (reinterpret_cast<uintptr_t>(d_kcache) & 15) ||
        (reinterpret_cast<uintptr_t>(d_vcache) & 15))
        return TRX_ERR_ARG;
    trx::AttnArgs A{};
    A.H = (int)H;
    A.Hkv = (int)Hkv;
    A.hd = (int)hd;
    A.rope_half = (int)sh->rope_dims / 2;
    A.gated = sh->gated ? 1 : 0;
    A.qstride = (int)hd * (A.gated ? 2 : 1);
    A.max_pos = (int)sh->max_pos;
    A.chunk = trx::attn_chunk((int)sh->max_pos, (int)hd, 2);
    A.nsplit = (A.max_pos + A.chunk - 1) / A.chunk;
    A.eps = sh->eps;
    A.scale = 1.0f / sqrtf((float)hd);
    const uint32_t rep = H / Hkv;
    // The fixed limits of the static scratch: n_kv <= 64 and the partials within 4 MiB.
    if (Hkv > trx::kStaticMaxKv || (uint64_t)Hkv * A.nsplit * rep * (hd + 2) > trx::kStaticPartFloats)
        return TRX_ERR_UNSUPPORTED;
    if (trx::attn_smem_bytes((int)hd, (int)rep, A.chunk, 2) > 226u * 1024u ||
        2ull * rep * A.nsplit > (uint64_t)A.chunk * (hd + 8))
        return TRX_ERR_UNSUPPORTED;
    trx::StaticScratch sc{};
    const trx_status st = trx::static_scratch(sc);
    if (st != TRX_OK) return st;
    A.q = d_q;
    A.k = d_k;
    A.v = d_v;
    A.qn = d_qnorm_w;
    A.kn = d_knorm_w;
    A.freq = d_rope_freq;
    A.pos = d_pos;
    A.kc = static_cast<__half *>(d_kcache);
    A.vc = static_cast<__half *>(d_vcache);
    A.out = d_out;
    A.part = sc.part;
    A.cnt = sc.cnt;
    A.scratch_merge = 1;  // the kernel whose partials and counts are the static arrays above
    return trx::launch_attn_decode(A, d_err, stream);
}
