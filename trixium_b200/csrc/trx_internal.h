// Internal launch interface between the C ABI (trx_capi.cu) and the kernels.
#pragma once
#include <atomic>
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/trixium_b200.h"

namespace trx {

// Whether launches carry the programmatic-stream-serialization attribute (always: every kernel of
// the library waits for its predecessor with griddepcontrol.wait before reading its inputs).
bool pdl_enabled();

// Launch `k` on `st`, as a programmatic dependent of the stream's previous kernel when enabled.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// Host set-up that a kernel needs once per device (its function attributes): bit d of `done` is
// set once it has run on device d.  Several host threads may launch at once, so the bit is set
// with an atomic OR (two threads may both run the set-up, which is idempotent).  A context torn
// down and recreated on a device (cudaDeviceReset) forgets the attributes while the bit stays set;
// such a program must not reuse the library's launches after the reset.
using DevBits = std::atomic<unsigned long long>;
template <typename F>
inline cudaError_t once_per_device(DevBits &done, F &&setup) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = setup();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

enum { OUT_I32 = 0, OUT_F32 = 1, OUT_SWIGLU = 2 };

// Tensor-parallel exchange of one launch over peer memory (trx_tp_xfer of the C ABI).  A producer
// stores its results into every rank's destination too and, once all its CTAs are done, adds 1 to
// every rank's counter of the gather point; a consumer waits (bounded) until its own counter holds
// (step + 1) * world arrivals before it reads its input.
constexpr int kTpMax = 8;
struct TpXfer {
    int world, rank;
    void *dst[kTpMax];          // each rank's destination base (nullptr: no copy to that rank)
    int offset;                 // elements: this rank's first element in every destination
    unsigned *signal[kTpMax];   // each rank's counter of the completed gather point (signal[0] null: none)
    const unsigned *wait;       // this rank's counter to wait on before reading the input (nullptr: none)
    const int *step;            // this rank's step counter
    unsigned *arrive;           // this launch's arrival count, zero between launches
    // Tagged words (tag_points > 0): an element is one 64-bit word, value bits | tag << 32, stored
    // in one single-copy-atomic access, so a reader that sees the tag sees the value (no fence, no
    // counter).  The tag of gather point p at step s is s * tag_points + p + 1.
    unsigned tag_points;        // gather points per step (0: no tagged words)
    int tag_out;                // the point this launch's output fills in every rank's dst, or -1
    int tag_in;                 // the point of the tagged input this launch reads, or -1
};

constexpr int kMaxSegs = 4;

// A row segment of a launch: rows [previous row_end, row_end) belong to one tensor with its
// own fixed point (B, R) and output.  Several tensors that read the same activation (q, k, v)
// are packed back to back and run as one launch.
struct MvSeg {
    int row_end;
    int B, R;
    void *y;               // output of this segment (row index relative to the segment)
    const float *resid;    // residual added to the float result, or nullptr
};

// One matvec launch: njobs copies of the same tensor geometry, strided (a single job has
// njobs = 1).  w2/B2/R2: the second tensor of a SwiGLU pair (same geometry, one segment).
struct MvJobs {
    const uint8_t *w;
    const uint8_t *w2;
    const float *x;        // fp32 input, or nullptr when x8 is given
    const int8_t *x8;      // pre-quantised input (OUT_I32 from trx_matvec_i8)
    const float *norm_w;   // RMSNorm weight or nullptr
    uint64_t w_stride;     // bytes between jobs' tensors
    uint64_t x_stride;     // elements between jobs' inputs
    uint64_t y_stride;     // elements between jobs' outputs
    int rows, cols, kind;
    int B2, R2;
    int out;
    int njobs;
    float eps;
    int nseg;
    MvSeg seg[kMaxSegs];
    unsigned long long *argmax;  // if set: greedy argmax key of the float results (see below)
    int *token;                  // if set (with argmax): per job, the argmax row; the keys and
    unsigned *arg_cnt;           // the arrival count arg_cnt are left at zero again
    unsigned long long *key_out; // if set (with argmax): per job, the argmax key itself (row + row_offset)
    int row_offset;              // added to the row in the argmax key (a shard's first global row)
    const int *skip;             // if set and *skip != 0, the launch does nothing
    TpXfer tp;                   // tensor-parallel exchange (tp.world == 0: none)
    // A K-segment of a wider input (one job, the staged prologue only): x holds x_cols elements,
    // the quantiser's exponent covers all of them, and this tensor's columns are x[x_off, x_off +
    // cols).  x_cols == 0: x is the tensor's own input.
    int x_cols, x_off;
    const int *part_in;          // OUT_F32: per row, the int32 sum of the earlier K-segments, added
                                 // before the float scaling (nullptr: none)
};

// Argmax key of (value, row): orderable float bits in the high word, ~row in the low word, so
// an unsigned max picks the largest value and, on ties, the smallest row (doc/units.md:149).
__host__ __device__ inline unsigned long long argmax_key(float v, uint32_t row) {
    uint32_t b;
    memcpy(&b, &v, 4);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xffffffffu - row);
}

// One decode-attention launch (trx_attn.cu).
struct AttnArgs {
    const float *q, *k, *v, *qn, *kn, *freq;
    const int *pos;
    __half *kc, *vc;
    float *out;
    float *part;        // scratch partials: [Hkv][nsplit][H/Hkv][hd + 2]
    unsigned *cnt;      // [Hkv] arrival counts, zero between launches
    int H, Hkv, hd, rope_half, qstride, gated, max_pos, chunk, nsplit;
    int merge_own;      // cluster kernel: the merge area has its own shared region
    int scratch_merge;  // run the scratch-merge kernel on part/cnt even where a cluster kernel applies
    int f32cache;       // kc/vc hold fp32 elements (the scratch-merge kernel only)
    // Independent sequences (the scratch-merge kernel: blockIdx.z = sequence; 0 for one): elements
    // between sequences of q, k/v, the caches, the output and the partials; pos and the arrival
    // counts are per sequence (pos + z, cnt + z * Hkv).
    long long q_bs, kv_bs, cache_bs, out_bs, part_bs;
    int nseq;
    TpXfer tp;          // tensor-parallel exchange of the output (tp.world == 0: none)
    float eps, scale;
};

trx_status launch_attn_decode(const AttnArgs &A, uint32_t *err, cudaStream_t st);

// One gated-DeltaNet step launch (trx_deltanet.cu).
struct DnArgs {
    const float *qkv, *z, *beta, *alpha, *dt_bias, *ssm_a, *conv_w, *norm_w;
    const int *pos;
    float *win;         // conv input ring [K][C]
    float *S;           // state [nv][hv][hk]
    float *out;         // [nv*hv], grouped head order
    float *part;        // scratch [nv][hv]
    unsigned *cnt;      // [nv] arrival counts, zero between launches
    int nk, hk, nv, hv, K, C, rows, nsplit;
    float eps, scale;
    int nseq;           // independent sequences (blockIdx.z; 0 or 1: one), each with its own
                        // inputs, ring, state, position, output, partials and counts
    TpXfer tp;          // tensor-parallel exchange of the output (tp.world == 0: none; one sequence)
};

trx_status launch_deltanet(const DnArgs &A, uint32_t *err, cudaStream_t st);

// The integer DeltaNet head step (trx_dn_int.cu, model/deltanet.py:99-147): nh heads, each an int16
// state hv x hk at exponent eM[h] with maxM[h] (< 0: computed from the state), fp32 k, q [nh][hk],
// v [nh][hv], decay and beta [nh]; M, eM, maxM updated in place, out [nh][hv].
struct DnIntArgs {
    int nh, hv, hk;
    int16_t *M;
    int *eM, *maxM;
    const float *k, *q, *v, *decay, *beta;
    float *out;
};
trx_status launch_dn_int(const DnIntArgs &A, uint32_t *err, cudaStream_t st);
size_t attn_smem_bytes(int hd, int rep, int chunk, int esize);
int attn_chunk(int max_pos, int hd, int esize);

trx_status launch_embed(const void *table, int vocab, int dim, int f16, const int *token, float *x, uint32_t *err,
                        cudaStream_t st);
trx_status launch_advance(int *pos, int n, cudaStream_t st);
trx_status launch_embed_rows(const void *table, int vocab, int dim, int f16, const int *tokens, int nrows, float *x,
                             uint32_t *err, cudaStream_t st);
trx_status launch_rmsnorm_rows(const float *x, const float *w, int n, int nrows, float eps, float *y, cudaStream_t st);
trx_status launch_silu_mul(const float *g, const float *u, long long n, float *act, cudaStream_t st);
trx_status launch_argmax_rows(const float *logits, int V, int nrows, int *tokens, cudaStream_t st);
trx_status launch_advance_rows(int *pos, int count, int n, cudaStream_t st);
trx_status launch_embed_bfp16(const int16_t *mant, const int *exps, int vocab, int dim, const int *token, float *x,
                              uint32_t *err, cudaStream_t st);
trx_status launch_rmsnorm(const float *x, const float *w, int n, float eps, float *y, cudaStream_t st);
trx_status launch_kseg_combine(const int *parts, int nseg, int rows, const int *e8, int R, int B, const float *resid,
                               float *y, cudaStream_t st, const TpXfer *tp = nullptr);
trx_status launch_argmax_keys(const unsigned long long *keys, int n, int *token, const TpXfer &tp, uint32_t *err,
                              cudaStream_t st);

trx_status launch_matvec(const MvJobs &J, const uint32_t *lut, uint32_t *err, cudaStream_t st);
// Batched rows on the tensor cores (trx_rows.cu): nb <= 32 rows of x (fp32, each quantised with its
// own exponent, optionally RMS-normalised first with norm_w) or x8 (int8), against nseg <= 4 tensors
// of the same cols and kind packed back to back (segment s: rows, its B and R, int32 or fp32 output
// [nb][rows], an optional fp32 residual [nb][rows]).  x8p/xsum/e8: scratch of nb*K bytes, K/128*32
// ints and nb ints; acc_scratch (acc_cap int64) and cnt (cnt_cap per-row counts) zero between
// launches.
struct RowsSeg {
    int rows, B, R;
    int32_t *out_i;
    float *out_f;
    const float *resid;
    const int32_t *part_in;  // [nb][rows] int32 sum of the earlier K-segments, added before the scaling
};
constexpr int kRowsMaxSegs = 4;
trx_status launch_matvec_rows(const uint8_t *w, int K, int kind, const RowsSeg *segs, int nseg, const float *x,
                              const int8_t *x8, int nb, const float *norm_w, float eps, int8_t *x8p, int *xsum,
                              int *e8, unsigned long long *acc_scratch, size_t acc_cap, unsigned *cnt, int cnt_cap,
                              uint32_t *err, int sms, int reserved, cudaStream_t st, int K_full = 0, int k_off = 0,
                              bool prep = true);
// K_full (0: K): the width of x (and of x8p, xsum); the tensor's columns are [k_off, k_off + K) of
// it.  prep: quantise x into x8p/xsum/e8 first (false: they already hold it, from a launch over
// another K-segment of the same x).
int device_sms();
int device_reserved_smem();
// The Q8 row dot (trx_q8.cu): int32 results, or with e8 the float projection (fp32 out).
trx_status launch_matvec_q8(const uint8_t *w, int rows, int cols, int B, int R, const int8_t *x8, const int *e8,
                            void *out, uint32_t *err, cudaStream_t st);
trx_status launch_matvec_fp(const MvJobs &J, uint32_t *err, cudaStream_t st);
trx_status launch_quantize(const float *x, int n, int8_t *x8, int *e8, cudaStream_t st);
// launch_matvec would accept J (its plan exists and its input path applies); launches nothing.
bool matvec_launchable(const MvJobs &J);
// The same over a tagged input (x: tagged words of tp.tag_in, polled, bounded).
trx_status launch_quantize_tagged(const void *x, int n, int8_t *x8, int *e8, const TpXfer &tp, uint32_t *err,
                                  cudaStream_t st);
trx_status launch_validate_t5(const uint8_t *w, int rows, int cols, uint32_t *err, cudaStream_t st);
trx_status launch_build_lut(uint32_t *lut, cudaStream_t st);
size_t lut_bytes();
trx_status note_cuda(cudaError_t e);   // TRX_OK, or TRX_ERR_CUDA after recording e
const char *last_cuda_error();

}  // namespace trx
