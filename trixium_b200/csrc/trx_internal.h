// Internal launch interface between the C ABI (trx_capi.cu) and the kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/trixium_b200.h"

namespace trx {

enum { OUT_I32 = 0, OUT_F32 = 1, OUT_SWIGLU = 2 };

// One matvec launch: njobs copies of the same tensor geometry, strided (a single job has
// njobs = 1).  w2/B2/R2: the second tensor of a SwiGLU pair (same geometry).
struct MvJobs {
    const uint8_t *w;
    const uint8_t *w2;
    const float *x;        // fp32 input, or nullptr when x8 is given
    const int8_t *x8;      // pre-quantised input (OUT_I32 from trx_matvec_i8)
    const float *norm_w;   // RMSNorm weight or nullptr
    const float *resid;    // residual added to the float result, or nullptr
    void *y;
    uint64_t w_stride;     // bytes between jobs' tensors
    uint64_t x_stride;     // elements between jobs' inputs
    uint64_t y_stride;     // elements between jobs' outputs
    int rows, cols, kind;
    int B, R, B2, R2;
    int out;
    int njobs;
    float eps;
};

trx_status launch_matvec(const MvJobs &J, const uint32_t *lut, uint32_t *err, cudaStream_t st);
trx_status launch_matvec_fp(const MvJobs &J, uint32_t *err, cudaStream_t st);
trx_status launch_quantize(const float *x, int n, int8_t *x8, int *e8, cudaStream_t st);
trx_status launch_validate_t5(const uint8_t *w, int rows, int cols, uint32_t *err, cudaStream_t st);
trx_status launch_build_lut(uint32_t *lut, cudaStream_t st);
size_t lut_bytes();

}  // namespace trx
