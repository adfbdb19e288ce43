// Output-gated RMSNorm (GatedRMSNorm.forward, model/model.py:150-158): one half-warp per row of
// 128, the row arithmetic in norm.cuh.

#include "launch.h"
#include "norm.cuh"

namespace gdn {

// x and y may alias (the fused decode layer normalises in place): every lane reads its eight
// elements before the reduction and writes them after it. A half-warp past the last row reads
// row 0 and stores nothing, so that every lane takes part in the shuffles.
__global__ void gated_rmsnorm_kernel(const bf16* x, const bf16* __restrict__ z, const bf16* __restrict__ w, bf16* y,
                                     int64_t rows, float eps) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    const bool valid = row < rows;
    const int sub = threadIdx.x & 15;
    const int64_t off = (valid ? row : 0) * kHeadDim + 8 * sub;
    float xs[8], zs[8], ws[8];
    load8f(z + off, zs);
    load8f(w + 8 * sub, ws);
    pdl_wait();  // x comes from the previous kernel when launched as its dependent
    load8f(x + off, xs);
    const uint4 raw = gated_norm_row8(xs, zs, ws, eps);
    if (valid) *reinterpret_cast<uint4*>(y + off) = raw;
}

int launch_gated_rmsnorm(const void* x, const void* z, const void* w, void* y, int64_t rows, int dim, float eps,
                         cudaStream_t s, bool dependent) {
    if (rows == 0) return GDN_OK;
    if (dim != kHeadDim) return GDN_ERR_UNSUPPORTED;
    constexpr int threads = 256;
    const int64_t per_block = threads / 16;
    const int64_t blocks = (rows + per_block - 1) / per_block;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(threads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gated_rmsnorm_kernel, static_cast<const bf16*>(x),
                                             static_cast<const bf16*>(z), static_cast<const bf16*>(w),
                                             static_cast<bf16*>(y), rows, eps);
    return e == cudaSuccess ? launch_status() : GDN_ERR_LAUNCH;
}

}  // namespace gdn
