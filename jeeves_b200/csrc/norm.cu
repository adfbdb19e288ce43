// Output-gated RMSNorm (GatedRMSNorm.forward, model/model.py:150-158): one half-warp per row of
// 128, the row arithmetic in norm.cuh.

#include "launch.h"
#include "norm.cuh"

namespace gdn {

// x and y may alias (the fused decode layer normalises in place): every lane reads its rows'
// elements before the reductions and writes them after. Half-warp h of the grid normalises rows
// h, h + H, ..., h + (R - 1) H (H half-warps in the grid), all R rows' loads in flight before the
// first reduction. A row past the last reads row 0 and stores nothing, so that every lane takes
// part in the shuffles.
template <int R>
__global__ void gated_rmsnorm_kernel(const bf16* x, const bf16* __restrict__ z, const bf16* __restrict__ w, bf16* y,
                                     int64_t rows, float eps) {
    const int64_t hw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    const int64_t nhw = ((int64_t)gridDim.x * blockDim.x) >> 4;
    const int sub = threadIdx.x & 15;
    int64_t off[R];
    uint4 zr[R], xr[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
        const int64_t row = hw + k * nhw;
        off[k] = (row < rows ? row : 0) * kHeadDim + 8 * sub;
        zr[k] = *reinterpret_cast<const uint4*>(z + off[k]);
    }
    float ws[8];
    load8f(w + 8 * sub, ws);
    pdl_launch_dependents();  // the next layer's conv, a dependent that waits for this kernel, may launch
    pdl_wait();  // x comes from the previous kernel when launched as its dependent
#pragma unroll
    for (int k = 0; k < R; ++k) xr[k] = *reinterpret_cast<const uint4*>(x + off[k]);
    // Row sums of squares, reduced over the half-warp; then each lane computes the inverse of one
    // row (lane l of a half-warp the row l % R) and the R inverses come back by shuffles.
    float sq[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
        float xs[8];
        unpack8f(xr[k], xs);
        sq[k] = sum_squares8(xs);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
        for (int k = 0; k < R; ++k) sq[k] = __fadd_rn(sq[k], __shfl_xor_sync(0xffffffffu, sq[k], o));
    float mine = sq[0];
#pragma unroll
    for (int k = 1; k < R; ++k) mine = (sub % R) == k ? sq[k] : mine;
    const float inv_mine = gated_norm_inv(mine, eps);
#pragma unroll
    for (int k = 0; k < R; ++k) {
        const float inv = R == 1 ? inv_mine : __shfl_sync(0xffffffffu, inv_mine, (threadIdx.x & 16) | k);
        float xs[8], zs[8];
        unpack8f(xr[k], xs);
        unpack8f(zr[k], zs);
        const uint4 raw = gated_norm_apply8(xs, zs, ws, inv);
        if (hw + k * nhw < rows) *reinterpret_cast<uint4*>(y + off[k]) = raw;
    }
}

int launch_gated_rmsnorm(const void* x, const void* z, const void* w, void* y, int64_t rows, int dim, float eps,
                         cudaStream_t s, bool dependent) {
    if (rows == 0) return GDN_OK;
    if (dim != kHeadDim) return GDN_ERR_UNSUPPORTED;
    constexpr int threads = 256;
    // Two rows a half-warp once the grid still fills the SMs many times over (prefill), one
    // for the small row counts of decode.
    const bool two = rows >= 65536;
    const int64_t per_block = (threads / 16) * (two ? 2 : 1);
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
    const bf16* xp = static_cast<const bf16*>(x);
    const bf16* zp = static_cast<const bf16*>(z);
    const bf16* wp = static_cast<const bf16*>(w);
    bf16* yp = static_cast<bf16*>(y);
    const cudaError_t e = two ? cudaLaunchKernelEx(&cfg, gated_rmsnorm_kernel<2>, xp, zp, wp, yp, rows, eps)
                               : cudaLaunchKernelEx(&cfg, gated_rmsnorm_kernel<1>, xp, zp, wp, yp, rows, eps);
    return e == cudaSuccess ? launch_status() : GDN_ERR_LAUNCH;
}

}  // namespace gdn
