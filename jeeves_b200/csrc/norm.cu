// Output-gated RMSNorm (GatedRMSNorm.forward, model/model.py:150-158).
//
// One warp per row of 128: lane l holds elements 4l..4l+3. Rounding follows the eager
// path on bf16: normed = bf16(x * rsqrt(mean(x^2) + eps)), weighted = bf16(w * normed),
// y = bf16(weighted * silu(z)) with silu in fp32.

#include "common.cuh"
#include "launch.h"

namespace gdn {

// x and y may alias (the fused decode layer normalises in place): every lane reads its four
// elements before the warp reduction and writes them after it.
__global__ void gated_rmsnorm_kernel(const bf16* x, const bf16* __restrict__ z, const bf16* __restrict__ w, bf16* y,
                                     int64_t rows, float eps) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int lane = threadIdx.x & 31;
    const int64_t off = row * kHeadDim + 4 * lane;
    const float4 xv = load4(x + off);
    const float4 zv = load4(z + off);
    const float4 wv = load4(w + 4 * lane);
    const float sq = warp_sum(xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w);
    const float inv = inv_sqrt_rn(sq * (1.0f / kHeadDim) + eps);
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w}, zs[4] = {zv.x, zv.y, zv.z, zv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
    float4 out;
    float* o = &out.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float normed = round_bf16(xs[i] * inv);
        const float weighted = round_bf16(ws[i] * normed);
        o[i] = weighted * silu_f32(zs[i]);
    }
    store4(y + off, out);
}

int launch_gated_rmsnorm(const void* x, const void* z, const void* w, void* y, int64_t rows, int dim, float eps,
                         cudaStream_t s) {
    if (rows == 0) return GDN_OK;
    if (dim != kHeadDim) return GDN_ERR_UNSUPPORTED;
    constexpr int threads = 256;
    const int64_t per_block = threads / 32;
    const int64_t blocks = (rows + per_block - 1) / per_block;
    gated_rmsnorm_kernel<<<(unsigned)blocks, threads, 0, s>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(z),
                                                              static_cast<const bf16*>(w), static_cast<bf16*>(y), rows,
                                                              eps);
    return launch_status();
}

}  // namespace gdn
