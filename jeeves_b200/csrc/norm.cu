// Output-gated RMSNorm (GatedRMSNorm.forward, model/model.py:150-158).
//
// Sixteen lanes per row of 128: lane l of the half-warp holds elements 8l..8l+7 (16-byte
// accesses). Rounding follows the eager path on bf16: normed = bf16(x * rsqrt(mean(x^2) + eps)),
// weighted = bf16(w * normed), y = bf16(weighted * silu(z)) with silu in fp32.

#include "common.cuh"
#include "launch.h"

namespace gdn {

__device__ __forceinline__ void load8f(const bf16* p, float (&v)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

// x and y may alias (the fused decode layer normalises in place): every lane reads its eight
// elements before the reduction and writes them after it. A half-warp past the last row reads
// row 0 and stores nothing, so that every lane takes part in the shuffles.
__global__ void gated_rmsnorm_kernel(const bf16* x, const bf16* __restrict__ z, const bf16* __restrict__ w, bf16* y,
                                     int64_t rows, float eps) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    const bool valid = row < rows;
    const int sub = threadIdx.x & 15;
    const int64_t off = (valid ? row : 0) * kHeadDim + 8 * sub;
    float xs[8], zs[8], ws[8], sil[8];
    load8f(x + off, xs);
    load8f(z + off, zs);
    load8f(w + 8 * sub, ws);
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sq = fmaf(xs[i], xs[i], sq);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float inv = inv_sqrt_rn(sq * (1.0f / kHeadDim) + eps);
    silu8(zs, sil);
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float o2[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int e = 2 * i + k;
            const float normed = round_bf16(xs[e] * inv);
            const float weighted = round_bf16(ws[e] * normed);
            o2[k] = weighted * sil[e];
        }
        h[i] = __floats2bfloat162_rn(o2[0], o2[1]);
    }
    if (valid) *reinterpret_cast<uint4*>(y + off) = raw;
}

int launch_gated_rmsnorm(const void* x, const void* z, const void* w, void* y, int64_t rows, int dim, float eps,
                         cudaStream_t s) {
    if (rows == 0) return GDN_OK;
    if (dim != kHeadDim) return GDN_ERR_UNSUPPORTED;
    constexpr int threads = 256;
    const int64_t per_block = threads / 16;
    const int64_t blocks = (rows + per_block - 1) / per_block;
    gated_rmsnorm_kernel<<<(unsigned)blocks, threads, 0, s>>>(static_cast<const bf16*>(x), static_cast<const bf16*>(z),
                                                              static_cast<const bf16*>(w), static_cast<bf16*>(y), rows,
                                                              eps);
    return launch_status();
}

}  // namespace gdn
