// Output-gated RMSNorm of one row of 128 (GatedRMSNorm.forward, model/model.py:150-158), shared by
// the standalone norm kernel and the chunked prefill's fused norm role, so that both round alike.
//
// Sixteen lanes hold one row: lane l of the half-warp holds elements 8l..8l+7. Rounding follows
// the eager path on bf16: normed = bf16(x * rsqrt(mean(x^2) + eps)), weighted = bf16(w * normed),
// y = bf16(weighted * silu(z)) with silu in fp32.
#pragma once

#include "common.cuh"

namespace gdn {

__device__ __forceinline__ void unpack8f(const uint4& raw, float (&v)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void load8f(const bf16* p, float (&v)[8]) { unpack8f(*reinterpret_cast<const uint4*>(p), v); }

// The normed, gated eight elements x (bf16-valued) of one row, given the row's
// inv = 1 / sqrt(mean(x^2) + eps), packed as bf16.
__device__ __forceinline__ uint4 gated_norm_apply8(const float (&xs)[8], const float (&zs)[8], const float (&ws)[8],
                                                   float inv) {
    float sil[8];
    silu8(zs, sil);
    uint32_t out[4];
    const f32x2 inv2 = pack2(inv, inv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // element pairs (2i, 2i + 1) in packed lanes
        const f32x2 normed = round_bf16x2(mul2(pack2(xs[2 * i], xs[2 * i + 1]), inv2));
        const f32x2 weighted = round_bf16x2(mul2(pack2(ws[2 * i], ws[2 * i + 1]), normed));
        out[i] = f2_to_bf2(mul2(weighted, pack2(sil[2 * i], sil[2 * i + 1])));
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// Sum of squares of the eight elements of one lane, in element order.
__device__ __forceinline__ float sum_squares8(const float (&xs)[8]) {
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sq = __fmaf_rn(xs[i], xs[i], sq);
    return sq;
}

// 1 / sqrt(mean(x^2) + eps) of a row of 128 from its sum of squares (the mean's division by 128
// is exact).
__device__ __forceinline__ float gated_norm_inv(float sq, float eps) { return inv_sqrt_rn(sq * (1.0f / kHeadDim) + eps); }

// The normed, gated eight elements of this lane, packed as bf16. Every lane of the warp must
// call it (the sum of squares is reduced over the half-warp with shuffles: offsets 8, 4, 2, 1).
__device__ __forceinline__ uint4 gated_norm_row8(const float (&xs)[8], const float (&zs)[8], const float (&ws)[8],
                                                 float eps) {
    float sq = sum_squares8(xs);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
    return gated_norm_apply8(xs, zs, ws, gated_norm_inv(sq, eps));
}

}  // namespace gdn
