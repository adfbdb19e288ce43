// Shared helpers for the sm_100a gated-delta-rule kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"

namespace gdn {

using bf16 = __nv_bfloat16;

constexpr int kHeadDim = 128;

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(bf16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ bf16 from_f32<bf16>(float x) { return __float2bfloat16_rn(x); }

// Round an fp32 value to bf16 and back (round to nearest even, NaN kept).
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Loads 4 consecutive elements as fp32 (8-byte load for bf16, 16-byte load for fp32).
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const bf16* p) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
    float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(bf16* p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 raw;
    raw.x = *reinterpret_cast<uint32_t*>(&a);
    raw.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = raw;
}

__device__ __forceinline__ float4 ldg_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void stg_stream(float4* p, float4 v) { __stcs(p, v); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// x / d rounded to nearest for 1 <= d < 2^120, by Markstein's method (P. Markstein, IA-64 and
// Elementary Functions, 2000, ch. 8): one Newton step refines the hardware reciprocal estimate
// y of 1/d, then one fused residual r = x - d q corrects the quotient q = x y.
__device__ __forceinline__ float div_markstein(float x, float d) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    y = fmaf(y, fmaf(-d, y, 1.0f), y);
    const float q = x * y;
    return fmaf(fmaf(-d, q, x), y, q);
}

// SiLU as the eager path evaluates it on bf16: x / (1 + exp(-x)) in fp32 with an IEEE division,
// computed without a division instruction. 0 < |x| <= 80: Markstein's quotient. The rest, in
// plain arithmetic (no call and no branch, so that the compiler keeps scheduling across
// unrolled elements): zero keeps its sign; x > 80 has d == 1 exactly, so x / d = x; x < -80
// scales d by 2^-64, which keeps the reciprocal estimate normal, and scales the quotient back
// exactly; d = inf (x below about -88.7) gives -0, or NaN for x = -inf; NaN stays NaN. Checked against the
// IEEE division __fdiv_rn on every bf16 x and every fp32 x with |x| <= 80: no difference
// (NaN compared as NaN).
__device__ __forceinline__ float silu_f32(float x) {
    constexpr float kInf = __builtin_huge_valf();
    const float d = 1.0f + expf(-x);
    const float sc = x < -80.f ? 0x1p-64f : 1.0f;  // powers of two: exact scalings
    float q = div_markstein(x, d * sc) * sc;
    q = (x == 0.f || x > 80.f) ? x : q;
    return d == kInf ? (x == -kInf ? __int_as_float(0x7fffffff) : -0.0f) : q;
}

// Two fp32 values in one 64-bit register pair, for sm_100's packed add / sub / mul / fma .rn.f32x2:
// each lane is rounded exactly as the scalar instruction rounds it, so a packed operation gives
// bit for bit the two scalar results at half the issued instructions.
struct f32x2 {
    unsigned long long v;
};
__device__ __forceinline__ f32x2 pack2(float a, float b) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 unpack2(f32x2 x) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(x.v));
    return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
// a * b + c with one rounding per lane
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
    return r;
}
// A bf16 pair (low half first) widened to fp32 lanes.
__device__ __forceinline__ f32x2 bf2_to_f2(uint32_t raw) { return pack2(__uint_as_float(raw << 16), __uint_as_float(raw & 0xffff0000u)); }
// Both lanes rounded to bf16, packed low lane first.
__device__ __forceinline__ uint32_t f2_to_bf2(f32x2 x) {
    const float2 f = unpack2(x);
    const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// Both lanes rounded to bf16 and widened back (round_bf16 of each lane).
__device__ __forceinline__ f32x2 round_bf16x2(f32x2 x) { return bf2_to_f2(f2_to_bf2(x)); }

// div_markstein(x, 1 + exp(-x)) on both lanes: the common-case SiLU quotient of a pair. The
// negated denominator -1 - e equals -(1 + e) exactly (round to nearest is symmetric), so the
// Newton step and the residual are the scalar ones with -d folded into the packed operand.
__device__ __forceinline__ f32x2 silu2_common(f32x2 x) {
    const float2 xs = unpack2(x);
    const f32x2 e = pack2(expf(-xs.x), expf(-xs.y));
    const f32x2 d = add2(pack2(1.0f, 1.0f), e);
    const f32x2 nd = sub2(pack2(-1.0f, -1.0f), e);
    const float2 ds = unpack2(d);
    float ya, yb;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(ya) : "f"(ds.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(yb) : "f"(ds.y));
    f32x2 y = pack2(ya, yb);
    y = fma2(y, fma2(nd, y, pack2(1.0f, 1.0f)), y);
    const f32x2 q = mul2(x, y);
    return fma2(fma2(nd, q, x), y, q);
}

// silu_f32 on 8 values: the common-case quotients first (in pairs); all 8 again with the full
// formula only when one of them is zero, beyond +-80 or NaN (a branch that real activations
// almost never take).
__device__ __forceinline__ void silu8(const float (&x)[8], float (&y)[8]) {
    bool rare = false;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float2 r = unpack2(silu2_common(pack2(x[i], x[i + 1])));
        y[i] = r.x;
        y[i + 1] = r.y;
        rare |= !(fabsf(x[i]) <= 80.f) || x[i] == 0.f || !(fabsf(x[i + 1]) <= 80.f) || x[i + 1] == 0.f;
    }
    if (rare) {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = silu_f32(x[i]);
    }
}

// 1 / sqrt(x) with an IEEE square root and an IEEE division, as the CPU evaluates rsqrt.
__device__ __forceinline__ float inv_sqrt_rn(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

// Programmatic dependent launch (sm_90+): a kernel launched with the programmatic-serialization
// attribute may start while the previous kernel in the stream still runs. pdl_wait() blocks until
// that kernel has finished and its writes are visible (it returns at once for an ordinary
// launch); pdl_launch_dependents() lets the next such kernel start before this one ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Device-side error word written by bounded waits (one per device image of the library;
// the library is built as a single translation unit, library.cu).
__device__ int g_device_error = 0;

__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
