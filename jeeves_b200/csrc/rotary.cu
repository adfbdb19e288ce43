// Rotary embedding with per-row positions and the drafter's cache writes (CUDA cores).
//
// apply_rotary (model/model.py:182-196) on bf16 with 3-D cos / sin ([B, T, F] fp32, F rotary
// frequencies, 2F <= D): over the first 2F elements of each head,
//   y[d] = bf16( bf16(x[d] * c) + bf16(t[d] * s) ),  c = bf16(cos[f]), s = bf16(sin[f]),
//   f = d mod F, t[d] = -x[d + F] for d < F and x[d - F] otherwise (rotate_half),
// which is the eager path's rounding on bf16 (every product and the sum rounded to bf16, as
// model/triton_kernels.py:36-51 also does); the other elements are copied. One thread per element.
//
// rotate_into_cache (model/model.py:342-351; model/triton_kernels.py:214-262): the K candidate
// rows' keys, rotated, and values go to k_cache / v_cache at (rows[b, t], positions[b, t]); the M
// mask rows' queries are rotated into q_out, and their keys (rotated) and values go to cache row b
// at positions tail_start + m.

#include "common.cuh"
#include "launch.h"

namespace gdn {

__device__ __forceinline__ bf16 rotated_element(const bf16* __restrict__ x, const float* __restrict__ cs,
                                                const float* __restrict__ sn, int d, int nf) {
    const float value = to_f32(x[d]);
    if (d >= 2 * nf) return x[d];
    const bool lower = d < nf;
    const int f = lower ? d : d - nf;
    const float partner = to_f32(x[lower ? d + nf : d - nf]);
    const float c = round_bf16(cs[f]), s = round_bf16(sn[f]);
    const float turned = lower ? -partner : partner;
    return __float2bfloat16_rn(round_bf16(value * c) + round_bf16(turned * s));
}

// x, out: [B, T, H, D] contiguous; cos, sin: [B, T, F] fp32 contiguous. Block: D threads, one
// (b, t, h) row per block.
__global__ void rotary_kernel(const bf16* __restrict__ x, const float* __restrict__ cs, const float* __restrict__ sn,
                              bf16* __restrict__ out, int H, int D, int nf) {
    const int64_t row = blockIdx.x;
    const int d = threadIdx.x;
    const int64_t bt = row / H;
    out[row * D + d] = rotated_element(x + row * D, cs + bt * nf, sn + bt * nf, d, nf);
}

__global__ void rotate_into_cache_kernel(RotateCacheArgs a) {
    const int64_t prog = blockIdx.x;
    const int d = threadIdx.x;
    const int h = (int)(prog % a.H);
    const int t = (int)((prog / a.H) % (a.K + a.M));
    const int64_t b = prog / ((int64_t)a.H * (a.K + a.M));
    const bf16* kin = static_cast<const bf16*>(a.k);
    const bf16* vin = static_cast<const bf16*>(a.v);
    bf16* kc = static_cast<bf16*>(a.k_cache);
    bf16* vc = static_cast<bf16*>(a.v_cache);
    if (t < a.K) {
        const int64_t x_off = ((b * a.K + t) * a.H + h) * a.D;
        const int64_t crow = a.rows[b * a.rsb + t * a.rst];
        const int64_t pos = a.positions[b * a.K + t];
        const int64_t c_off = crow * a.csb + pos * a.css + (int64_t)h * a.D;
        const int64_t f_off = (b * a.K + t) * a.nf;
        kc[c_off + d] = rotated_element(kin + x_off, a.cos_c + f_off, a.sin_c + f_off, d, a.nf);
        vc[c_off + d] = vin[x_off + d];
    } else {
        const int m = t - a.K;
        const int64_t x_off = b * a.msb + m * a.mst + (int64_t)h * a.D;
        const int64_t f_off = (b * a.M + m) * a.nf;
        bf16* qo = static_cast<bf16*>(a.q_out);
        qo[((b * a.M + m) * a.H + h) * a.D + d] =
            rotated_element(static_cast<const bf16*>(a.qm) + x_off, a.cos_m + f_off, a.sin_m + f_off, d, a.nf);
        const int64_t c_off = b * a.csb + (a.tail_start + m) * a.css + (int64_t)h * a.D;
        kc[c_off + d] = rotated_element(static_cast<const bf16*>(a.km) + x_off, a.cos_m + f_off, a.sin_m + f_off, d, a.nf);
        vc[c_off + d] = static_cast<const bf16*>(a.vm)[x_off + d];
    }
}

int launch_rotary(const void* x, const float* cs, const float* sn, void* out, int64_t rows, int H, int D, int nf,
                  cudaStream_t s) {
    if (rows == 0) return GDN_OK;
    rotary_kernel<<<(unsigned)rows, D, 0, s>>>(static_cast<const bf16*>(x), cs, sn, static_cast<bf16*>(out), H, D, nf);
    return launch_status();
}

int launch_rotate_into_cache(const RotateCacheArgs& a, cudaStream_t s) {
    const int64_t progs = a.B * (int64_t)(a.K + a.M) * a.H;
    if (progs == 0) return GDN_OK;
    rotate_into_cache_kernel<<<(unsigned)progs, a.D, 0, s>>>(a);
    return launch_status();
}

}  // namespace gdn
