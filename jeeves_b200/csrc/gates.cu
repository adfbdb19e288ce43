// Delta-rule gates from the layer's raw projections (delta_gates, model/model.py:314-321):
//   beta = bf16(sigmoid(b)),  g = log_decay_rate * softplus(a + dt_bias)   (fp32)
// and, with a per-row `valid` flag, beta * valid and g * valid.
//
// Rounding is PyTorch's CUDA eager path: sigmoid as 1 / (1 + expf(-x)) with an IEEE division,
// softplus as x for x > 20 and log1pf(expf(x)) otherwise, subnormals kept (the library is built
// without flush-to-zero). One thread per (row, head).

#include "common.cuh"
#include "launch.h"

namespace gdn {

template <bool DT_F32, bool HAS_VALID>
__global__ void delta_gates_kernel(const bf16* __restrict__ b, int64_t sb, const bf16* __restrict__ a, int64_t sa,
                                   const void* __restrict__ dt_bias, const float* __restrict__ rate,
                                   const uint8_t* __restrict__ valid, bf16* __restrict__ beta, float* __restrict__ g,
                                   int64_t rows, int HV) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * HV) return;
    const int64_t row = idx / HV;
    const int h = (int)(idx % HV);
    const float bv = to_f32(b[row * sb + h]);
    const float av = to_f32(a[row * sa + h]);
    const float dt = DT_F32 ? static_cast<const float*>(dt_bias)[h] : to_f32(static_cast<const bf16*>(dt_bias)[h]);
    float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-bv)));
    const float x = __fadd_rn(av, dt);
    const float sp = x > 20.0f ? x : log1pf(expf(x));
    float lg = __fmul_rn(rate[h], sp);
    if (HAS_VALID) {
        const float kept = valid[row] ? 1.0f : 0.0f;
        sig = __fmul_rn(round_bf16(sig), kept);
        lg = __fmul_rn(lg, kept);
    }
    beta[idx] = __float2bfloat16_rn(sig);
    g[idx] = lg;
}

int launch_delta_gates(const void* b, int64_t sb, const void* a, int64_t sa, const void* dt_bias, int dt_f32,
                       const float* rate, const uint8_t* valid, void* beta, float* g, int64_t rows, int HV,
                       cudaStream_t s) {
    if (rows == 0) return GDN_OK;
    constexpr int threads = 256;
    const int64_t blocks = (rows * HV + threads - 1) / threads;
    auto bp = static_cast<const bf16*>(b);
    auto ap = static_cast<const bf16*>(a);
    auto out = static_cast<bf16*>(beta);
#define GDN_GATES(F32, VALID) \
    delta_gates_kernel<F32, VALID><<<(unsigned)blocks, threads, 0, s>>>(bp, sb, ap, sa, dt_bias, rate, valid, out, g, rows, HV)
    if (dt_f32) {
        if (valid) GDN_GATES(true, true);
        else GDN_GATES(true, false);
    } else {
        if (valid) GDN_GATES(false, true);
        else GDN_GATES(false, false);
    }
#undef GDN_GATES
    return launch_status();
}

}  // namespace gdn
