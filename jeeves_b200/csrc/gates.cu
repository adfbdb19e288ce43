// Delta-rule gates from the layer's raw projections (delta_gates, model/model.py:314-321), one
// thread per (row, head); the arithmetic is delta_gate (gates.cuh).

#include "gates.cuh"
#include "launch.h"

namespace gdn {

__global__ void delta_gates_kernel(const GateInputs G, bf16* __restrict__ beta, float* __restrict__ g, int64_t rows,
                                   int HV) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * HV) return;
    float bv, gv;
    delta_gate(G, idx / HV, (int)(idx % HV), bv, gv);
    beta[idx] = __float2bfloat16_rn(bv);
    g[idx] = gv;
}

int launch_delta_gates(const void* b, int64_t sb, const void* a, int64_t sa, const void* dt_bias, int dt_f32,
                       const float* rate, const uint8_t* valid, void* beta, float* g, int64_t rows, int HV,
                       cudaStream_t s) {
    if (rows == 0) return GDN_OK;
    constexpr int threads = 256;
    const int64_t blocks = (rows * HV + threads - 1) / threads;
    GateInputs G{b, sb, a, sa, dt_bias, dt_f32, rate, valid};
    delta_gates_kernel<<<(unsigned)blocks, threads, 0, s>>>(G, static_cast<bf16*>(beta), g, rows, HV);
    return launch_status();
}

}  // namespace gdn
