// Delta-rule gates from the layer's raw projections (delta_gates, model/model.py:314-321), per
// (row, value head), shared by the standalone gates kernel and the kernels that take the raw
// projections instead of g and beta (the chunked prefill's factor work, the recurrent kernel):
//   beta = bf16(sigmoid(b)),  g = log_decay_rate * softplus(a + dt_bias)   (fp32)
// and, with a per-row `valid` flag, beta * valid and g * valid.
//
// Rounding is PyTorch's CUDA eager path: sigmoid as 1 / (1 + expf(-x)) with an IEEE division,
// softplus as x for x > 20 and log1pf(expf(x)) otherwise, subnormals kept (the library is built
// without flush-to-zero).
#pragma once

#include "common.cuh"
#include "launch.h"

namespace gdn {

// beta as the fp32 value of its bf16 rounding, and g, for row `row` and value head h.
__device__ __forceinline__ void delta_gate(const GateInputs& G, int64_t row, int h, float& beta, float& g) {
    const float bv = to_f32(static_cast<const bf16*>(G.b)[row * G.sb + h]);
    const float av = to_f32(static_cast<const bf16*>(G.a)[row * G.sa + h]);
    const float dt = G.dt_f32 ? static_cast<const float*>(G.dt_bias)[h] : to_f32(static_cast<const bf16*>(G.dt_bias)[h]);
    float sig = round_bf16(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-bv))));
    const float x = __fadd_rn(av, dt);
    const float sp = x > 20.0f ? x : log1pf(expf(x));
    float lg = __fmul_rn(G.rate[h], sp);
    if (G.valid) {
        const float kept = G.valid[row] ? 1.0f : 0.0f;
        sig = round_bf16(__fmul_rn(sig, kept));
        lg = __fmul_rn(lg, kept);
    }
    beta = sig;
    g = lg;
}

}  // namespace gdn
