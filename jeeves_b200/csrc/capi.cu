// C ABI: argument checks and dispatch. Declarations and contracts are in include/gdn_b200.h.

#include "common.cuh"
#include "launch.h"

using namespace gdn;

namespace {

constexpr int kAbiVersion = 2;

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

inline int elem_size(int dtype) { return dtype == GDN_BF16 ? 2 : 4; }

inline bool known_dtype(int dtype) { return dtype == GDN_BF16 || dtype == GDN_F32; }

// Vector loads need 16-byte alignment of every row start: base pointer aligned and every
// stride a multiple of 16 bytes (the head dim, 128, always is).
inline bool rows_aligned(const void* p, int esize, int64_t s0, int64_t s1, int64_t s2) {
    return aligned16(p) && (s0 * esize) % 16 == 0 && (s1 * esize) % 16 == 0 && (s2 * esize) % 16 == 0;
}

}  // namespace

extern "C" {

const char* gdn_status_string(int status) {
    switch (status) {
        case GDN_OK: return "ok";
        case GDN_ERR_SHAPE: return "invalid shape, head count or stride";
        case GDN_ERR_DTYPE: return "unsupported element type";
        case GDN_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
        case GDN_ERR_NULL: return "required pointer is NULL";
        case GDN_ERR_LAUNCH: return "CUDA kernel launch failed";
        case GDN_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
        case GDN_ERR_UNSUPPORTED: return "unsupported configuration";
        case GDN_ERR_SCRATCH: return "request larger than the fixed scratch of the no-allocation entry point";
        case GDN_ERR_WORKSPACE: return "workspace missing or smaller than the call's *_workspace_size";
        default: return "unknown status";
    }
}

int gdn_abi_version(void) { return kAbiVersion; }

int gdn_probe_bounded_wait(int64_t limit_cycles, void* stream) {
    if (limit_cycles < 1000 || limit_cycles > 2000000000LL) return GDN_ERR_SHAPE;
    return launch_bounded_wait_probe(limit_cycles, as_stream(stream));
}

int gdn_device_error(void* stream, int reset) {
    int value = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, as_stream(stream)) !=
        cudaSuccess)
        return -1;
    if (cudaStreamSynchronize(as_stream(stream)) != cudaSuccess) return -1;
    if (reset) {
        const int zero = 0;
        if (cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, as_stream(stream)) !=
            cudaSuccess)
            return -1;
        if (cudaStreamSynchronize(as_stream(stream)) != cudaSuccess) return -1;
    }
    return value;
}

// gdn_gate_inputs -> the kernels' GateInputs; status of its checks (null pointers, dtype).
static int gate_args(const gdn_gate_inputs* in, GateInputs* out) {
    if (!in->b || !in->a || !in->dt_bias || !in->log_decay_rate) return GDN_ERR_NULL;
    if (!known_dtype(in->dt_bias_dtype)) return GDN_ERR_DTYPE;
    out->b = in->b;
    out->sb = in->b_row_stride;
    out->a = in->a;
    out->sa = in->a_row_stride;
    out->dt_bias = in->dt_bias;
    out->dt_f32 = in->dt_bias_dtype == GDN_F32;
    out->rate = in->log_decay_rate;
    out->valid = in->valid;
    return GDN_OK;
}

static int recurrent(const void* q, const void* k, const void* v, int qkv_dtype, const float* g, const void* beta,
                     int beta_dtype, const gdn_gate_inputs* gates, const float* state_in, float* state_out,
                     float* snapshots, void* o, const int64_t* steps, const int32_t* cu_seqlens, int64_t batch,
                     int64_t seqlen, int64_t key_heads, int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v,
                     int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, int64_t k_stride_b,
                     int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_t,
                     int64_t v_stride_h, float scale, void* stream, float* deltas = nullptr) {
    if (!known_dtype(qkv_dtype) || !known_dtype(beta_dtype)) return GDN_ERR_DTYPE;
    if (batch < 0 || seqlen < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads) return GDN_ERR_SHAPE;
    if (batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (batch == 0 || seqlen == 0) {
        // nothing to run; a zero-length call still copies the state through
        if (batch > 0 && state_out && state_out != state_in && !steps) {
            const size_t bytes = (size_t)batch * value_heads * kHeadDim * kHeadDim * sizeof(float);
            cudaError_t e = state_in ? cudaMemcpyAsync(state_out, state_in, bytes, cudaMemcpyDeviceToDevice, as_stream(stream))
                                     : cudaMemsetAsync(state_out, 0, bytes, as_stream(stream));
            return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
        }
        return GDN_OK;
    }
    if (!k || !v || (!gates && (!g || !beta))) return GDN_ERR_NULL;
    if (o && !q) return GDN_ERR_NULL;
    GateInputs G{};
    if (gates) {
        const int st = gate_args(gates, &G);
        if (st != GDN_OK) return st;
    }
    if (steps && (o || snapshots)) return GDN_ERR_SHAPE;  // an advance writes only the state
    const int es = elem_size(qkv_dtype);
    if (!rows_aligned(k, es, k_stride_b, k_stride_t, k_stride_h) || !rows_aligned(v, es, v_stride_b, v_stride_t, v_stride_h))
        return GDN_ERR_ALIGN;
    if (q && !rows_aligned(q, es, q_stride_b, q_stride_t, q_stride_h)) return GDN_ERR_ALIGN;
    if ((state_in && !aligned16(state_in)) || (state_out && !aligned16(state_out)) ||
        (snapshots && !aligned16(snapshots)) || (o && !aligned16(o)) || (deltas && !aligned16(deltas)))
        return GDN_ERR_ALIGN;
    RecurrentArgs a{};
    a.q = q; a.k = k; a.v = v; a.qkv_dtype = qkv_dtype;
    a.g = g; a.beta = beta; a.beta_dtype = beta_dtype;
    a.state_in = state_in; a.state_out = state_out; a.snapshots = snapshots; a.o = o;
    a.steps = steps; a.cu_seqlens = cu_seqlens;
    a.rows = batch; a.T = seqlen; a.H = (int)key_heads; a.HV = (int)value_heads;
    a.qsb = q_stride_b; a.qst = q_stride_t; a.qsh = q_stride_h;
    a.ksb = k_stride_b; a.kst = k_stride_t; a.ksh = k_stride_h;
    a.vsb = v_stride_b; a.vst = v_stride_t; a.vsh = v_stride_h;
    a.scale = scale;
    a.gates = G;
    a.deltas = deltas;
    if (deltas && qkv_dtype == GDN_BF16 && seqlen <= 8 && !cu_seqlens && state_in && !gates && !state_out &&
        !snapshots && !steps) {
        // a verify block of up to 8 tokens: one tensor-core pass over each state
        VerifyBlockArgs vb{};
        vb.q = q; vb.k = k; vb.v = v; vb.g = g; vb.beta = beta; vb.beta_dtype = beta_dtype;
        vb.state_in = state_in; vb.o = o; vb.deltas = deltas;
        vb.rows = batch; vb.T = seqlen; vb.H = (int)key_heads; vb.HV = (int)value_heads;
        vb.qsb = q_stride_b; vb.qst = q_stride_t; vb.qsh = q_stride_h;
        vb.ksb = k_stride_b; vb.kst = k_stride_t; vb.ksh = k_stride_h;
        vb.vsb = v_stride_b; vb.vst = v_stride_t; vb.vsh = v_stride_h;
        vb.scale = scale;
        return launch_verify_block(vb, as_stream(stream));
    }
    return launch_recurrent(a, as_stream(stream));
}

int gdn_recurrent(const void* q, const void* k, const void* v, int qkv_dtype, const float* g, const void* beta,
                  int beta_dtype, const float* state_in, float* state_out, float* snapshots, void* o,
                  const int64_t* steps, const int32_t* cu_seqlens, int64_t batch, int64_t seqlen, int64_t key_heads,
                  int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v, int64_t q_stride_b, int64_t q_stride_t,
                  int64_t q_stride_h, int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b,
                  int64_t v_stride_t, int64_t v_stride_h, float scale, void* stream) {
    return recurrent(q, k, v, qkv_dtype, g, beta, beta_dtype, nullptr, state_in, state_out, snapshots, o, steps,
                     cu_seqlens, batch, seqlen, key_heads, value_heads, head_dim_k, head_dim_v, q_stride_b, q_stride_t,
                     q_stride_h, k_stride_b, k_stride_t, k_stride_h, v_stride_b, v_stride_t, v_stride_h, scale, stream);
}

int gdn_recurrent_gates(const void* q, const void* k, const void* v, int qkv_dtype, const gdn_gate_inputs* gates,
                        const float* state_in, float* state_out, float* snapshots, void* o, const int64_t* steps,
                        const int32_t* cu_seqlens, int64_t batch, int64_t seqlen, int64_t key_heads,
                        int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v, int64_t q_stride_b,
                        int64_t q_stride_t, int64_t q_stride_h, int64_t k_stride_b, int64_t k_stride_t,
                        int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h, float scale,
                        void* stream) {
    if (!gates) return GDN_ERR_NULL;
    return recurrent(q, k, v, qkv_dtype, nullptr, nullptr, GDN_BF16, gates, state_in, state_out, snapshots, o, steps,
                     cu_seqlens, batch, seqlen, key_heads, value_heads, head_dim_k, head_dim_v, q_stride_b, q_stride_t,
                     q_stride_h, k_stride_b, k_stride_t, k_stride_h, v_stride_b, v_stride_t, v_stride_h, scale, stream);
}

int gdn_recurrent_deltas(const void* q, const void* k, const void* v, int qkv_dtype, const float* g, const void* beta,
                         int beta_dtype, const float* state_in, void* o, float* deltas, int64_t batch, int64_t seqlen,
                         int64_t key_heads, int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v,
                         int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, int64_t k_stride_b,
                         int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_t,
                         int64_t v_stride_h, float scale, void* stream) {
    if (batch > 0 && seqlen > 0 && (!q || !o || !deltas)) return GDN_ERR_NULL;
    return recurrent(q, k, v, qkv_dtype, g, beta, beta_dtype, nullptr, state_in, nullptr, nullptr, o, nullptr, nullptr,
                     batch, seqlen, key_heads, value_heads, head_dim_k, head_dim_v, q_stride_b, q_stride_t, q_stride_h,
                     k_stride_b, k_stride_t, k_stride_h, v_stride_b, v_stride_t, v_stride_h, scale, stream, deltas);
}

int gdn_recurrent_deltas_gated_norm(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                    int beta_dtype, const float* state_in, const void* z, const void* norm_weight,
                                    float eps, void* y, float* deltas, int64_t batch, int64_t seqlen,
                                    int64_t key_heads, int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v,
                                    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, int64_t k_stride_b,
                                    int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_t,
                                    int64_t v_stride_h, float scale, void* stream) {
    if (!known_dtype(beta_dtype)) return GDN_ERR_DTYPE;
    if (batch < 0 || seqlen < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads) return GDN_ERR_SHAPE;
    if (batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (seqlen > 8) return GDN_ERR_UNSUPPORTED;  // the tensor-core block takes up to 8 tokens
    if (batch == 0 || seqlen == 0) return GDN_OK;
    if (!q || !k || !v || !g || !beta || !state_in || !z || !norm_weight || !y || !deltas) return GDN_ERR_NULL;
    if (!rows_aligned(q, 2, q_stride_b, q_stride_t, q_stride_h) || !rows_aligned(k, 2, k_stride_b, k_stride_t, k_stride_h) ||
        !rows_aligned(v, 2, v_stride_b, v_stride_t, v_stride_h) || !aligned16(state_in) || !aligned16(z) ||
        !aligned16(deltas))
        return GDN_ERR_ALIGN;
    VerifyBlockArgs vb{};
    vb.q = q; vb.k = k; vb.v = v; vb.g = g; vb.beta = beta; vb.beta_dtype = beta_dtype;
    vb.state_in = state_in; vb.o = nullptr; vb.deltas = deltas;
    vb.rows = batch; vb.T = seqlen; vb.H = (int)key_heads; vb.HV = (int)value_heads;
    vb.qsb = q_stride_b; vb.qst = q_stride_t; vb.qsh = q_stride_h;
    vb.ksb = k_stride_b; vb.kst = k_stride_t; vb.ksh = k_stride_h;
    vb.vsb = v_stride_b; vb.vst = v_stride_t; vb.vsh = v_stride_h;
    vb.scale = scale;
    vb.z = z; vb.norm_w = norm_weight; vb.y = y; vb.eps = eps;
    return launch_verify_block(vb, as_stream(stream));
}

static int delta_commit(float* const* states, const void* const* ks, int k_dtype, const float* const* gs,
                        const float* const* deltas, int64_t layers, const int64_t* accepted, int64_t batch,
                        int64_t seqlen, int64_t key_heads, int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v,
                        int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h, void* stream) {
    if (!known_dtype(k_dtype)) return GDN_ERR_DTYPE;
    if (layers < 0 || batch < 0 || seqlen < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads)
        return GDN_ERR_SHAPE;
    if (batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (batch == 0 || seqlen == 0 || layers == 0) return GDN_OK;
    if (!states || !ks || !gs || !deltas || !accepted) return GDN_ERR_NULL;
    const int64_t state_bytes = batch * value_heads * kHeadDim * kHeadDim * (int64_t)sizeof(float);
    for (int64_t l = 0; l < layers; ++l) {
        if (!states[l] || !ks[l] || !gs[l] || !deltas[l]) return GDN_ERR_NULL;
        if (!aligned16(states[l]) || !aligned16(deltas[l]) ||
            !rows_aligned(ks[l], elem_size(k_dtype), k_stride_b, k_stride_t, k_stride_h))
            return GDN_ERR_ALIGN;
        // the layers' states are advanced by one launch: no two may overlap
        const char* a0 = reinterpret_cast<const char*>(states[l]);
        for (int64_t m = 0; m < l; ++m) {
            const char* b0 = reinterpret_cast<const char*>(states[m]);
            if (a0 < b0 + state_bytes && b0 < a0 + state_bytes) return GDN_ERR_SHAPE;
        }
    }
    DeltaCommitArgs a{};
    a.states = states; a.ks = ks; a.k_dtype = k_dtype; a.gs = gs; a.deltas = deltas; a.layers = layers;
    a.accepted = accepted;
    a.rows = batch; a.T = seqlen; a.H = (int)key_heads; a.HV = (int)value_heads;
    a.ksb = k_stride_b; a.kst = k_stride_t; a.ksh = k_stride_h;
    return launch_delta_commit(a, as_stream(stream));
}

int gdn_delta_commit(float* state, const void* k, int k_dtype, const float* g, const float* deltas,
                     const int64_t* accepted, int64_t batch, int64_t seqlen, int64_t key_heads, int64_t value_heads,
                     int64_t head_dim_k, int64_t head_dim_v, int64_t k_stride_b, int64_t k_stride_t,
                     int64_t k_stride_h, void* stream) {
    return delta_commit(&state, &k, k_dtype, &g, &deltas, 1, accepted, batch, seqlen, key_heads, value_heads,
                        head_dim_k, head_dim_v, k_stride_b, k_stride_t, k_stride_h, stream);
}

int gdn_delta_commit_layers(float* const* states, const void* const* k, int k_dtype, const float* const* g,
                            const float* const* deltas, int64_t layers, const int64_t* accepted, int64_t batch,
                            int64_t seqlen, int64_t key_heads, int64_t value_heads, int64_t head_dim_k,
                            int64_t head_dim_v, int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
                            void* stream) {
    return delta_commit(states, k, k_dtype, g, deltas, layers, accepted, batch, seqlen, key_heads, value_heads,
                        head_dim_k, head_dim_v, k_stride_b, k_stride_t, k_stride_h, stream);
}

int gdn_verify_layer_deltas(const void* qkv, int64_t qkv_stride_b, int64_t qkv_stride_t, const void* conv_state,
                            const void* conv_w, void* ext, void* q, void* k, void* v, const float* g,
                            const void* beta, int beta_dtype, const float* state, const void* z, const void* norm_w,
                            void* y, float* deltas, int64_t batch, int64_t seqlen, int64_t key_heads,
                            int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v, int64_t taps,
                            int64_t kernel_size, float scale, float eps, void* stream) {
    if (!known_dtype(beta_dtype)) return GDN_ERR_DTYPE;
    if (batch < 0 || seqlen < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads) return GDN_ERR_SHAPE;
    if (taps < 1 || taps > 8 || kernel_size < 1 || kernel_size > taps + 1 || kernel_size > 8) return GDN_ERR_SHAPE;
    if (batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (seqlen > 8) return GDN_ERR_UNSUPPORTED;  // the tensor-core block takes up to 8 tokens
    if (batch == 0 || seqlen == 0) return GDN_OK;
    if (!qkv || !conv_state || !conv_w || !ext || !q || !k || !v || !g || !beta || !state || !z || !norm_w || !y ||
        !deltas)
        return GDN_ERR_NULL;
    // qkv may have any row strides (the conv step takes 16-byte accesses only where they are aligned)
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(state) || !aligned16(z) || !aligned16(y) ||
        !aligned16(deltas) || !aligned16(norm_w))
        return GDN_ERR_ALIGN;
    VerifyLayerArgs a{};
    a.qkv = qkv; a.qkv_sb = qkv_stride_b; a.qkv_st = qkv_stride_t;
    a.conv_state = conv_state; a.conv_w = conv_w; a.ext = ext;
    a.q = q; a.k = k; a.v = v;
    a.g = g; a.beta = beta; a.beta_dtype = beta_dtype;
    a.state = state; a.z = z; a.norm_w = norm_w; a.y = y; a.deltas = deltas;
    a.B = batch; a.T = seqlen; a.H = (int)key_heads; a.HV = (int)value_heads;
    a.taps = (int)taps; a.K = (int)kernel_size;
    a.scale = scale; a.eps = eps;
    return launch_verify_layer(a, as_stream(stream));
}

static int chunk_prefill(const void* q, const void* k, const void* v, const float* g, const void* beta, int beta_dtype,
                         const gdn_gate_inputs* gates, const float* initial_state, float* final_state, void* o, const int32_t* cu_seqlens,
                         int64_t batch, int64_t seqlen, int64_t key_heads, int64_t value_heads, int64_t head_dim_k,
                         int64_t head_dim_v, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
                         int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b,
                         int64_t v_stride_t, int64_t v_stride_h, float scale, void* workspace, size_t workspace_bytes,
                         const void* z, const void* norm_weight, float eps, void* out, void* stream) {
    if (!known_dtype(beta_dtype)) return GDN_ERR_DTYPE;
    if (batch < 0 || seqlen < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads) return GDN_ERR_SHAPE;
    if (batch > 65535 || value_heads > 512) return GDN_ERR_SHAPE;
    if (seqlen > INT32_MAX - 64) return GDN_ERR_SHAPE;  // TMA coordinates are 32-bit
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (batch == 0) return GDN_OK;
    if (!q || !k || !v || !o || (!gates && (!g || !beta))) return GDN_ERR_NULL;
    GateInputs G{};
    if (gates) {
        const int st = gate_args(gates, &G);
        if (st != GDN_OK) return st;
    }
    if (cu_seqlens == nullptr && seqlen == 0) return GDN_OK;
    if (!rows_aligned(q, 2, q_stride_b, q_stride_t, q_stride_h) || !rows_aligned(k, 2, k_stride_b, k_stride_t, k_stride_h) ||
        !rows_aligned(v, 2, v_stride_b, v_stride_t, v_stride_h) || !aligned16(o))
        return GDN_ERR_ALIGN;
    if ((initial_state && !aligned16(initial_state)) || (final_state && !aligned16(final_state))) return GDN_ERR_ALIGN;
    ChunkArgs a{};
    a.q = q; a.k = k; a.v = v; a.g = g; a.beta = beta; a.beta_dtype = beta_dtype;
    a.h0 = initial_state; a.ht = final_state; a.o = o; a.cu_seqlens = cu_seqlens;
    a.B = cu_seqlens ? 1 : batch; a.T = seqlen; a.nseq = batch;
    a.H = (int)key_heads; a.HV = (int)value_heads;
    a.qsb = q_stride_b; a.qst = q_stride_t; a.qsh = q_stride_h;
    a.ksb = k_stride_b; a.kst = k_stride_t; a.ksh = k_stride_h;
    a.vsb = v_stride_b; a.vst = v_stride_t; a.vsh = v_stride_h;
    a.scale = scale;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    a.gates = G;
    a.z = z;
    a.norm_w = norm_weight;
    a.y = out;
    a.eps = eps;
    if (workspace && !aligned16(workspace)) return GDN_ERR_ALIGN;
    return launch_chunk(a, as_stream(stream));
}

int gdn_chunk_prefill(const void* q, const void* k, const void* v, const float* g, const void* beta, int beta_dtype,
                      const float* initial_state, float* final_state, void* o, const int32_t* cu_seqlens,
                      int64_t batch, int64_t seqlen, int64_t key_heads, int64_t value_heads, int64_t head_dim_k,
                      int64_t head_dim_v, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
                      int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b,
                      int64_t v_stride_t, int64_t v_stride_h, float scale, void* workspace, size_t workspace_bytes,
                      void* stream) {
    return chunk_prefill(q, k, v, g, beta, beta_dtype, nullptr, initial_state, final_state, o, cu_seqlens, batch, seqlen,
                         key_heads, value_heads, head_dim_k, head_dim_v, q_stride_b, q_stride_t, q_stride_h, k_stride_b,
                         k_stride_t, k_stride_h, v_stride_b, v_stride_t, v_stride_h, scale, workspace, workspace_bytes,
                         nullptr, nullptr, 0.f, nullptr, stream);
}

int gdn_chunk_prefill_gated_norm(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                 int beta_dtype, const float* initial_state, float* final_state, void* o,
                                 const int32_t* cu_seqlens, int64_t batch, int64_t seqlen, int64_t key_heads,
                                 int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v, int64_t q_stride_b,
                                 int64_t q_stride_t, int64_t q_stride_h, int64_t k_stride_b, int64_t k_stride_t,
                                 int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
                                 float scale, const void* z, const void* norm_weight, float eps, void* out,
                                 void* workspace, size_t workspace_bytes, void* stream) {
    if (batch > 0 && (!z || !norm_weight || !out)) return GDN_ERR_NULL;
    if (!aligned16(z) || !aligned16(norm_weight) || !aligned16(out)) return GDN_ERR_ALIGN;
    return chunk_prefill(q, k, v, g, beta, beta_dtype, nullptr, initial_state, final_state, o, cu_seqlens, batch, seqlen,
                         key_heads, value_heads, head_dim_k, head_dim_v, q_stride_b, q_stride_t, q_stride_h, k_stride_b,
                         k_stride_t, k_stride_h, v_stride_b, v_stride_t, v_stride_h, scale, workspace, workspace_bytes,
                         z, norm_weight, eps, out, stream);
}

int gdn_chunk_prefill_gates(const void* q, const void* k, const void* v, const gdn_gate_inputs* gates,
                            const float* initial_state, float* final_state, void* o, const int32_t* cu_seqlens,
                            int64_t batch, int64_t seqlen, int64_t key_heads, int64_t value_heads, int64_t head_dim_k,
                            int64_t head_dim_v, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
                            int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_b,
                            int64_t v_stride_t, int64_t v_stride_h, float scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
    if (!gates) return GDN_ERR_NULL;
    return chunk_prefill(q, k, v, nullptr, nullptr, GDN_BF16, gates, initial_state, final_state, o, cu_seqlens, batch,
                         seqlen, key_heads, value_heads, head_dim_k, head_dim_v, q_stride_b, q_stride_t, q_stride_h,
                         k_stride_b, k_stride_t, k_stride_h, v_stride_b, v_stride_t, v_stride_h, scale, workspace,
                         workspace_bytes, nullptr, nullptr, 0.f, nullptr, stream);
}

size_t gdn_chunk_prefill_workspace_size(int64_t batch, int64_t seqlen, int64_t value_heads, int packed) {
    if (batch < 0 || seqlen < 0 || value_heads <= 0) return 0;
    return chunk_workspace_bytes(packed ? 1 : batch, seqlen, batch, packed != 0, value_heads);
}

int gdn_snapshot_commit(float* state, const float* snapshots, const int64_t* accepted, int64_t batch, int64_t seqlen,
                        int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v, void* stream) {
    if (batch < 0 || seqlen <= 0 || value_heads <= 0 || batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (batch == 0) return GDN_OK;
    if (!state || !snapshots || !accepted) return GDN_ERR_NULL;
    if (!aligned16(state) || !aligned16(snapshots)) return GDN_ERR_ALIGN;
    return launch_snapshot_commit(state, snapshots, accepted, batch, seqlen, value_heads, as_stream(stream));
}

int gdn_conv1d_silu(const void* x, int64_t x_stride_b, int64_t x_stride_t, const void* w, void* y,
                    const int32_t* cu_seqlens, int64_t batch, int64_t seqlen, int64_t channels, int64_t kernel_size,
                    void* stream) {
    if (batch < 0 || seqlen < 0 || channels <= 0 || channels % 8) return GDN_ERR_SHAPE;
    if (kernel_size < 2 || kernel_size > 4) return GDN_ERR_UNSUPPORTED;
    if (batch == 0 || seqlen == 0) return GDN_OK;
    if (!x || !w || !y) return GDN_ERR_NULL;
    if (!rows_aligned(x, 2, x_stride_b, x_stride_t, 0) || !aligned16(y) || !aligned16(w)) return GDN_ERR_ALIGN;
    if (!cu_seqlens && batch > 65535) return GDN_ERR_SHAPE;
    if (channels / 8 > 65535 * 128 || seqlen > INT32_MAX) return GDN_ERR_SHAPE;
    return launch_conv1d_silu(x, x_stride_b, x_stride_t, w, y, cu_seqlens, batch, seqlen, channels, (int)kernel_size,
                              as_stream(stream));
}

int gdn_conv1d_silu_step(const void* x, int64_t x_stride_b, void* state, const void* w, void* y, int64_t batch,
                         int64_t channels, int64_t taps, int64_t kernel_size, void* stream) {
    if (batch < 0 || channels <= 0 || channels % 8 || taps < 1 || kernel_size < 1 || kernel_size > taps + 1)
        return GDN_ERR_SHAPE;
    if (taps < 2 || taps > 4 || kernel_size < 2) return GDN_ERR_UNSUPPORTED;
    if (batch == 0) return GDN_OK;
    if (!x || !state || !w || !y) return GDN_ERR_NULL;
    if (!rows_aligned(x, 2, x_stride_b, 0, 0) || !aligned16(state) || !aligned16(y) || !aligned16(w)) return GDN_ERR_ALIGN;
    return launch_conv1d_silu_step(x, x_stride_b, state, w, y, batch, channels, (int)taps, (int)kernel_size,
                                   as_stream(stream));
}

int gdn_conv_step(const void* state, const void* qkv, int64_t qkv_stride_b, int64_t qkv_stride_t, const void* w,
                  void* ext, void* q, void* k, void* v, int64_t batch, int64_t seqlen, int64_t taps, int64_t kernel_size,
                  int64_t key_dim, int64_t value_dim, int64_t head_dim_k, int64_t head_dim_v, void* stream) {
    if (batch < 0 || seqlen < 0 || taps < 1 || taps > 8 || kernel_size < 1 || kernel_size > taps + 1 || kernel_size > 8)
        return GDN_ERR_SHAPE;
    if (head_dim_k <= 0 || head_dim_v <= 0 || key_dim <= 0 || value_dim <= 0) return GDN_ERR_SHAPE;
    if (key_dim % head_dim_k || value_dim % head_dim_v) return GDN_ERR_SHAPE;
    const int64_t kh = key_dim / head_dim_k, vh = value_dim / head_dim_v;
    if (vh % kh) return GDN_ERR_SHAPE;
    if (batch > 65535) return GDN_ERR_SHAPE;
    if (batch == 0 || seqlen == 0) {
        if (batch == 0) return GDN_OK;
    }
    if (!state || !qkv || !w || !ext || !q || !k || !v) return GDN_ERR_NULL;
    return launch_conv_step(state, qkv, qkv_stride_b, qkv_stride_t, w, ext, q, k, v, batch, seqlen, (int)taps,
                            (int)kernel_size, key_dim, value_dim, (int)head_dim_k, (int)head_dim_v, as_stream(stream));
}

int gdn_conv_state_commit(const void* ext, void* state, const int64_t* accepted, int64_t layers, int64_t batch,
                          int64_t channels, int64_t taps, int64_t seqlen, int64_t ext_stride_layer,
                          int64_t ext_stride_b, int64_t state_stride_layer, int64_t state_stride_b, void* stream) {
    if (layers < 0 || batch < 0 || channels < 0 || seqlen < 0 || taps < 1 || taps > 8) return GDN_ERR_SHAPE;
    if (layers > 65535 || batch > 65535) return GDN_ERR_SHAPE;
    if (layers == 0 || batch == 0 || channels == 0) return GDN_OK;
    if (!ext || !state || !accepted) return GDN_ERR_NULL;
    if (ext_stride_b < channels * (taps + seqlen) || state_stride_b < channels * taps ||
        (layers > 1 && (ext_stride_layer < batch * ext_stride_b || state_stride_layer < batch * state_stride_b)))
        return GDN_ERR_SHAPE;
    return launch_conv_state_commit(ext, state, accepted, layers, batch, channels, (int)taps, seqlen, ext_stride_layer,
                                    ext_stride_b, state_stride_layer, state_stride_b, as_stream(stream));
}

int gdn_delta_gates(const void* b, int64_t b_stride, const void* a, int64_t a_stride, const void* dt_bias,
                    int dt_bias_dtype, const float* log_decay_rate, const uint8_t* valid, void* beta, float* g,
                    int64_t rows, int64_t value_heads, void* stream) {
    if (!known_dtype(dt_bias_dtype)) return GDN_ERR_DTYPE;
    if (rows < 0 || value_heads <= 0 || value_heads > 4096 || b_stride < value_heads || a_stride < value_heads)
        return GDN_ERR_SHAPE;
    if (rows > INT64_MAX / value_heads || rows * value_heads > (int64_t)INT32_MAX * 256) return GDN_ERR_SHAPE;
    if (rows == 0) return GDN_OK;
    if (!b || !a || !dt_bias || !log_decay_rate || !beta || !g) return GDN_ERR_NULL;
    return launch_delta_gates(b, b_stride, a, a_stride, dt_bias, dt_bias_dtype == GDN_F32, log_decay_rate, valid,
                              beta, g, rows, (int)value_heads, as_stream(stream));
}

int gdn_gated_rmsnorm(const void* x, const void* z, const void* w, void* y, int64_t rows, int64_t dim, float eps,
                      void* stream) {
    if (rows < 0 || dim <= 0) return GDN_ERR_SHAPE;
    if (dim != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (rows == 0) return GDN_OK;
    if (!x || !z || !w || !y) return GDN_ERR_NULL;
    if (!aligned16(x) || !aligned16(z) || !aligned16(y) || !aligned16(w)) return GDN_ERR_ALIGN;
    if (rows > (int64_t)65535 * 65535) return GDN_ERR_SHAPE;
    return launch_gated_rmsnorm(x, z, w, y, rows, (int)dim, eps, as_stream(stream));
}

size_t gdn_decode_attention_workspace_size(int64_t batch, int64_t kv_heads, int64_t keys, int64_t head_dim) {
    if (batch < 0 || kv_heads <= 0 || keys < 0 || (head_dim != 128 && head_dim != 256)) return 0;
    return decode_attention_workspace_bytes(batch, kv_heads, keys, head_dim);
}

int gdn_decode_attention(const void* q, int64_t q_stride_b, int64_t q_stride_r, int64_t q_stride_h,
                         const void* k_cache, int64_t k_stride_b, int64_t k_stride_s, int64_t k_stride_h,
                         const void* v_cache, int64_t v_stride_b, int64_t v_stride_s, int64_t v_stride_h,
                         const void* mask, int64_t mask_stride_b, int64_t mask_stride_r, void* o, int64_t batch,
                         int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t keys,
                         int64_t cache_rows, int64_t cache_len, float scale, void* workspace, size_t workspace_bytes,
                         void* stream) {
    if (batch < 0 || rows <= 0 || kv_heads <= 0 || heads <= 0 || heads % kv_heads || keys < 0) return GDN_ERR_SHAPE;
    if (batch > cache_rows || keys > cache_len || batch > 65535 || kv_heads > 65535 || cache_len > INT32_MAX)
        return GDN_ERR_SHAPE;
    if (head_dim != 128 && head_dim != 256) return GDN_ERR_UNSUPPORTED;
    if (rows * (heads / kv_heads) > 64) return GDN_ERR_UNSUPPORTED;  // query rows per key head
    if (batch == 0) return GDN_OK;
    if (!q || !o || (keys > 0 && (!k_cache || !v_cache || !mask))) return GDN_ERR_NULL;
    if (!aligned16(o) || !rows_aligned(q, 2, q_stride_b, q_stride_r, q_stride_h)) return GDN_ERR_ALIGN;
    if (keys > 0 && (!rows_aligned(k_cache, 2, k_stride_b, k_stride_s, k_stride_h) ||
                     !rows_aligned(v_cache, 2, v_stride_b, v_stride_s, v_stride_h) ||
                     !rows_aligned(mask, 2, mask_stride_b, mask_stride_r, 0)))
        return GDN_ERR_ALIGN;
    if (workspace && !aligned16(workspace)) return GDN_ERR_ALIGN;
    AttentionArgs a{};
    a.q = q; a.qsb = q_stride_b; a.qsr = q_stride_r; a.qsh = q_stride_h;
    a.k = k_cache; a.ksb = k_stride_b; a.kss = k_stride_s; a.ksh = k_stride_h;
    a.v = v_cache; a.vsb = v_stride_b; a.vss = v_stride_s; a.vsh = v_stride_h;
    a.mask = mask; a.msb = mask_stride_b; a.msr = mask_stride_r;
    a.o = o;
    a.B = batch; a.R = rows; a.H = heads; a.Hkv = kv_heads; a.D = head_dim; a.L = keys;
    a.cache_rows = cache_rows; a.cache_len = cache_len;
    a.scale = scale;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    return launch_decode_attention(a, as_stream(stream));
}

int gdn_rotary(const void* x, const float* cos, const float* sin, void* out, int64_t batch, int64_t seqlen,
               int64_t heads, int64_t head_dim, int64_t n_freqs, void* stream) {
    if (batch < 0 || seqlen < 0 || heads <= 0 || head_dim <= 0 || n_freqs < 0) return GDN_ERR_SHAPE;
    if (2 * n_freqs > head_dim) return GDN_ERR_SHAPE;
    if (head_dim > 1024) return GDN_ERR_UNSUPPORTED;
    const int64_t rows = batch * seqlen * heads;
    if (rows == 0) return GDN_OK;
    if (!x || !out || (n_freqs > 0 && (!cos || !sin))) return GDN_ERR_NULL;
    if (rows > INT32_MAX) return GDN_ERR_SHAPE;
    return launch_rotary(x, cos, sin, out, rows, (int)heads, (int)head_dim, (int)n_freqs, as_stream(stream));
}

int gdn_rotate_into_cache(const void* k, const void* v, const void* qm, const void* km, const void* vm,
                          int64_t m_stride_b, int64_t m_stride_t, const float* cos_c, const float* sin_c,
                          const float* cos_m, const float* sin_m, void* k_cache, void* v_cache, int64_t cache_stride_b,
                          int64_t cache_stride_s, void* q_out, const int64_t* rows, int64_t rows_stride_b,
                          int64_t rows_stride_t, const int64_t* positions, int64_t tail_start, int64_t batch,
                          int64_t candidates, int64_t mask_rows, int64_t heads, int64_t head_dim, int64_t n_freqs,
                          void* stream) {
    if (batch < 0 || candidates < 0 || mask_rows < 0 || heads <= 0 || head_dim <= 0 || n_freqs < 0 || tail_start < 0)
        return GDN_ERR_SHAPE;
    if (2 * n_freqs > head_dim) return GDN_ERR_SHAPE;
    if (head_dim > 1024) return GDN_ERR_UNSUPPORTED;
    const int64_t progs = batch * (candidates + mask_rows) * heads;
    if (progs == 0) return GDN_OK;
    if (progs > INT32_MAX || candidates + mask_rows > INT32_MAX) return GDN_ERR_SHAPE;
    if (!k_cache || !v_cache) return GDN_ERR_NULL;
    if (candidates > 0 && (!k || !v || !rows || !positions || (n_freqs > 0 && (!cos_c || !sin_c)))) return GDN_ERR_NULL;
    if (mask_rows > 0 && (!qm || !km || !vm || !q_out || (n_freqs > 0 && (!cos_m || !sin_m)))) return GDN_ERR_NULL;
    RotateCacheArgs a{};
    a.k = k; a.v = v; a.qm = qm; a.km = km; a.vm = vm; a.msb = m_stride_b; a.mst = m_stride_t;
    a.cos_c = cos_c; a.sin_c = sin_c; a.cos_m = cos_m; a.sin_m = sin_m;
    a.k_cache = k_cache; a.v_cache = v_cache; a.csb = cache_stride_b; a.css = cache_stride_s;
    a.q_out = q_out; a.rows = rows; a.rsb = rows_stride_b; a.rst = rows_stride_t; a.positions = positions;
    a.tail_start = tail_start;
    a.B = batch; a.K = (int)candidates; a.M = (int)mask_rows; a.H = (int)heads; a.D = (int)head_dim; a.nf = (int)n_freqs;
    return launch_rotate_into_cache(a, as_stream(stream));
}

// The checks both forms of the merged projection share; GDN_OK lets the call go on (tokens > 0).
static int in_proj_checks(const void* x, int64_t x_stride, const void* conv_w, const int32_t* cu_seqlens, void* out,
                          int64_t out_stride, void* conv_state, int64_t tokens, int64_t hidden, int64_t out_channels,
                          int64_t conv_channels, int64_t sequences, int64_t conv_kernel) {
    if (tokens < 0 || hidden <= 0 || out_channels <= 0 || conv_channels < 0 || conv_channels > out_channels)
        return GDN_ERR_SHAPE;
    if (hidden % 64 || out_channels % 8 || conv_channels % 8 || tokens > INT32_MAX - 256) return GDN_ERR_SHAPE;
    if (out_channels > (int64_t)65535 * 256 || hidden > INT32_MAX) return GDN_ERR_SHAPE;
    if (conv_kernel != 4) return GDN_ERR_UNSUPPORTED;
    if (cu_seqlens ? sequences < 1 : sequences != 1) return GDN_ERR_SHAPE;
    if (tokens == 0) return GDN_OK;
    if (!x || !out || (conv_channels > 0 && !conv_w)) return GDN_ERR_NULL;
    if (!rows_aligned(x, 2, x_stride, 0, 0) || !rows_aligned(out, 2, out_stride, 0, 0) ||
        (conv_w && !aligned16(conv_w)) || (conv_state && !aligned16(conv_state)))
        return GDN_ERR_ALIGN;
    return GDN_OK;
}

size_t gdn_in_proj_fp8_workspace_size(int64_t tokens, int64_t hidden) {
    if (tokens <= 0 || hidden <= 0) return 0;
    return in_proj_fp8_workspace_bytes(tokens, hidden);
}

size_t gdn_in_proj_fp8_prefill_workspace_size(int64_t tokens, int64_t hidden, int64_t out_channels,
                                              int64_t conv_channels) {
    if (tokens <= 0 || hidden <= 0 || out_channels <= 0 || conv_channels < 0) return 0;
    return in_proj_fp8_prefill_workspace_bytes(tokens, hidden, out_channels, conv_channels);
}

int gdn_in_proj_conv_fp8(const void* x, int64_t x_stride, const void* codes, int64_t codes_stride,
                         const float* w_scale, const void* conv_w, const int32_t* cu_seqlens, void* out,
                         int64_t out_stride, void* conv_state, void* workspace, size_t workspace_bytes,
                         int64_t tokens, int64_t hidden, int64_t out_channels, int64_t conv_channels,
                         int64_t sequences, int64_t conv_kernel, void* stream) {
    const int st = in_proj_checks(x, x_stride, conv_w, cu_seqlens, out, out_stride, conv_state, tokens, hidden,
                                  out_channels, conv_channels, sequences, conv_kernel);
    if (st != GDN_OK || tokens == 0) return st;
    if (!codes || !w_scale) return GDN_ERR_NULL;
    if (!aligned16(codes) || codes_stride < hidden || codes_stride % 16) return GDN_ERR_ALIGN;
    if (!workspace || workspace_bytes < in_proj_fp8_workspace_bytes(tokens, hidden)) return GDN_ERR_WORKSPACE;
    if (!aligned16(workspace)) return GDN_ERR_ALIGN;
    InProjArgs a{};
    a.x = x; a.ldx = x_stride; a.conv_w = conv_w; a.cu_seqlens = cu_seqlens;
    a.out = out; a.ldo = out_stride; a.conv_tail = conv_channels > 0 ? conv_state : nullptr;
    a.T = tokens; a.K = hidden; a.N = out_channels; a.C = conv_channels; a.nseq = sequences;
    a.codes = codes; a.ldc = codes_stride; a.w_scale = w_scale; a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    return launch_in_proj_conv(a, as_stream(stream));
}

int gdn_in_proj_conv(const void* x, int64_t x_stride, const void* w, int64_t w_stride, const void* conv_w,
                     const int32_t* cu_seqlens, void* out, int64_t out_stride, void* conv_state, int64_t tokens,
                     int64_t hidden, int64_t out_channels, int64_t conv_channels, int64_t sequences,
                     int64_t conv_kernel, void* stream) {
    const int st = in_proj_checks(x, x_stride, conv_w, cu_seqlens, out, out_stride, conv_state, tokens, hidden,
                                  out_channels, conv_channels, sequences, conv_kernel);
    if (st != GDN_OK || tokens == 0) return st;
    if (!w) return GDN_ERR_NULL;
    if (!rows_aligned(w, 2, w_stride, 0, 0)) return GDN_ERR_ALIGN;
    InProjArgs a{};
    a.x = x; a.ldx = x_stride; a.w = w; a.ldw = w_stride; a.conv_w = conv_w; a.cu_seqlens = cu_seqlens;
    a.out = out; a.ldo = out_stride; a.conv_tail = conv_channels > 0 ? conv_state : nullptr;
    a.T = tokens; a.K = hidden; a.N = out_channels; a.C = conv_channels; a.nseq = sequences;
    return launch_in_proj_conv(a, as_stream(stream));
}

int gdn_decode_layer(const void* qkv, int64_t qkv_stride_b, void* conv_state, const void* conv_w, const float* g,
                     const void* beta, float* state, const void* z, const void* norm_w, void* out, void* workspace,
                     int64_t batch, int64_t key_heads, int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v,
                     int64_t taps, int64_t kernel_size, float scale, float eps, void* stream) {
    if (batch < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads) return GDN_ERR_SHAPE;
    if (taps < 1 || kernel_size < 1 || kernel_size > taps + 1) return GDN_ERR_SHAPE;
    if (taps < 2 || taps > 4 || kernel_size < 2) return GDN_ERR_UNSUPPORTED;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    if (batch == 0) return GDN_OK;
    if (!qkv || !conv_state || !conv_w || !g || !beta || !state || !z || !norm_w || !out || !workspace)
        return GDN_ERR_NULL;
    if (!rows_aligned(qkv, 2, qkv_stride_b, 0, 0) || !aligned16(conv_state) || !aligned16(state) || !aligned16(z) ||
        !aligned16(conv_w) ||
        !aligned16(out) || !aligned16(workspace) || !aligned16(norm_w))
        return GDN_ERR_ALIGN;
    DecodeLayerArgs a;
    a.qkv = qkv; a.qkv_sb = qkv_stride_b; a.conv_state = conv_state; a.conv_w = conv_w;
    a.g = g; a.beta = beta; a.state = state; a.z = z; a.norm_w = norm_w; a.out = out; a.workspace = workspace;
    a.B = batch; a.H = (int)key_heads; a.HV = (int)value_heads; a.taps = (int)taps; a.K = (int)kernel_size;
    a.scale = scale; a.eps = eps;
    return launch_decode_layer(a, as_stream(stream));
}

}  // extern "C"
