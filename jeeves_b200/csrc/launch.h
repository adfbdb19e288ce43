// Internal launcher declarations shared by the kernel files and the C ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

// The layer's raw gate projections, from which a kernel computes beta and g itself (the
// device copy of gdn_gate_inputs; the arithmetic is delta_gate in gates.cuh). b == null: none.
struct GateInputs {
    const void* b;  // [rows, HV] bf16 with row stride sb
    int64_t sb;
    const void* a;  // [rows, HV] bf16 with row stride sa
    int64_t sa;
    const void* dt_bias;  // [HV], fp32 (dt_f32) or bf16
    int dt_f32;
    const float* rate;     // [HV] log decay rate (-exp(A_log))
    const uint8_t* valid;  // [rows] or null
};

struct RecurrentArgs {
    const void* q;
    const void* k;
    const void* v;
    int qkv_dtype;
    const float* g;
    const void* beta;
    int beta_dtype;
    const float* state_in;
    float* state_out;
    float* snapshots;
    void* o;
    const int64_t* steps;
    const int32_t* cu_seqlens;
    int64_t rows;    // batch rows, or sequences when cu_seqlens is set
    int64_t T;       // token extent of the [B, T, ...] tensors (total tokens when packed)
    int H, HV;
    int64_t qsb, qst, qsh, ksb, kst, ksh, vsb, vst, vsh;
    float scale;
    GateInputs gates;  // used instead of g and beta when gates.b is set
    bool dependent = false;  // programmatic launch: may start while the previous kernel in the stream runs
    float* deltas = nullptr;  // [B, T, HV, 128] fp32: each token's update vector, or null
};
int launch_recurrent(const RecurrentArgs& a, cudaStream_t s);

// Per layer l < layers (host arrays of device pointers; the layers' states must not overlap):
struct DeltaCommitArgs {
    float* const* states;          // [rows, HV, 128, 128] fp32, advanced in place
    const void* const* ks;         // [rows, T, H, 128] with element strides ksb, kst, ksh (every layer)
    int k_dtype;
    const float* const* gs;        // [rows, T, HV]
    const float* const* deltas;    // [rows, T, HV, 128] fp32 from the verify
    int64_t layers;
    const int64_t* accepted;       // [rows], shared by the layers
    int64_t rows, T;
    int H, HV;
    int64_t ksb, kst, ksh;
};
int launch_delta_commit(const DeltaCommitArgs& a, cudaStream_t s);

// The verify that keeps its update vectors, for T <= 8 tokens of bf16 rows (verify_block.cu):
// outputs o and deltas ([rows, T, HV, 128]) from state_in ([rows, HV, 128, 128] fp32).
struct VerifyBlockArgs {
    const void* q;
    const void* k;
    const void* v;
    const float* g;
    const void* beta;
    int beta_dtype;
    const float* state_in;
    void* o;
    float* deltas;
    int64_t rows, T;
    int H, HV;
    int64_t qsb, qst, qsh, ksb, kst, ksh, vsb, vst, vsh;
    float scale;
    // the output-gated RMSNorm fused into the drain: y instead of o when y is set
    const void* z = nullptr;
    const void* norm_w = nullptr;
    void* y = nullptr;
    float eps = 1e-6f;
    // programmatic launch: the CTAs set up and load their first states while the previous kernel in
    // the stream runs, and wait for it before reading anything else. Only for a previous kernel that
    // does not write the states (the verify layer's conv step).
    bool dependent = false;
};
int launch_verify_block(const VerifyBlockArgs& a, cudaStream_t s);

// The verify branch of one delta layer that keeps its update vectors (verify_block.cu): the conv
// step over the conv-state window and the T new tokens (ext [B, C, taps + T]; q, k
// repeat-interleaved to the value heads and v, each [B, T, HV, 128] bf16), then the block verify of
// `state` (a programmatic dependent of the conv step) with the output-gated RMSNorm: y [B, T, HV,
// 128] bf16, deltas [B, T, HV, 128] fp32. bf16 throughout, T <= 8, 128-wide heads.
struct VerifyLayerArgs {
    const void* qkv;
    int64_t qkv_sb, qkv_st;
    const void* conv_state;
    const void* conv_w;
    void* ext;
    void* q;
    void* k;
    void* v;
    const float* g;
    const void* beta;
    int beta_dtype;
    const float* state;
    const void* z;
    const void* norm_w;
    void* y;
    float* deltas;
    int64_t B, T;
    int H, HV, taps, K;
    float scale, eps;
};
int launch_verify_layer(const VerifyLayerArgs& a, cudaStream_t s);
// Below this many (row, value head) states the verify layer runs the gated norm in the block's drain
// (a launch saved); from here up the block's per-state chain is the limit and the standalone norm
// after it is faster.
constexpr int64_t kVerifyFusedNormStates = 2048;

struct ChunkArgs {
    const void* q;
    const void* k;
    const void* v;
    const float* g;
    const void* beta;
    int beta_dtype;
    const float* h0;
    float* ht;
    void* o;
    const int32_t* cu_seqlens;
    int64_t B, T, nseq;
    int H, HV;
    int64_t qsb, qst, qsh, ksb, kst, ksh, vsb, vst, vsh;
    float scale;
    void* workspace;
    size_t workspace_bytes;
    GateInputs gates;  // used instead of g and beta when gates.b is set
    // output-gated RMSNorm of o fused into the call (y null: none); z in o's row layout, y may be o
    const void* z;
    const void* norm_w;
    void* y;
    float eps;
};
int launch_chunk(const ChunkArgs& a, cudaStream_t s);
size_t chunk_workspace_bytes(int64_t B, int64_t T, int64_t nseq, bool packed, int64_t HV);

int launch_snapshot_commit(float* state, const float* snapshots, const int64_t* accepted, int64_t B, int64_t T,
                           int64_t HV, cudaStream_t s);

struct DecodeLayerArgs {
    const void* qkv;
    int64_t qkv_sb;
    void* conv_state;
    const void* conv_w;
    const float* g;
    const void* beta;
    float* state;
    const void* z;
    const void* norm_w;
    void* out;
    void* workspace;  // [B, C] bf16: post-conv activations
    int64_t B;
    int H, HV, taps, K;
    float scale, eps;
};
int launch_decode_layer(const DecodeLayerArgs& a, cudaStream_t s);

int launch_conv1d_silu(const void* x, int64_t sxb, int64_t sxt, const void* w, void* y, const int32_t* cu, int64_t B,
                       int64_t T, int64_t C, int K, cudaStream_t s);
// dependent: launched as a programmatic dependent of the previous kernel in the stream (the kernel
// waits for it before its first memory access).
int launch_conv1d_silu_step(const void* x, int64_t sxb, void* state, const void* w, void* y, int64_t B, int64_t C,
                            int taps, int K, cudaStream_t s, bool dependent = false);
int launch_conv_step(const void* state, const void* qkv, int64_t sqb, int64_t sqt, const void* w, void* ext, void* q,
                     void* k, void* v, int64_t B, int64_t T, int taps, int K, int64_t key_dim, int64_t value_dim, int dk,
                     int dv, cudaStream_t s, bool dependent = false);
int launch_conv_state_commit(const void* ext, void* state, const int64_t* accepted, int64_t layers, int64_t B,
                             int64_t C, int taps, int64_t T, int64_t esl, int64_t esb, int64_t ssl, int64_t ssb,
                             cudaStream_t s);
int launch_delta_gates(const void* b, int64_t sb, const void* a, int64_t sa, const void* dt_bias, int dt_f32,
                       const float* rate, const uint8_t* valid, void* beta, float* g, int64_t rows, int HV,
                       cudaStream_t s);
// Decode attention over a KV cache (attention.cu). q: [B, R, H, D]; caches [cache_rows,
// cache_len, Hkv, D]; mask [B, 1, R, L] bf16 additive; o [B, R, H, D] contiguous.
struct AttentionArgs {
    const void* q;
    int64_t qsb, qsr, qsh;
    const void* k;
    int64_t ksb, kss, ksh;
    const void* v;
    int64_t vsb, vss, vsh;
    const void* mask;
    int64_t msb, msr;
    void* o;
    int64_t B, R, H, Hkv, D, L, cache_rows, cache_len;
    float scale;
    void* workspace;
    size_t workspace_bytes;
};
int launch_decode_attention(const AttentionArgs& a, cudaStream_t s);
size_t decode_attention_workspace_bytes(int64_t B, int64_t Hkv, int64_t L, int64_t D);

// Rotary embedding with per-row cos / sin, and the drafter's rotate-into-cache (rotary.cu).
int launch_rotary(const void* x, const float* cs, const float* sn, void* out, int64_t rows, int H, int D, int nf,
                  cudaStream_t s);
struct RotateCacheArgs {
    const void* k;   // [B, K, H, D] contiguous
    const void* v;
    const void* qm;  // [B, M, H, D] with element strides (msb, mst); heads contiguous
    const void* km;
    const void* vm;
    int64_t msb, mst;
    const float* cos_c;  // [B, K, F] fp32 contiguous
    const float* sin_c;
    const float* cos_m;  // [B, M, F]
    const float* sin_m;
    void* k_cache;  // element strides (csb, css); [.., H, D] contiguous
    void* v_cache;
    int64_t csb, css;
    void* q_out;             // [B, M, H, D] contiguous
    const int64_t* rows;     // [B, K] with element strides (rsb, rst)
    int64_t rsb, rst;
    const int64_t* positions;  // [B, K] contiguous
    int64_t tail_start;
    int64_t B;
    int K, M, H, D, nf;
};
int launch_rotate_into_cache(const RotateCacheArgs& a, cudaStream_t s);

// Merged input projection with the causal conv in the epilogue (inproj.cu). x: [T, K] (row
// stride ldx); w: [N, K] (row stride ldw); conv_w: [C, 4]; out: [T, N] (row stride ldo);
// conv_tail: [nseq, C, 4] or null; cu_seqlens: [nseq + 1] or null.
struct InProjArgs {
    const void* x;
    int64_t ldx;
    const void* w;
    int64_t ldw;
    const void* conv_w;
    const int32_t* cu_seqlens;
    void* out;
    int64_t ldo;
    void* conv_tail;
    int64_t T, K, N, C, nseq;
    // fp8 weights (codes non-null): e4m3 codes [N, K] with row stride ldc bytes, one fp32 scale
    // per row, and a workspace of in_proj_fp8_workspace_bytes for the fp16 activation rows
    const void* codes;
    int64_t ldc;
    const float* w_scale;
    void* workspace;
    size_t workspace_bytes;
};
int launch_in_proj_conv(const InProjArgs& a, cudaStream_t s);
size_t in_proj_fp8_workspace_bytes(int64_t T, int64_t K);
size_t in_proj_fp8_pair_workspace_bytes(int64_t T, int64_t K, int64_t N);
// the pair size when the shape runs on CTA pairs on the current device, else the base size
size_t in_proj_fp8_prefill_workspace_bytes(int64_t T, int64_t K, int64_t N, int64_t C);

// Runs a bounded device wait that is meant to run out after `limit_cycles` (probe.cu).
int launch_bounded_wait_probe(int64_t limit_cycles, cudaStream_t s);

int launch_gated_rmsnorm(const void* x, const void* z, const void* w, void* y, int64_t rows, int dim, float eps,
                         cudaStream_t s,
                         bool dependent = false);

}  // namespace gdn
