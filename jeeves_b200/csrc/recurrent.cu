// Gated delta rule in recurrent form on CUDA cores (fp32 state, fp32 math).
//
// Reference semantics: torch_recurrent_gated_delta_rule (model/model.py:221-239), the
// fla in-place decode step it dispatches to (model/fla_inplace.py:17-26) and the advance
// kernel used for rollback (model/fla_inplace.py:29-60).
//
// Work split: one CTA owns a 128 x VS column slice of one (row, value head) state. The
// slice lives in registers for the whole token loop: a row group of VS/4 threads covers
// one state row with 16-byte accesses, so state loads and stores are fully coalesced.
// Per token the CTA needs r = k^T S and p = q^T S (sums over the 128 key rows); each
// warp reduces its rows with shuffles, then one shared-memory round adds the warps.
// With S' = e^g S + k delta^T it follows that q^T S' = e^g p + (q.k) delta, so one
// reduction round per token serves both the delta and the output.

#include "common.cuh"
#include "launch.h"

namespace gdn {

struct RecurrentParams {
    const void* q;
    const void* k;
    const void* v;
    const float* g;
    const void* beta;
    const float* state_in;
    float* state_out;
    float* snapshots;
    void* o;
    const int64_t* steps;
    const int32_t* cu_seqlens;
    int64_t T;
    int HV, rep;
    int64_t qsb, qst, qsh, ksb, kst, ksh, vsb, vst, vsh;
    float scale;
};

template <typename TIn, typename TBeta, int VS, int NT>
__global__ void __launch_bounds__(NT) recurrent_kernel(const RecurrentParams p) {
    constexpr int COLG = VS / 4;   // threads along one state row
    constexpr int NW = NT / 32;
    constexpr int ROWG = NT / COLG;
    constexpr int RPT = kHeadDim / ROWG;  // state rows per thread
    static_assert(COLG <= 32 && 32 % COLG == 0 && RPT % 4 == 0, "bad tile");
    __shared__ float4 red[2][2][NW][COLG];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cg = tid % COLG, rg = tid / COLG;
    const int row0 = rg * RPT;
    const int hv = blockIdx.y;
    const int64_t n = blockIdx.z;
    const int h = hv / p.rep;
    const int col = blockIdx.x * VS + cg * 4;

    int64_t bos = 0, len = p.T, brow = n;
    if (p.cu_seqlens) {
        bos = p.cu_seqlens[n];
        len = p.cu_seqlens[n + 1] - bos;
        brow = 0;
    }
    int64_t nsteps = len;
    if (p.steps) {
        const int64_t s = p.steps[n];
        nsteps = s < 0 ? 0 : (s > len ? len : s);
        if (nsteps == 0) return;  // advancing by 0 tokens leaves the state untouched
    }

    const int64_t tile = (n * p.HV + hv) * (int64_t)(kHeadDim * kHeadDim);
    float4 S[RPT];
    if (p.state_in) {
        const float* src = p.state_in + tile + (int64_t)row0 * kHeadDim + col;
#pragma unroll
        for (int r = 0; r < RPT; ++r) S[r] = ldg_stream(reinterpret_cast<const float4*>(src + r * kHeadDim));
    } else {
#pragma unroll
        for (int r = 0; r < RPT; ++r) S[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    const bool outputs = p.o != nullptr;
    const TIn* kbase = static_cast<const TIn*>(p.k) + brow * p.ksb + h * p.ksh;
    const TIn* qbase = static_cast<const TIn*>(p.q) + brow * p.qsb + h * p.qsh;
    const TIn* vbase = static_cast<const TIn*>(p.v) + brow * p.vsb + hv * p.vsh;
    const TBeta* beta = static_cast<const TBeta*>(p.beta);

    int buf = 0;
    for (int64_t t = 0; t < nsteps; ++t) {
        const int64_t tok = bos + t;
        const float4 kl = load4(kbase + tok * p.kst + 4 * lane);
        float4 ql = make_float4(0.f, 0.f, 0.f, 0.f);
        if (outputs) ql = load4(qbase + tok * p.qst + 4 * lane);
        const float4 vv = load4(vbase + tok * p.vst + col);
        const int64_t gi = (brow * p.T + tok) * p.HV + hv;
        const float decay = expf(p.g[gi]);
        const float bt = to_f32(beta[gi]);

        const float kk = warp_sum(kl.x * kl.x + kl.y * kl.y + kl.z * kl.z + kl.w * kl.w);
        const float rk = rsqrtf(kk + 1e-6f);
        float rq = 0.f, qk = 0.f;
        if (outputs) {
            const float qq = warp_sum(ql.x * ql.x + ql.y * ql.y + ql.z * ql.z + ql.w * ql.w);
            qk = warp_sum(ql.x * kl.x + ql.y * kl.y + ql.z * kl.z + ql.w * kl.w);
            rq = rsqrtf(qq + 1e-6f) * p.scale;
        }

        // Partial sums over this thread's rows. Row i of k sits in lane i/4, element i%4;
        // RPT is a multiple of 4, so the element index is the same across the warp.
        float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            const int src = (row0 + r) >> 2;
            const float kr = (r & 3) == 0 ? kl.x : (r & 3) == 1 ? kl.y : (r & 3) == 2 ? kl.z : kl.w;
            const float ki = __shfl_sync(0xffffffffu, kr, src) * rk;
            pk.x += ki * S[r].x; pk.y += ki * S[r].y; pk.z += ki * S[r].z; pk.w += ki * S[r].w;
            if (outputs) {
                const float qr = (r & 3) == 0 ? ql.x : (r & 3) == 1 ? ql.y : (r & 3) == 2 ? ql.z : ql.w;
                const float qi = __shfl_sync(0xffffffffu, qr, src) * rq;
                pq.x += qi * S[r].x; pq.y += qi * S[r].y; pq.z += qi * S[r].z; pq.w += qi * S[r].w;
            }
        }
#pragma unroll
        for (int off = COLG; off < 32; off <<= 1) {
            pk.x += __shfl_xor_sync(0xffffffffu, pk.x, off);
            pk.y += __shfl_xor_sync(0xffffffffu, pk.y, off);
            pk.z += __shfl_xor_sync(0xffffffffu, pk.z, off);
            pk.w += __shfl_xor_sync(0xffffffffu, pk.w, off);
            if (outputs) {
                pq.x += __shfl_xor_sync(0xffffffffu, pq.x, off);
                pq.y += __shfl_xor_sync(0xffffffffu, pq.y, off);
                pq.z += __shfl_xor_sync(0xffffffffu, pq.z, off);
                pq.w += __shfl_xor_sync(0xffffffffu, pq.w, off);
            }
        }
        if (lane < COLG) {
            red[buf][0][warp][cg] = pk;
            if (outputs) red[buf][1][warp][cg] = pq;
        }
        __syncthreads();
        float4 rs = red[buf][0][0][cg];
#pragma unroll
        for (int w = 1; w < NW; ++w) {
            const float4 x = red[buf][0][w][cg];
            rs.x += x.x; rs.y += x.y; rs.z += x.z; rs.w += x.w;
        }
        float4 delta;
        delta.x = bt * (vv.x - decay * rs.x);
        delta.y = bt * (vv.y - decay * rs.y);
        delta.z = bt * (vv.z - decay * rs.z);
        delta.w = bt * (vv.w - decay * rs.w);
        if (outputs && rg == 0) {
            float4 ps = red[buf][1][0][cg];
#pragma unroll
            for (int w = 1; w < NW; ++w) {
                const float4 x = red[buf][1][w][cg];
                ps.x += x.x; ps.y += x.y; ps.z += x.z; ps.w += x.w;
            }
            const float qkn = qk * rk * rq;
            float4 out;
            out.x = decay * ps.x + qkn * delta.x;
            out.y = decay * ps.y + qkn * delta.y;
            out.z = decay * ps.z + qkn * delta.z;
            out.w = decay * ps.w + qkn * delta.w;
            store4(static_cast<TIn*>(p.o) + gi * kHeadDim + col, out);
        }
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            const int src = (row0 + r) >> 2;
            const float kr = (r & 3) == 0 ? kl.x : (r & 3) == 1 ? kl.y : (r & 3) == 2 ? kl.z : kl.w;
            const float ki = __shfl_sync(0xffffffffu, kr, src) * rk;
            S[r].x = decay * S[r].x + ki * delta.x;
            S[r].y = decay * S[r].y + ki * delta.y;
            S[r].z = decay * S[r].z + ki * delta.z;
            S[r].w = decay * S[r].w + ki * delta.w;
        }
        if (p.snapshots) {
            float* dst = p.snapshots + ((brow * p.T + tok) * p.HV + hv) * (int64_t)(kHeadDim * kHeadDim) +
                         (int64_t)row0 * kHeadDim + col;
#pragma unroll
            for (int r = 0; r < RPT; ++r) stg_stream(reinterpret_cast<float4*>(dst + r * kHeadDim), S[r]);
        }
        buf ^= 1;
    }
    if (p.state_out) {
        float* dst = p.state_out + tile + (int64_t)row0 * kHeadDim + col;
#pragma unroll
        for (int r = 0; r < RPT; ++r) stg_stream(reinterpret_cast<float4*>(dst + r * kHeadDim), S[r]);
    }
}

template <typename TIn, typename TBeta>
static int dispatch_recurrent(const RecurrentParams& p, int64_t rows, cudaStream_t s) {
    // Small grids split the value columns finer so that more SMs share the work.
    const int64_t heads = rows * p.HV;
    if (heads >= 2048) {
        dim3 grid(kHeadDim / 32, p.HV, (unsigned)rows);
        recurrent_kernel<TIn, TBeta, 32, 128><<<grid, 128, 0, s>>>(p);
    } else {
        dim3 grid(kHeadDim / 16, p.HV, (unsigned)rows);
        recurrent_kernel<TIn, TBeta, 16, 64><<<grid, 64, 0, s>>>(p);
    }
    return launch_status();
}

int launch_recurrent(const RecurrentArgs& a, cudaStream_t s) {
    RecurrentParams p;
    p.q = a.q; p.k = a.k; p.v = a.v; p.g = a.g; p.beta = a.beta;
    p.state_in = a.state_in; p.state_out = a.state_out; p.snapshots = a.snapshots; p.o = a.o;
    p.steps = a.steps; p.cu_seqlens = a.cu_seqlens;
    p.T = a.T; p.HV = a.HV; p.rep = a.HV / a.H;
    p.qsb = a.qsb; p.qst = a.qst; p.qsh = a.qsh;
    p.ksb = a.ksb; p.kst = a.kst; p.ksh = a.ksh;
    p.vsb = a.vsb; p.vst = a.vst; p.vsh = a.vsh;
    p.scale = a.scale;
    if (a.rows == 0) return GDN_OK;
    if (a.qkv_dtype == GDN_BF16) {
        return a.beta_dtype == GDN_BF16 ? dispatch_recurrent<bf16, bf16>(p, a.rows, s)
                                        : dispatch_recurrent<bf16, float>(p, a.rows, s);
    }
    return a.beta_dtype == GDN_BF16 ? dispatch_recurrent<float, bf16>(p, a.rows, s)
                                    : dispatch_recurrent<float, float>(p, a.rows, s);
}

// Rollback by snapshot: state[b] <- snapshots[b, accepted[b] - 1].
__global__ void snapshot_commit_kernel(float* __restrict__ state, const float* __restrict__ snaps,
                                       const int64_t* __restrict__ accepted, int64_t T, int HV) {
    const int64_t b = blockIdx.z;
    const int64_t j = accepted[b];
    if (j <= 0) return;
    const int64_t t = (j > T ? T : j) - 1;
    const int hv = blockIdx.y;
    constexpr int64_t tile = kHeadDim * kHeadDim;
    const int64_t part = (int64_t)blockIdx.x * blockDim.x * 4 + threadIdx.x * 4;
    const float* src = snaps + ((b * T + t) * HV + hv) * tile + part;
    float* dst = state + (b * HV + hv) * tile + part;
    stg_stream(reinterpret_cast<float4*>(dst), ldg_stream(reinterpret_cast<const float4*>(src)));
}

int launch_snapshot_commit(float* state, const float* snapshots, const int64_t* accepted, int64_t B, int64_t T,
                           int64_t HV, cudaStream_t s) {
    if (B == 0) return GDN_OK;
    constexpr int threads = 256;
    dim3 grid(kHeadDim * kHeadDim / (threads * 4), (unsigned)HV, (unsigned)B);
    snapshot_commit_kernel<<<grid, threads, 0, s>>>(state, snapshots, accepted, T, (int)HV);
    return launch_status();
}

// ---------------------------------------------------------------------------------------
// Fused decode layer: conv step (+SiLU) over the pre-conv token, q/k L2 norm, gated delta
// rule step on the state in place, output-gated RMSNorm. One CTA per (row, value head)
// owns the full 128 x 128 state so that the norm over the head's 128 outputs stays in
// one warp. The conv state is only read here; launch_conv_state_shift rolls it forward
// afterwards (an in-place update inside this kernel would race with the other value
// heads that read the same q/k channels).
// ---------------------------------------------------------------------------------------

struct DecodeParams {
    const bf16* qkv;
    int64_t qkv_sb;
    const bf16* conv_state;
    const bf16* conv_w;
    const float* g;
    const bf16* beta;
    float* state;
    const bf16* z;
    const bf16* norm_w;
    bf16* out;
    int H, HV, rep, taps, K;
    int64_t C;
    float scale, eps;
};

// Conv + SiLU of one channel for the decode token, rounded like the eager step
// (model/model.py:207-214): bf16 products, fp32 sum, bf16, silu in fp32, bf16.
__device__ __forceinline__ float conv_token(const DecodeParams& p, int64_t b, int64_t c) {
    const bf16* st = p.conv_state + (b * p.C + c) * p.taps;
    const bf16* w = p.conv_w + c * p.K;
    float acc = 0.f;
    for (int i = 0; i < p.K; ++i) {
        // window = last K of (state ++ x): entry i is state[taps - K + 1 + i] or x for i = K-1
        const float xi = (i == p.K - 1) ? to_f32(p.qkv[b * p.qkv_sb + c]) : to_f32(st[p.taps - p.K + 1 + i]);
        acc = __fadd_rn(acc, round_bf16(__fmul_rn(xi, to_f32(w[i]))));
    }
    return round_bf16(silu_f32(round_bf16(acc)));
}

template <int NT>
__global__ void __launch_bounds__(NT) decode_layer_kernel(const DecodeParams p) {
    constexpr int VS = kHeadDim, COLG = VS / 4, NW = NT / 32, ROWG = NT / COLG, RPT = kHeadDim / ROWG;
    __shared__ float4 red[2][NW][COLG];
    __shared__ float kq[2][kHeadDim];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cg = tid % COLG, rg = tid / COLG, row0 = rg * RPT, col = cg * 4;
    const int hv = blockIdx.x;
    const int64_t b = blockIdx.y;
    const int h = hv / p.rep;
    const int64_t tile = (b * p.HV + hv) * (int64_t)(kHeadDim * kHeadDim);

    float4 S[RPT];
    const float* src = p.state + tile + (int64_t)row0 * kHeadDim + col;
#pragma unroll
    for (int r = 0; r < RPT; ++r) S[r] = ldg_stream(reinterpret_cast<const float4*>(src + r * kHeadDim));

    // conv outputs: q and k of key head h (256 channels), v of value head hv (128)
    const int64_t key_dim = (int64_t)p.H * kHeadDim;
    if (tid < 2 * kHeadDim) {
        const int part = tid / kHeadDim, d = tid % kHeadDim;
        kq[part][d] = conv_token(p, b, part * key_dim + (int64_t)h * kHeadDim + d);
    }
    float4 vv;
    {
        const int64_t c0 = 2 * key_dim + (int64_t)hv * kHeadDim + col;
        vv.x = conv_token(p, b, c0);
        vv.y = conv_token(p, b, c0 + 1);
        vv.z = conv_token(p, b, c0 + 2);
        vv.w = conv_token(p, b, c0 + 3);
    }
    __syncthreads();
    const float4 ql = *reinterpret_cast<const float4*>(&kq[0][4 * lane]);
    const float4 kl = *reinterpret_cast<const float4*>(&kq[1][4 * lane]);
    const float rk = rsqrtf(warp_sum(kl.x * kl.x + kl.y * kl.y + kl.z * kl.z + kl.w * kl.w) + 1e-6f);
    const float rq = rsqrtf(warp_sum(ql.x * ql.x + ql.y * ql.y + ql.z * ql.z + ql.w * ql.w) + 1e-6f) * p.scale;
    const float qk = warp_sum(ql.x * kl.x + ql.y * kl.y + ql.z * kl.z + ql.w * kl.w);
    const int64_t gi = b * p.HV + hv;
    const float decay = expf(p.g[gi]);
    const float bt = to_f32(p.beta[gi]);

    float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const float ki = kq[1][row0 + r] * rk;
        const float qi = kq[0][row0 + r] * rq;
        pk.x += ki * S[r].x; pk.y += ki * S[r].y; pk.z += ki * S[r].z; pk.w += ki * S[r].w;
        pq.x += qi * S[r].x; pq.y += qi * S[r].y; pq.z += qi * S[r].z; pq.w += qi * S[r].w;
    }
    if (lane < COLG || COLG == 32) {
        red[0][warp][cg] = pk;
        red[1][warp][cg] = pq;
    }
    __syncthreads();
    float4 rs = red[0][0][cg];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
        const float4 x = red[0][w][cg];
        rs.x += x.x; rs.y += x.y; rs.z += x.z; rs.w += x.w;
    }
    float4 delta;
    delta.x = bt * (vv.x - decay * rs.x);
    delta.y = bt * (vv.y - decay * rs.y);
    delta.z = bt * (vv.z - decay * rs.z);
    delta.w = bt * (vv.w - decay * rs.w);
    if (warp == 0) {
        float4 ps = red[1][0][cg];
#pragma unroll
        for (int w = 1; w < NW; ++w) {
            const float4 x = red[1][w][cg];
            ps.x += x.x; ps.y += x.y; ps.z += x.z; ps.w += x.w;
        }
        const float qkn = qk * rk * rq;
        float o[4] = {decay * ps.x + qkn * delta.x, decay * ps.y + qkn * delta.y, decay * ps.z + qkn * delta.z,
                      decay * ps.w + qkn * delta.w};
        // The reference rounds o to bf16 before the norm (o.to(q.dtype), model/model.py:239).
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[i] = round_bf16(o[i]);
            sq += o[i] * o[i];
        }
        const float inv = inv_sqrt_rn(warp_sum(sq) * (1.0f / kHeadDim) + p.eps);
        const float4 zz = load4(p.z + gi * kHeadDim + col);
        const float4 ww = load4(p.norm_w + col);
        const float zv[4] = {zz.x, zz.y, zz.z, zz.w}, wv[4] = {ww.x, ww.y, ww.z, ww.w};
        float4 y;
        float* yv = &y.x;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float normed = round_bf16(o[i] * inv);
            const float weighted = round_bf16(wv[i] * normed);
            yv[i] = weighted * silu_f32(zv[i]);
        }
        store4(p.out + gi * kHeadDim + col, y);
    }
    float* dst = p.state + tile + (int64_t)row0 * kHeadDim + col;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const float ki = kq[1][row0 + r] * rk;
        float4 x;
        x.x = decay * S[r].x + ki * delta.x;
        x.y = decay * S[r].y + ki * delta.y;
        x.z = decay * S[r].z + ki * delta.z;
        x.w = decay * S[r].w + ki * delta.w;
        stg_stream(reinterpret_cast<float4*>(dst + r * kHeadDim), x);
    }
}

int launch_decode_layer(const DecodeLayerArgs& a, cudaStream_t s) {
    if (a.B == 0) return GDN_OK;
    DecodeParams p;
    p.qkv = static_cast<const bf16*>(a.qkv);
    p.qkv_sb = a.qkv_sb;
    p.conv_state = static_cast<const bf16*>(a.conv_state);
    p.conv_w = static_cast<const bf16*>(a.conv_w);
    p.g = a.g;
    p.beta = static_cast<const bf16*>(a.beta);
    p.state = a.state;
    p.z = static_cast<const bf16*>(a.z);
    p.norm_w = static_cast<const bf16*>(a.norm_w);
    p.out = static_cast<bf16*>(a.out);
    p.H = a.H; p.HV = a.HV; p.rep = a.HV / a.H; p.taps = a.taps; p.K = a.K;
    p.C = 2 * (int64_t)a.H * kHeadDim + (int64_t)a.HV * kHeadDim;
    p.scale = a.scale; p.eps = a.eps;
    dim3 grid((unsigned)a.HV, (unsigned)a.B);
    decode_layer_kernel<256><<<grid, 256, 0, s>>>(p);
    int st = launch_status();
    if (st != GDN_OK) return st;
    return launch_conv_state_shift(a.qkv, a.qkv_sb, a.conv_state, a.B, p.C, a.taps, s);
}

}  // namespace gdn
