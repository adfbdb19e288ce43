// Causal depthwise conv1d + SiLU kernels around the gated delta rule.
//
// Rounding follows the reference's eager path: the prefill conv and the verify conv use
// F.conv1d (an fp32 sum of fp32 products in tap order, without fused multiply-add,
// rounded once to bf16;
// model/model.py:199-204, :324-332) and the decode step multiplies in bf16 before an
// fp32 sum (model/model.py:207-214). SiLU is x / (1 + exp(-x)) in fp32 on the bf16 value.

#include "common.cuh"
#include "launch.h"

namespace gdn {

constexpr int kMaxTaps = 8;

// Prefill: one thread per (8 channels, run of kConvRun tokens). It loads the run plus the
// K - 1 tokens before it with 16-byte loads into registers (neighbouring runs re-read only
// that halo) and writes 16 bytes per token. With cu_seqlens a tap before the start of the
// token's sequence reads as zero, exactly like the zero padding of a per-sequence conv.
constexpr int kConvRun = 4;

__device__ __forceinline__ void unpack8(const uint4& raw, float* out) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void load8(const bf16* p, float* out) { unpack8(*reinterpret_cast<const uint4*>(p), out); }

__device__ __forceinline__ void store8(bf16* p, const float* v) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = raw;
}

template <int K, bool PACKED>
__global__ void __launch_bounds__(128) conv1d_silu_kernel(const bf16* __restrict__ x, int64_t sxb, int64_t sxt,
                                                          const bf16* __restrict__ w, bf16* __restrict__ y,
                                                          const int32_t* __restrict__ cu, int nseq, int64_t T,
                                                          int64_t C) {
    const int64_t c8 = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 8;
    if (c8 >= C) return;
    const int64_t t0 = (int64_t)blockIdx.x * kConvRun;  // runs on x: up to 2^31 - 1
    const int64_t b = blockIdx.z;
    constexpr int R = kConvRun + K - 1;
    uint4 raw[R];
    const bf16* xb = x + b * sxb + c8;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t tt = t0 - (K - 1) + r;
        raw[r] = (tt >= 0 && tt < T) ? __ldg(reinterpret_cast<const uint4*>(xb + tt * sxt)) : make_uint4(0, 0, 0, 0);
    }
    bf16 wr[8 * K];  // channel j's taps at j * K
    {
        const uint4* wsrc = reinterpret_cast<const uint4*>(w + c8 * K);
#pragma unroll
        for (int i = 0; i < K; ++i) reinterpret_cast<uint4*>(wr)[i] = __ldg(wsrc + i);
    }
    // With cu_seqlens: the start of each token's sequence, and whether a window reaches before it.
    int64_t seq_start[kConvRun];
    bool edge = false;
    if (PACKED) {
        int lo = 0, hi = nseq;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (cu[mid] <= t0) lo = mid;
            else hi = mid;
        }
#pragma unroll
        for (int j = 0; j < kConvRun; ++j) {
            const int64_t t = t0 + j;
            while (lo + 1 < nseq && cu[lo + 1] <= t) ++lo;
            seq_start[j] = cu[lo];
            edge |= t < T && t - (K - 1) < seq_start[j];
        }
    }
    bf16* yb = y + (b * T + t0) * C + c8;
    if (!edge) {
        // Every window lies inside its sequence. Channel pairs (2p, 2p + 1) one after the other:
        // the pair's inputs are widened once, its sums run in packed lanes (products rounded,
        // then added in tap order from zero), and its outputs are packed back to bf16.
        uint32_t packed[kConvRun][4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            f32x2 w2[K], xv[R];
#pragma unroll
            for (int i = 0; i < K; ++i) w2[i] = pack2(to_f32(wr[2 * p * K + i]), to_f32(wr[(2 * p + 1) * K + i]));
#pragma unroll
            for (int r = 0; r < R; ++r)
                xv[r] = bf2_to_f2(p == 0 ? raw[r].x : p == 1 ? raw[r].y : p == 2 ? raw[r].z : raw[r].w);
            float pre[2 * kConvRun], out[2 * kConvRun];
            static_assert(2 * kConvRun == 8, "silu8 takes one pair of channels over the run");
#pragma unroll
            for (int j = 0; j < kConvRun; ++j) {
                f32x2 acc = pack2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < K; ++i) acc = add2(acc, mul2(w2[i], xv[j + i]));
                const float2 r2 = unpack2(round_bf16x2(acc));
                pre[2 * j] = r2.x;
                pre[2 * j + 1] = r2.y;
            }
            silu8(pre, out);
#pragma unroll
            for (int j = 0; j < kConvRun; ++j) packed[j][p] = f2_to_bf2(pack2(out[2 * j], out[2 * j + 1]));
        }
#pragma unroll
        for (int j = 0; j < kConvRun; ++j)
            if (t0 + j < T)
                *reinterpret_cast<uint4*>(yb + j * C) = make_uint4(packed[j][0], packed[j][1], packed[j][2], packed[j][3]);
        return;
    }
    // A window that reaches before the start of its token's sequence: those taps read as zero.
#pragma unroll
    for (int j = 0; j < kConvRun; ++j) {
        const int64_t t = t0 + j;
        if (t >= T) break;
        float win[K][8];
#pragma unroll
        for (int i = 0; i < K; ++i) {
            if (t - (K - 1) + i >= seq_start[j]) unpack8(raw[j + i], win[i]);
            else
#pragma unroll
                for (int q = 0; q < 8; ++q) win[i][q] = 0.f;
        }
        float pre[8], out[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < K; ++i) acc = __fadd_rn(acc, __fmul_rn(to_f32(wr[q * K + i]), win[i][q]));
            pre[q] = round_bf16(acc);
        }
        silu8(pre, out);
        store8(yb + j * C, out);
    }
}

int launch_conv1d_silu(const void* x, int64_t sxb, int64_t sxt, const void* w, void* y, const int32_t* cu, int64_t B,
                       int64_t T, int64_t C, int K, cudaStream_t s) {
    if (B == 0 || T == 0) return GDN_OK;
    constexpr int threads = 128;
    const int nseq = cu ? (int)B : 0;  // with cu_seqlens the caller passes the sequence count as B
    dim3 grid((unsigned)((T + kConvRun - 1) / kConvRun), (unsigned)((C / 8 + threads - 1) / threads), cu ? 1u : (unsigned)B);
    auto xp = static_cast<const bf16*>(x);
    auto wp = static_cast<const bf16*>(w);
    auto yp = static_cast<bf16*>(y);
#define GDN_CONV_CASE(KK)                                                                               \
    case KK:                                                                                            \
        if (cu) conv1d_silu_kernel<KK, true><<<grid, threads, 0, s>>>(xp, sxb, sxt, wp, yp, cu, nseq, T, C); \
        else conv1d_silu_kernel<KK, false><<<grid, threads, 0, s>>>(xp, sxb, sxt, wp, yp, cu, nseq, T, C);  \
        break;
    switch (K) {
        GDN_CONV_CASE(2)
        GDN_CONV_CASE(3)
        GDN_CONV_CASE(4)
        default: return GDN_ERR_UNSUPPORTED;
    }
#undef GDN_CONV_CASE
    return launch_status();
}

// Launches `kernel` on `s`; with `dependent` as a programmatic dependent of the previous kernel in
// the stream (the kernels launched so wait for it before their first memory access).
template <typename... Params, typename... Args>
static int launch_conv_kernel(void (*kernel)(Params...), dim3 grid, int threads, bool dependent, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...) == cudaSuccess ? launch_status()
                                                                                        : GDN_ERR_LAUNCH;
}

// Decode step: y = silu(bf16(sum_i bf16(w_i * window_i))); the state keeps the last `taps`
// inputs. One thread owns 8 consecutive channels, so every access is a 16-byte vector: the
// channels' conv states are 8 * taps contiguous bf16 values, and x, y are 8 contiguous bf16.
template <int TAPS, int K>
__global__ void conv1d_silu_step_kernel(const bf16* __restrict__ x, int64_t sxb, bf16* __restrict__ state,
                                        const bf16* __restrict__ w, bf16* __restrict__ y, int64_t B, int64_t C) {
    // Launched as a programmatic dependent of the previous layer's last kernel: wait for it before
    // any memory access, and only then let the recurrent step start loading its state (so that no
    // kernel before this one can still be writing that state).
    pdl_wait();
    pdl_launch_dependents();
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // group of 8 channels
    const int64_t groups = C / 8;
    if (idx >= B * groups) return;
    const int64_t b = idx / groups, c8 = (idx % groups) * 8;
    constexpr int N = 8 * TAPS;  // bf16 state values of 8 channels
    constexpr int NW = 8 * K;    // bf16 weights of 8 channels
    bf16 st[N], wt[NW];
    {
        uint4* st_vec = reinterpret_cast<uint4*>(st);
        const uint4* src = reinterpret_cast<const uint4*>(state + (b * C + c8) * TAPS);
#pragma unroll
        for (int i = 0; i < N / 8; ++i) st_vec[i] = src[i];
        uint4* w_vec = reinterpret_cast<uint4*>(wt);
        const uint4* wsrc = reinterpret_cast<const uint4*>(w + c8 * K);
#pragma unroll
        for (int i = 0; i < NW / 8; ++i) w_vec[i] = __ldg(wsrc + i);
    }
    float xv[8];
    load8(x + b * sxb + c8, xv);
    float out[8];
    bf16 nst[N];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float win[TAPS + 1];
#pragma unroll
        for (int i = 0; i < TAPS; ++i) win[i] = to_f32(st[j * TAPS + i]);
        win[TAPS] = xv[j];
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < K; ++i)
            acc = __fadd_rn(acc, round_bf16(__fmul_rn(to_f32(wt[j * K + i]), win[TAPS + 1 - K + i])));
        out[j] = silu_f32(round_bf16(acc));
#pragma unroll
        for (int i = 0; i < TAPS; ++i) nst[j * TAPS + i] = __float2bfloat16_rn(win[i + 1]);
    }
    store8(y + b * C + c8, out);
    uint4* dst = reinterpret_cast<uint4*>(state + (b * C + c8) * TAPS);
    const uint4* nst_vec = reinterpret_cast<const uint4*>(nst);
#pragma unroll
    for (int i = 0; i < N / 8; ++i) dst[i] = nst_vec[i];
}

template <int TAPS>
static int conv_step_taps(const bf16* x, int64_t sxb, bf16* st, const bf16* w, bf16* y, int64_t B, int64_t C, int K,
                          unsigned blocks, int threads, cudaStream_t s, bool dependent) {
    switch (K) {
        case 2:
            return launch_conv_kernel(conv1d_silu_step_kernel<TAPS, 2>, blocks, threads, dependent, s, x, sxb, st, w, y,
                                      B, C);
        case 3:
            return launch_conv_kernel(conv1d_silu_step_kernel<TAPS, 3>, blocks, threads, dependent, s, x, sxb, st, w, y,
                                      B, C);
        case 4:
            if (TAPS < 3) return GDN_ERR_SHAPE;
            return launch_conv_kernel(conv1d_silu_step_kernel<TAPS, (TAPS >= 3 ? 4 : 3)>, blocks, threads, dependent, s,
                                      x, sxb, st, w, y, B, C);
        default: return GDN_ERR_UNSUPPORTED;
    }
}

int launch_conv1d_silu_step(const void* x, int64_t sxb, void* state, const void* w, void* y, int64_t B, int64_t C,
                            int taps, int K, cudaStream_t s, bool dependent) {
    if (B * C == 0) return GDN_OK;
    if (C % 8 || K > taps + 1 || K < 2) return GDN_ERR_SHAPE;
    constexpr int threads = 256;
    const unsigned blocks = (unsigned)((B * (C / 8) + threads - 1) / threads);
    auto xp = static_cast<const bf16*>(x);
    auto sp = static_cast<bf16*>(state);
    auto wp = static_cast<const bf16*>(w);
    auto yp = static_cast<bf16*>(y);
    switch (taps) {
        case 2: return conv_step_taps<2>(xp, sxb, sp, wp, yp, B, C, K, blocks, threads, s, dependent);
        case 3: return conv_step_taps<3>(xp, sxb, sp, wp, yp, B, C, K, blocks, threads, s, dependent);
        case 4: return conv_step_taps<4>(xp, sxb, sp, wp, yp, B, C, K, blocks, threads, s, dependent);
        default: return GDN_ERR_UNSUPPORTED;
    }
}

// Verify conv: ext = state ++ qkv^T; output t = silu(bf16(sum_i w_i ext[t + taps - K + 1 + i]))
// split into q, k (repeat-interleaved over the value heads) and v. One thread per channel.
__global__ void conv_step_kernel(const bf16* __restrict__ state, const bf16* __restrict__ qkv, int64_t sqb, int64_t sqt,
                                 const bf16* __restrict__ w, bf16* __restrict__ ext, bf16* __restrict__ q,
                                 bf16* __restrict__ k, bf16* __restrict__ v, int64_t T, int taps, int K, int64_t C,
                                 int64_t key_dim, int64_t value_dim, int dk, int dv, int rep) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int64_t b = blockIdx.y;
    const int64_t L = taps + T;
    bf16* e = ext + (b * C + c) * L;
    const bf16* st = state + (b * C + c) * taps;
    for (int i = 0; i < taps; ++i) e[i] = st[i];
    for (int64_t t = 0; t < T; ++t) e[taps + t] = qkv[b * sqb + t * sqt + c];
    float wt[kMaxTaps];
    for (int i = 0; i < K; ++i) wt[i] = to_f32(w[c * K + i]);
    const int64_t k_heads = key_dim / dk, v_heads = value_dim / dv;
    for (int64_t t = 0; t < T; ++t) {
        float acc = 0.f;
        for (int i = 0; i < K; ++i) {
            const int64_t col = t + taps - K + 1 + i;
            const float xv = col < taps ? to_f32(st[col]) : to_f32(qkv[b * sqb + (col - taps) * sqt + c]);
            acc = __fadd_rn(acc, __fmul_rn(wt[i], xv));
        }
        const bf16 yv = __float2bfloat16_rn(silu_f32(round_bf16(acc)));
        if (c < 2 * key_dim) {
            const int64_t kc = c < key_dim ? c : c - key_dim;
            const int64_t head = kc / dk, d = kc % dk;
            bf16* dst = c < key_dim ? q : k;
            for (int r = 0; r < rep; ++r) dst[((b * T + t) * v_heads + head * rep + r) * dk + d] = yv;
        } else {
            v[(b * T + t) * value_dim + (c - 2 * key_dim)] = yv;
        }
    }
    (void)k_heads;
}

// The same conv with 16-byte accesses: one thread per (row, 8 consecutive channels), for the
// engine's shapes (K = 4 taps of weight, L = taps + T ext columns known at compile time). The 8
// channels' ext rows are one contiguous block of 8 L values: the state block and the T token
// vectors are loaded with 16-byte loads, the block is stored with 16-byte stores, and each token's
// 8 outputs go out as one 16-byte store (per repeated head for q and k). Same arithmetic as above.
// (One thread per token as well, the window shared through L2, was slower at 16 to 128 rows.)
template <int TAPS, int T>
__global__ void conv_step_vec_kernel(const bf16* __restrict__ state, const bf16* __restrict__ qkv, int64_t sqb,
                                     int64_t sqt, const bf16* __restrict__ w, bf16* __restrict__ ext,
                                     bf16* __restrict__ q, bf16* __restrict__ k, bf16* __restrict__ v, int64_t B,
                                     int64_t C, int64_t key_dim, int64_t value_dim, int dk, int rep) {
    constexpr int K = 4, L = TAPS + T;
    static_assert(TAPS >= K - 1 && TAPS <= 8, "the window covers every tap");
    // When launched as a programmatic dependent, wait for the previous kernel before any memory
    // access; then a block verify that follows as this kernel's dependent may set up and load its
    // states (which no kernel before this one can still be writing).
    pdl_wait();
    pdl_launch_dependents();
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t groups = C / 8;
    if (idx >= B * groups) return;
    const int64_t b = idx / groups, c8 = (idx % groups) * 8;
    // the ext block: value j of channel c at e[c * L + j]
    bf16 e[8 * L];
    {
        bf16 st[8 * TAPS];  // 8 channels x TAPS, channel-major as stored
        const uint4* src = reinterpret_cast<const uint4*>(state + (b * C + c8) * TAPS);
#pragma unroll
        for (int i = 0; i < TAPS; ++i) reinterpret_cast<uint4*>(st)[i] = src[i];
#pragma unroll
        for (int c = 0; c < 8; ++c)
#pragma unroll
            for (int j = 0; j < TAPS; ++j) e[c * L + j] = st[c * TAPS + j];
#pragma unroll
        for (int t = 0; t < T; ++t) {
            uint4 raw = *reinterpret_cast<const uint4*>(qkv + b * sqb + (int64_t)t * sqt + c8);
            const bf16* x = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
            for (int c = 0; c < 8; ++c) e[c * L + TAPS + t] = x[c];
        }
    }
    uint4* edst = reinterpret_cast<uint4*>(ext + (b * C + c8) * L);
#pragma unroll
    for (int i = 0; i < L; ++i) edst[i] = reinterpret_cast<const uint4*>(e)[i];
    // channel pairs (2p, 2p + 1) in packed lanes: the window's values and the taps' weights
    f32x2 w2[4][K], x2[L][4];
    {
        bf16 wr[8 * K];
        const uint4* wsrc = reinterpret_cast<const uint4*>(w + c8 * K);
#pragma unroll
        for (int i = 0; i < K; ++i) reinterpret_cast<uint4*>(wr)[i] = __ldg(wsrc + i);
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int i = 0; i < K; ++i) w2[p][i] = pack2(to_f32(wr[2 * p * K + i]), to_f32(wr[(2 * p + 1) * K + i]));
#pragma unroll
        for (int j = 0; j < L; ++j)
#pragma unroll
            for (int p = 0; p < 4; ++p) x2[j][p] = pack2(to_f32(e[2 * p * L + j]), to_f32(e[(2 * p + 1) * L + j]));
    }
    bf16* dst;
    int64_t head_stride = 0, base;
    const int64_t v_heads = value_dim / dk;
    if (c8 < 2 * key_dim) {
        const int64_t kc = c8 < key_dim ? c8 : c8 - key_dim;
        dst = c8 < key_dim ? q : k;
        base = ((kc / dk) * rep) * dk + kc % dk;
        head_stride = dk;
    } else {
        dst = v;
        base = c8 - 2 * key_dim;
    }
    const int64_t tok_stride = v_heads * dk;
#pragma unroll
    for (int t = 0; t < T; ++t) {
        // products rounded, then added in tap order from zero (two channels a packed instruction),
        // rounded to bf16, SiLU in fp32 (silu8: the scalar formula's bits)
        float pre[8], sil[8];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            f32x2 acc = pack2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < K; ++i) acc = add2(acc, mul2(w2[p][i], x2[t + TAPS - K + 1 + i][p]));
            const float2 r2 = unpack2(round_bf16x2(acc));
            pre[2 * p] = r2.x;
            pre[2 * p + 1] = r2.y;
        }
        silu8(pre, sil);
        uint4 out;
        uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
        for (int p = 0; p < 4; ++p) o[p] = f2_to_bf2(pack2(sil[2 * p], sil[2 * p + 1]));
        bf16* row = dst + (b * T + t) * tok_stride + base;
        if (head_stride) {
            for (int r = 0; r < rep; ++r) *reinterpret_cast<uint4*>(row + r * head_stride) = out;
        } else {
            *reinterpret_cast<uint4*>(row) = out;
        }
    }
}

template <int TAPS, int T>
static int conv_step_vec(const bf16* state, const bf16* qkv, int64_t sqb, int64_t sqt, const bf16* w, bf16* ext,
                         bf16* q, bf16* k, bf16* v, int64_t B, int64_t C, int64_t key_dim, int64_t value_dim, int dk,
                         int rep, cudaStream_t s, bool dependent) {
    constexpr int threads = 128;
    const unsigned blocks = (unsigned)((B * (C / 8) + threads - 1) / threads);
    return launch_conv_kernel(conv_step_vec_kernel<TAPS, T>, blocks, threads, dependent, s, state, qkv, sqb, sqt, w,
                              ext, q, k, v, B, C, key_dim, value_dim, dk, rep);
}

template <int TAPS>
static int conv_step_vec_t(int64_t T, const bf16* sp, const bf16* xp, int64_t sqb, int64_t sqt, const bf16* wp,
                           bf16* ep, bf16* qp, bf16* kp, bf16* vp, int64_t B, int64_t C, int64_t key_dim,
                           int64_t value_dim, int dk, int rep, cudaStream_t s, bool dependent) {
    switch (T) {
#define GDN_CONV_STEP_T(n) \
    case n: return conv_step_vec<TAPS, n>(sp, xp, sqb, sqt, wp, ep, qp, kp, vp, B, C, key_dim, value_dim, dk, rep, s, \
                                          dependent);
        GDN_CONV_STEP_T(1) GDN_CONV_STEP_T(2) GDN_CONV_STEP_T(3) GDN_CONV_STEP_T(4)
        GDN_CONV_STEP_T(5) GDN_CONV_STEP_T(6) GDN_CONV_STEP_T(7) GDN_CONV_STEP_T(8)
#undef GDN_CONV_STEP_T
        default: return GDN_ERR_UNSUPPORTED;
    }
}

int launch_conv_step(const void* state, const void* qkv, int64_t sqb, int64_t sqt, const void* w, void* ext, void* q,
                     void* k, void* v, int64_t B, int64_t T, int taps, int K, int64_t key_dim, int64_t value_dim, int dk,
                     int dv, cudaStream_t s, bool dependent) {
    const int64_t C = 2 * key_dim + value_dim;
    if (B == 0 || C == 0) return GDN_OK;
    const int rep = (int)((value_dim / dv) / (key_dim / dk));
    auto sp = static_cast<const bf16*>(state);
    auto xp = static_cast<const bf16*>(qkv);
    auto wp = static_cast<const bf16*>(w);
    auto ep = static_cast<bf16*>(ext);
    auto qp = static_cast<bf16*>(q);
    auto kp = static_cast<bf16*>(k);
    auto vp = static_cast<bf16*>(v);
    // 16-byte path: 8-channel groups that never straddle q / k / v or a head, 16-byte aligned
    // rows, the engine's 4-tap weight with a 3- or 4-column state, and up to 8 new tokens
    const bool vec = K == 4 && (taps == 3 || taps == 4) && T >= 1 && T <= 8 && key_dim % 8 == 0 &&
                     value_dim % 8 == 0 && dk % 8 == 0 && dv == dk && sqb % 8 == 0 && sqt % 8 == 0 &&
                     aligned16(state) && aligned16(qkv) && aligned16(w) && aligned16(ext) && aligned16(q) &&
                     aligned16(k) && aligned16(v);
    if (vec) {
        if (taps == 3)
            return conv_step_vec_t<3>(T, sp, xp, sqb, sqt, wp, ep, qp, kp, vp, B, C, key_dim, value_dim, dk, rep, s,
                                      dependent);
        return conv_step_vec_t<4>(T, sp, xp, sqb, sqt, wp, ep, qp, kp, vp, B, C, key_dim, value_dim, dk, rep, s,
                                  dependent);
    }
    constexpr int threads = 128;
    dim3 grid((unsigned)((C + threads - 1) / threads), (unsigned)B);
    conv_step_kernel<<<grid, threads, 0, s>>>(static_cast<const bf16*>(state), static_cast<const bf16*>(qkv), sqb, sqt,
                                              static_cast<const bf16*>(w), static_cast<bf16*>(ext),
                                              static_cast<bf16*>(q), static_cast<bf16*>(k), static_cast<bf16*>(v), T,
                                              taps, K, C, key_dim, value_dim, dk, dv, rep);
    return launch_status();
}


// Conv-state commit after a verify step (the gather of inference/engine.py:473-474 and :381):
// state[l, b, c, i] = ext[l, b, c, clamp(accepted[b], 0, T) + i] for i < taps, over every layer of
// one launch. One thread per (layer, row, channel); ext rows are taps + T contiguous values.
__global__ void conv_state_commit_kernel(const bf16* __restrict__ ext, bf16* __restrict__ state,
                                         const int64_t* __restrict__ accepted, int64_t B, int64_t C, int taps,
                                         int64_t T, int64_t esl, int64_t esb, int64_t ssl, int64_t ssb) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int64_t b = blockIdx.y, l = blockIdx.z;
    int64_t j = accepted[b];
    j = j < 0 ? 0 : (j > T ? T : j);
    const bf16* src = ext + l * esl + b * esb + c * (taps + T) + j;
    bf16* dst = state + l * ssl + b * ssb + c * taps;
    for (int i = 0; i < taps; ++i) dst[i] = src[i];
}

// The same for the engine's shape, taps + T = 8 values a channel (one 16-byte vector): one thread
// per (layer, row, channel) reads its channel's vector (a warp reads 512 contiguous bytes), takes
// the taps values at j (two 64-bit halves, a shift by a run-time multiple of 16 bits) into shared
// memory, and the CTA's 128 channels' taps x 2 bytes go out as contiguous 16-byte stores.
template <int TAPS>
__global__ void __launch_bounds__(128) conv_state_commit_vec_kernel(const bf16* __restrict__ ext,
                                                                    bf16* __restrict__ state,
                                                                    const int64_t* __restrict__ accepted, int64_t C,
                                                                    int64_t T, int64_t esl, int64_t esb, int64_t ssl,
                                                                    int64_t ssb) {
    constexpr int L = 8, CH = 128;
    __shared__ alignas(16) uint16_t out[CH * TAPS];
    const int64_t c0 = (int64_t)blockIdx.x * CH;
    const int64_t b = blockIdx.y, l = blockIdx.z;
    const int n = (int)(C - c0 < CH ? C - c0 : CH);  // channels of this CTA, a multiple of 8
    int64_t j = accepted[b];
    j = j < 0 ? 0 : (j > T ? T : j);
    if ((int)threadIdx.x < n) {
        const uint4 v = reinterpret_cast<const uint4*>(ext + l * esl + b * esb + c0 * L)[threadIdx.x];
        const uint64_t lo = ((uint64_t)v.y << 32) | v.x, hi = ((uint64_t)v.w << 32) | v.z;
#pragma unroll
        for (int i = 0; i < TAPS; ++i) {
            const int k = (int)j + i;  // < L: j <= T = L - TAPS
            out[threadIdx.x * TAPS + i] = (uint16_t)(k < 4 ? lo >> (16 * k) : hi >> (16 * (k - 4)));
        }
    }
    __syncthreads();
    const int vecs = n * TAPS / 8;  // 16-byte vectors of the CTA's outputs
    uint4* dst = reinterpret_cast<uint4*>(state + l * ssl + b * ssb + c0 * TAPS);
    for (int i = threadIdx.x; i < vecs; i += CH) dst[i] = reinterpret_cast<const uint4*>(out)[i];
}

int launch_conv_state_commit(const void* ext, void* state, const int64_t* accepted, int64_t layers, int64_t B,
                             int64_t C, int taps, int64_t T, int64_t esl, int64_t esb, int64_t ssl, int64_t ssb,
                             cudaStream_t s) {
    if (layers == 0 || B == 0 || C == 0) return GDN_OK;
    const bool vec = taps + T == 8 && (taps == 3 || taps == 4) && C % 8 == 0 && aligned16(ext) && aligned16(state) &&
                     (esl * 2) % 16 == 0 && (esb * 2) % 16 == 0 && (ssl * 2) % 16 == 0 && (ssb * 2) % 16 == 0;
    if (vec) {
        constexpr int threads = 128;
        dim3 grid((unsigned)((C + threads - 1) / threads), (unsigned)B, (unsigned)layers);
        if (taps == 3)
            conv_state_commit_vec_kernel<3><<<grid, threads, 0, s>>>(static_cast<const bf16*>(ext),
                                                                     static_cast<bf16*>(state), accepted, C, T, esl,
                                                                     esb, ssl, ssb);
        else
            conv_state_commit_vec_kernel<4><<<grid, threads, 0, s>>>(static_cast<const bf16*>(ext),
                                                                     static_cast<bf16*>(state), accepted, C, T, esl,
                                                                     esb, ssl, ssb);
        return launch_status();
    }
    constexpr int threads = 256;
    dim3 grid((unsigned)((C + threads - 1) / threads), (unsigned)B, (unsigned)layers);
    conv_state_commit_kernel<<<grid, threads, 0, s>>>(static_cast<const bf16*>(ext), static_cast<bf16*>(state),
                                                      accepted, B, C, taps, T, esl, esb, ssl, ssb);
    return launch_status();
}

}  // namespace gdn
