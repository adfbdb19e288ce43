// Chunked gated-delta-rule prefill on tcgen05 tensor cores (chunk 64, WY/UT form).
//
// Reference semantics: torch_chunk_gated_delta_rule, model/model.py:242-286 (fp32 eager;
// fla's chunk_gated_delta_rule on CUDA, model/model.py:289-294), with varlen packing
// through cu_seqlens as in fla 0.5.x.
//
// One CTA owns one (sequence, value head, slice of VS value columns) and walks the
// sequence's chunks in order with the fp32 state slice S [128 x VS] resident in TMEM.
// Per chunk of 64 tokens (gc = cumulative log decay, rk / rq = inverse L2 norms of the
// raw bf16 k / q rows, q scale folded into rq):
//   KK = K K^T, QK = Q K^T                              (tcgen05, raw bf16 operands)
//   A  = strict_lower(beta_i rk_i rk_j KK_ij e^{gc_i - gc_j}),  P = rq_i rk_j QK_ij e^{..} (j <= i)
//   X  = (I + A)^-1: 16x16 diagonal blocks and the 16->32 merge on CUDA cores in fp32,
//        the 32->64 merge as two tcgen05 products
//   U  = X diag(beta) V                                 (accumulated in fp32 TMEM)
//   W  = X diag(beta e^{gc} rk) K
//   VN = U - W S          O1 = Q S                      (S as bf16 operand)
//   o  = rq e^{gc} O1 + P VN
//   S <- e^{g_last} S + K^T diag(rk e^{g_last - gc}) VN (VN split into bf16 hi + lo)
// Rows past the end of a sequence get beta = 0 and g = 0, which makes them identity steps.
//
// Every wait is bounded (sm100.cuh); a wait that gives up raises the device error word
// and the CTA unwinds: it drains the copies it started, frees TMEM and returns.

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace gdn {

using namespace sm100;

struct ChunkParams {
    CUtensorMap tm_q;  // 4-D (128, H, T, B) bf16, box (64, 1, 64, 1), 128-byte swizzle
    CUtensorMap tm_k;
    CUtensorMap tm_v;  // 4-D (128, HV, T, B)
    const float* g;    // [B, T, HV]
    const void* beta;  // [B, T, HV] bf16 or fp32
    int beta_f32;
    const float* h0;   // [N, HV, 128, 128] or null
    float* ht;         // [N, HV, 128, 128] or null
    bf16* o;           // [B, T, HV, 128]
    const int32_t* cu_seqlens;
    int64_t T;
    int HV, rep;
    float scale;
};

template <int VS>
struct Layout {
    static constexpr uint32_t kPanelK = 64 * 128;  // one 128-byte panel of 64 rows
    static constexpr uint32_t K0 = 0;              // K tile, stage 0: two d-panels
    static constexpr uint32_t K1 = 16384;          // K tile, stage 1
    static constexpr uint32_t Q = 32768;           // Q tile
    static constexpr uint32_t V = 49152;           // V tile: VS/64 column panels
    static constexpr uint32_t AF = V + VS * 128;   // fp32 64x64, row-major (inverse workspace)
    static constexpr uint32_t PM = AF + 16384;     // bf16 P, K-major
    static constexpr uint32_t AU = PM + 8192;      // bf16 X diag(beta); E32 during the inverse
    static constexpr uint32_t AW = AU + 8192;      // bf16 X diag(beta e^gc rk); D32 during the inverse
    static constexpr uint32_t WB = AW + 8192;      // bf16 W (two d-panels); T2 during the inverse
    static constexpr uint32_t SB = WB + 16384;     // bf16 S^T [v][d], two d-panels of VS rows
    static constexpr uint32_t VHI = SB + VS * 256; // bf16 hi(ctilde VN) [tok][v]
    static constexpr uint32_t VLO = VHI + VS * 128;
    static constexpr uint32_t VBF = VLO + VS * 128; // bf16 VN [tok][v]
    static constexpr uint32_t END = VBF + VS * 128;
    static constexpr uint32_t SMEM = END + 1024;   // + alignment slack
};

struct ChunkShared {
    uint64_t bar_k[2];
    uint64_t bar_q;
    uint64_t bar_v;
    uint64_t bar_mma;
    uint32_t tmem_base;
    int abort;
    float gcl[64];   // cumulative log2 decay
    float beta[64];
    float rk[64];    // 1 / |k| (0 past the end)
    float rq[64];    // scale / |q|
    float cw[64];    // beta e^gc rk
    float ce[64];    // rk e^(g_last - gc)
    float eq[64];    // rq e^gc
    float red[4];
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kR = 128;        // TMEM column of the scratch accumulators
constexpr uint32_t kHalfB = 16u << 16;  // lane offset of the second M=64 accumulator

__device__ __forceinline__ bf16* smem_bf(uint8_t* base, uint32_t off) { return reinterpret_cast<bf16*>(base + off); }

// Writes 8 fp32 values as one 16-byte bf16 chunk of a swizzled panel row.
__device__ __forceinline__ void put_chunk(uint8_t* panel, uint32_t row, uint32_t chunk, const float* v) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(panel + sw128(row, chunk)) = raw;
}

__device__ __forceinline__ void get_chunk(const uint8_t* panel, uint32_t row, uint32_t chunk, float* v) {
    const uint4 raw = *reinterpret_cast<const uint4*>(panel + sw128(row, chunk));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

// CTA barrier that also carries the abort flag: returns true when every thread may go on.
__device__ __forceinline__ bool cta_sync(ChunkShared& sh, bool ok) {
    if (!ok) sh.abort = 1;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return sh.abort == 0;
}

template <int VS>
__global__ void __launch_bounds__(128, 1) chunk_prefill_kernel(const __grid_constant__ ChunkParams p) {
    using L = Layout<VS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ ChunkShared sh;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int kSlices = kHeadDim / VS;
    const int hv = blockIdx.x / kSlices;
    const int v0 = (blockIdx.x % kSlices) * VS;
    const int h = hv / p.rep;
    const int n = blockIdx.y;
    int64_t bos = 0, len = p.T, brow = n;
    if (p.cu_seqlens) {
        bos = p.cu_seqlens[n];
        len = p.cu_seqlens[n + 1] - bos;
        brow = 0;
    }
    const int nchunks = (int)((len + 63) / 64);
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const int half_row = 16 * warp + (lane & 15);  // row of an M=64 accumulator held by this thread
    const bool in_half_a = lane < 16;

    if (tid == 0) {
        sh.abort = 0;
        mbar_init(&sh.bar_k[0], 1);
        mbar_init(&sh.bar_k[1], 1);
        mbar_init(&sh.bar_q, 1);
        mbar_init(&sh.bar_v, 1);
        mbar_init(&sh.bar_mma, 1);
        fence_mbar_init();
        tma_prefetch_map(&p.tm_q);
        tma_prefetch_map(&p.tm_k);
        tma_prefetch_map(&p.tm_v);
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    cta_sync(sh, true);
    const uint32_t tb = sh.tmem_base;
    const uint32_t tS = tb;            // state slice, all 128 lanes, VS columns
    const uint32_t tRa = tb + kR;      // M=64 accumulator, lanes 0-15 of each quarter
    const uint32_t tRb = tb + kR + kHalfB;  // M=64 accumulator, lanes 16-31 of each quarter

    // Outstanding TMA loads per barrier (tracked by the issuing thread, tid 0) and the
    // parity each one completes with, so that an abort can drain them.
    int k_pend[2] = {0, 0}, k_par[2] = {0, 0}, q_pend = 0, q_par = 0, v_pend = 0, v_par = 0;
    auto issue_k = [&](int c) {
        const int stage = c & 1;
        uint8_t* dst = sm + (stage ? L::K1 : L::K0);
        mbar_arrive_expect_tx(&sh.bar_k[stage], 16384);
        const int t = (int)(bos + 64 * c);
        tma_load_4d(dst, &p.tm_k, &sh.bar_k[stage], 0, h, t, (int)brow);
        tma_load_4d(dst + L::kPanelK, &p.tm_k, &sh.bar_k[stage], 64, h, t, (int)brow);
        k_pend[stage] = 1;
        k_par[stage] = (c >> 1) & 1;
    };
    auto issue_q = [&](int c) {
        mbar_arrive_expect_tx(&sh.bar_q, 16384);
        const int t = (int)(bos + 64 * c);
        tma_load_4d(sm + L::Q, &p.tm_q, &sh.bar_q, 0, h, t, (int)brow);
        tma_load_4d(sm + L::Q + L::kPanelK, &p.tm_q, &sh.bar_q, 64, h, t, (int)brow);
        q_pend = 1;
        q_par = c & 1;
    };
    auto issue_v = [&](int c) {
        mbar_arrive_expect_tx(&sh.bar_v, VS * 128);
        const int t = (int)(bos + 64 * c);
#pragma unroll
        for (int pnl = 0; pnl < VS / 64; ++pnl)
            tma_load_4d(sm + L::V + pnl * L::kPanelK, &p.tm_v, &sh.bar_v, v0 + 64 * pnl, hv, t, (int)brow);
        v_pend = 1;
        v_par = c & 1;
    };

    uint32_t mma_phase = 0;
    auto mma_done = [&]() -> bool {
        const bool ok = mbar_wait(&sh.bar_mma, mma_phase, kSiteMma);
        mma_phase ^= 1;
        return ok;
    };

    if (nchunks > 0 && tid == 0) {
        issue_k(0);
        issue_q(0);
        issue_v(0);
        if (nchunks > 1) issue_k(1);
    }

    // Initial state: thread t holds state row t (lane t) -> TMEM and the bf16 S^T operand.
    {
        const int d = tid;
        uint8_t* sb = sm + L::SB + (d >> 6) * (VS * 128);
        for (int c0 = 0; c0 < VS; c0 += 16) {
            float r[16];
            if (p.h0) {
                const float* src = p.h0 + (((int64_t)n * p.HV + hv) * kHeadDim + d) * kHeadDim + v0 + c0;
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    const float4 x = *reinterpret_cast<const float4*>(src + j);
                    r[j] = x.x; r[j + 1] = x.y; r[j + 2] = x.z; r[j + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) r[j] = 0.f;
            }
            tmem_st16(tS + lane_base + c0, r);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int v = c0 + j;
                *reinterpret_cast<bf16*>(sb + sw128(v, (d & 63) >> 3) + (d & 7) * 2) = __float2bfloat16_rn(r[j]);
            }
        }
        tmem_wait_st();
    }
    fence_async_smem();
    bool ok = cta_sync(sh, true);

    int c = 0;
    for (; ok && c < nchunks; ++c) {
        const int stage = c & 1;
        const uint8_t* kb = sm + (stage ? L::K1 : L::K0);
        const int64_t t0 = bos + 64 * (int64_t)c;
        const int nvalid = (int)((len - 64 * (int64_t)c) < 64 ? (len - 64 * (int64_t)c) : 64);

        // ---- 1. gates: cumulative log decay (log2 units) and beta, zero past the end
        if (tid < 64) {
            float gv = 0.f, bv = 0.f;
            if (tid < nvalid) {
                const int64_t gi = (brow * p.T + t0 + tid) * p.HV + hv;
                gv = p.g[gi] * kLog2e;
                bv = p.beta_f32 ? static_cast<const float*>(p.beta)[gi] : to_f32(static_cast<const bf16*>(p.beta)[gi]);
            }
            float x = gv;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (tid == 31) sh.red[0] = x;
            sh.gcl[tid] = x;
            sh.beta[tid] = bv;
        }
        // ---- 2. wait for this chunk's K and Q tiles
        bool wok = true;
        wok = mbar_wait(&sh.bar_k[stage], (c >> 1) & 1, kSiteTmaLoad) && wok;
        wok = mbar_wait(&sh.bar_q, c & 1, kSiteTmaLoad) && wok;
        if (wok) k_pend[stage] = q_pend = 0;
        if (!cta_sync(sh, wok)) break;
        if (tid >= 32 && tid < 64) sh.gcl[tid] += sh.red[0];

        // ---- 3. inverse norms of the raw rows (thread t: k row t, or q row t-64)
        {
            const bool is_k = tid < 64;
            const int row = tid & 63;
            const uint8_t* base = is_k ? kb : sm + L::Q;
            float ss = 0.f;
#pragma unroll
            for (int pnl = 0; pnl < 2; ++pnl)
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    float v8[8];
                    get_chunk(base + pnl * L::kPanelK, row, ch, v8);
#pragma unroll
                    for (int e = 0; e < 8; ++e) ss += v8[e] * v8[e];
                }
            const bool valid = row < nvalid;
            const float inv = rsqrtf(ss + 1e-6f);
            if (is_k) sh.rk[row] = valid ? inv : 0.f;
            else sh.rq[row] = inv * p.scale;
        }
        // ---- 4. KK = K K^T (lanes A), QK = Q K^T (lanes B)
        if (tid == 0) {
            const uint32_t id = make_idesc(64, 64, kFmtBF16, false, false);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t po = (kk >> 2) * L::kPanelK, ko = (kk & 3) * 32;
                const uint64_t bdesc = sdesc_kmajor(kb + po, ko);
                mma_f16(tRa, sdesc_kmajor(kb + po, ko), bdesc, id, kk > 0);
                mma_f16(tRb, sdesc_kmajor(sm + L::Q + po, ko), bdesc, id, kk > 0);
            }
            mma_commit(&sh.bar_mma);
        }
        if (!cta_sync(sh, mma_done())) break;

        // per-row scalars that need the full gc / rk vectors
        if (tid < 64) {
            const float gcl = sh.gcl[tid];
            const float glast = sh.gcl[63];
            const float bt = sh.beta[tid];
            const float rk = sh.rk[tid];
            sh.cw[tid] = bt * exp2f(gcl) * rk;
            sh.ce[tid] = rk * exp2f(glast - gcl);
            sh.eq[tid] = sh.rq[tid] * exp2f(gcl);
        }
        // ---- 5. A (fp32, lanes A) and P (bf16, lanes B) from the score accumulators
        {
            const int i = half_row;
            const float gci = sh.gcl[i];
            float* arow = reinterpret_cast<float*>(sm + L::AF) + i * 64;
            const float ri = in_half_a ? sh.beta[i] * sh.rk[i] : sh.rq[i];
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 16) {
                float r[16];
                tmem_ld16(tb + kR + lane_base + c0, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int col = c0 + j;
                    const bool keep = in_half_a ? (col < i) : (col <= i);
                    const float dec = keep ? exp2f(gci - sh.gcl[col]) : 0.f;
                    r[j] = keep ? r[j] * ri * sh.rk[col] * dec : 0.f;
                }
                if (in_half_a) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4*>(arow + c0 + j) = make_float4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                } else {
                    put_chunk(sm + L::PM, i, c0 / 8, r);
                    put_chunk(sm + L::PM, i, c0 / 8 + 1, r + 8);
                }
            }
        }
        if (!cta_sync(sh, true)) break;

        // ---- 6a. inverses of the four 16x16 diagonal blocks of I + A (fp32, CUDA cores)
        {
            float x[16];
            const int b = (tid >> 4) & 3, col = tid & 15;
            const float* Af = reinterpret_cast<const float*>(sm + L::AF);
            if (tid < 64) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float s = 0.f;
#pragma unroll
                    for (int j = 0; j < i; ++j) s += Af[(16 * b + i) * 64 + 16 * b + j] * x[j];
                    x[i] = (i == col) ? 1.f : (i > col ? -s : 0.f);
                }
            }
            __syncthreads();
            if (tid < 64) {
                float* Aw = reinterpret_cast<float*>(sm + L::AF);
#pragma unroll
                for (int i = 0; i < 16; ++i) Aw[(16 * b + i) * 64 + 16 * b + col] = x[i];
            }
        }
        __syncthreads();
        // ---- 6b. 16 -> 32 merge inside each 32-block: X10 = -X11 (A10 X00)
        {
            float* Af = reinterpret_cast<float*>(sm + L::AF);
            const int blk = tid >> 6;        // 32-block 0 or 1
            const int e = tid & 63;
            const int i = e >> 2, j0 = (e & 3) * 4;
            const int r0 = 32 * blk;
            float t4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kx = 0; kx < 16; ++kx) {
                const float a = Af[(r0 + 16 + i) * 64 + r0 + kx];
                const float4 x = *reinterpret_cast<const float4*>(&Af[(r0 + kx) * 64 + r0 + j0]);
                t4[0] += a * x.x; t4[1] += a * x.y; t4[2] += a * x.z; t4[3] += a * x.w;
            }
            __syncthreads();
            *reinterpret_cast<float4*>(&Af[(r0 + 16 + i) * 64 + r0 + j0]) = make_float4(t4[0], t4[1], t4[2], t4[3]);
            __syncthreads();
            float x4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kx = 0; kx < 16; ++kx) {
                const float a = Af[(r0 + 16 + i) * 64 + r0 + 16 + kx];
                const float4 t = *reinterpret_cast<const float4*>(&Af[(r0 + 16 + kx) * 64 + r0 + j0]);
                x4[0] += a * t.x; x4[1] += a * t.y; x4[2] += a * t.z; x4[3] += a * t.w;
            }
            __syncthreads();
            *reinterpret_cast<float4*>(&Af[(r0 + 16 + i) * 64 + r0 + j0]) = make_float4(-x4[0], -x4[1], -x4[2], -x4[3]);
        }
        __syncthreads();
        // ---- 6c. bf16 operands of the 32 -> 64 merge: E32 (lower-left block of A) and D32
        if (tid < 64) {
            const float* Af = reinterpret_cast<const float*>(sm + L::AF);
            const int i = tid;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                float e8[8], d8[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int j = ch * 8 + q;
                    const float a = Af[i * 64 + j];
                    const bool lower_left = i >= 32 && j < 32;
                    const bool diag = (i >> 5) == (j >> 5) && j <= i;
                    e8[q] = lower_left ? a : 0.f;
                    d8[q] = diag ? a : 0.f;
                }
                put_chunk(sm + L::AU, i, ch, e8);
                put_chunk(sm + L::AW, i, ch, d8);
            }
        }
        fence_async_smem();
        if (!cta_sync(sh, true)) break;
        // T2 = E32 D32 (lanes A)
        if (tid == 0) {
            const uint32_t id = make_idesc(64, 64, kFmtBF16, false, true);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_f16(tRa, sdesc_kmajor(sm + L::AU, kk * 32), sdesc_mnmajor(sm + L::AW + kk * 2048, 8192), id, kk > 0);
            mma_commit(&sh.bar_mma);
        }
        if (!cta_sync(sh, mma_done())) break;
        {
            float r[16];
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 16) {
                tmem_ld16(tb + kR + lane_base + c0, r);
                tmem_wait_ld();
                if (in_half_a) {
                    put_chunk(sm + L::WB, half_row, c0 / 8, r);
                    put_chunk(sm + L::WB, half_row, c0 / 8 + 1, r + 8);
                }
            }
        }
        fence_async_smem();
        if (!cta_sync(sh, true)) break;
        // X_LL = D32 T2 (lanes B)
        if (tid == 0) {
            const uint32_t id = make_idesc(64, 64, kFmtBF16, false, true);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_f16(tRb, sdesc_kmajor(sm + L::AW, kk * 32), sdesc_mnmajor(sm + L::WB + kk * 2048, 8192), id, kk > 0);
            mma_commit(&sh.bar_mma);
        }
        if (!cta_sync(sh, mma_done())) break;
        // X = D32 - X_LL; the two scaled bf16 copies feed U and W
        {
            const float* Af = reinterpret_cast<const float*>(sm + L::AF);
            const int i = half_row;
            float r[16];
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 16) {
                tmem_ld16(tb + kR + lane_base + c0, r);
                tmem_wait_ld();
                if (!in_half_a) {
                    float xu[16], xw[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int col = c0 + j;
                        float x;
                        if (col > i) x = 0.f;
                        else if (i >= 32 && col < 32) x = -r[j];
                        else x = Af[i * 64 + col];
                        xu[j] = x * sh.beta[col];
                        xw[j] = x * sh.cw[col];
                    }
                    put_chunk(sm + L::AU, i, c0 / 8, xu);
                    put_chunk(sm + L::AU, i, c0 / 8 + 1, xu + 8);
                    put_chunk(sm + L::AW, i, c0 / 8, xw);
                    put_chunk(sm + L::AW, i, c0 / 8 + 1, xw + 8);
                }
            }
        }
        fence_async_smem();
        if (!cta_sync(sh, true)) break;

        // ---- 7. W = (X diag(cw)) K (lanes A, 128 cols); U = (X diag(beta)) V (lanes B)
        if (tid == 0) {
            const bool vok = mbar_wait(&sh.bar_v, c & 1, kSiteTmaLoad);
            if (vok) v_pend = 0;
            else sh.abort = 1;
            const uint32_t idw = make_idesc(64, 128, kFmtBF16, false, true);
            const uint32_t idu = make_idesc(64, VS, kFmtBF16, false, true);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                mma_f16(tRa, sdesc_kmajor(sm + L::AW, kk * 32), sdesc_mnmajor(kb + kk * 2048, L::kPanelK), idw, kk > 0);
                mma_f16(tRb, sdesc_kmajor(sm + L::AU, kk * 32), sdesc_mnmajor(sm + L::V + kk * 2048, L::kPanelK), idu,
                        kk > 0);
            }
            mma_commit(&sh.bar_mma);
        }
        if (!cta_sync(sh, mma_done())) break;
        if (tid == 0 && c + 1 < nchunks) issue_v(c + 1);
        // ---- 8. W -> bf16 operand
        {
            float r[16];
#pragma unroll
            for (int c0 = 0; c0 < 128; c0 += 16) {
                tmem_ld16(tb + kR + lane_base + c0, r);
                tmem_wait_ld();
                if (in_half_a) {
                    uint8_t* panel = sm + L::WB + (c0 >> 6) * L::kPanelK;
                    put_chunk(panel, half_row, (c0 & 63) / 8, r);
                    put_chunk(panel, half_row, (c0 & 63) / 8 + 1, r + 8);
                }
            }
        }
        fence_async_smem();
        if (!cta_sync(sh, true)) break;
        // ---- 9. VN = U - W S (lanes B, accumulate); O1 = Q S (lanes A)
        if (tid == 0) {
            const uint32_t idn = make_idesc(64, VS, kFmtBF16, false, false, true);
            const uint32_t ido = make_idesc(64, VS, kFmtBF16, false, false);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t ko = (kk & 3) * 32;
                const uint8_t* sbp = sm + L::SB + (kk >> 2) * (VS * 128);
                const uint64_t bdesc = sdesc_kmajor(sbp, ko);
                mma_f16(tRb, sdesc_kmajor(sm + L::WB + (kk >> 2) * L::kPanelK, ko), bdesc, idn, 1);
                mma_f16(tRa, sdesc_kmajor(sm + L::Q + (kk >> 2) * L::kPanelK, ko), bdesc, ido, kk > 0);
            }
            mma_commit(&sh.bar_mma);
        }
        if (!cta_sync(sh, mma_done())) break;
        if (tid == 0 && c + 1 < nchunks) issue_q(c + 1);
        // ---- 10. VN -> bf16 VN and the split ctilde VN; decay the state in TMEM
        {
            const int i = half_row;
            const float cei = sh.ce[i];
            float r[16];
#pragma unroll
            for (int c0 = 0; c0 < VS; c0 += 16) {
                tmem_ld16(tb + kR + lane_base + c0, r);
                tmem_wait_ld();
                if (!in_half_a) {
                    float hi[16], lo[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float x = cei * r[j];
                        hi[j] = round_bf16(x);
                        lo[j] = x - hi[j];
                    }
                    const uint32_t pnl = (c0 >> 6) * L::kPanelK, ch = (c0 & 63) / 8;
                    put_chunk(sm + L::VBF + pnl, i, ch, r);
                    put_chunk(sm + L::VBF + pnl, i, ch + 1, r + 8);
                    put_chunk(sm + L::VHI + pnl, i, ch, hi);
                    put_chunk(sm + L::VHI + pnl, i, ch + 1, hi + 8);
                    put_chunk(sm + L::VLO + pnl, i, ch, lo);
                    put_chunk(sm + L::VLO + pnl, i, ch + 1, lo + 8);
                }
            }
            const float decay = exp2f(sh.gcl[63]);
#pragma unroll
            for (int c0 = 0; c0 < VS; c0 += 16) {
                tmem_ld16(tS + lane_base + c0, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) r[j] *= decay;
                tmem_st16(tS + lane_base + c0, r);
            }
            tmem_wait_st();
        }
        fence_async_smem();
        if (!cta_sync(sh, true)) break;
        // ---- 11. S += K^T (hi + lo) (all lanes); O2 = P VN (lanes B)
        if (tid == 0) {
            const uint32_t ids = make_idesc(128, VS, kFmtBF16, true, true);
            const uint32_t ido = make_idesc(64, VS, kFmtBF16, false, true);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t adesc = sdesc_mnmajor(kb + kk * 2048, L::kPanelK);
                mma_f16(tS, adesc, sdesc_mnmajor(sm + L::VHI + kk * 2048, L::kPanelK), ids, 1);
                mma_f16(tS, adesc, sdesc_mnmajor(sm + L::VLO + kk * 2048, L::kPanelK), ids, 1);
                mma_f16(tRb, sdesc_kmajor(sm + L::PM, kk * 32), sdesc_mnmajor(sm + L::VBF + kk * 2048, L::kPanelK), ido,
                        kk > 0);
            }
            mma_commit(&sh.bar_mma);
        }
        if (!cta_sync(sh, mma_done())) break;
        if (tid == 0 && c + 2 < nchunks) issue_k(c + 2);
        // ---- 12. o = eq O1 + O2 -> global; S -> bf16 operand (or the final state)
        {
            const int i = half_row;
            const bool row_ok = i < nvalid;
            const float eqi = sh.eq[i];
            bf16* orow = p.o + ((brow * p.T + t0 + i) * p.HV + hv) * kHeadDim + v0;
            float r[16];
#pragma unroll
            for (int c0 = 0; c0 < VS; c0 += 16) {
                tmem_ld16(tb + kR + lane_base + c0, r);
                tmem_wait_ld();
                float partner[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, r[j], 16);
                // lanes A hold O1 and see O2 in partner; lanes B the other way round
                float out[8];
                const int jb = in_half_a ? 0 : 8;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float o1 = in_half_a ? r[jb + j] : partner[jb + j];
                    const float o2 = in_half_a ? partner[jb + j] : r[jb + j];
                    out[j] = eqi * o1 + o2;
                }
                if (row_ok) {
                    uint4 raw;
                    __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(out[2 * j], out[2 * j + 1]);
                    *reinterpret_cast<uint4*>(orow + c0 + jb) = raw;
                }
            }
            const bool last = c + 1 == nchunks;
            const int d = tid;
            uint8_t* sb = sm + L::SB + (d >> 6) * (VS * 128);
#pragma unroll
            for (int c0 = 0; c0 < VS; c0 += 16) {
                tmem_ld16(tS + lane_base + c0, r);
                tmem_wait_ld();
                if (last) {
                    if (p.ht) {
                        float* dst = p.ht + (((int64_t)n * p.HV + hv) * kHeadDim + d) * kHeadDim + v0 + c0;
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4*>(dst + j) = make_float4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        *reinterpret_cast<bf16*>(sb + sw128(c0 + j, (d & 63) >> 3) + (d & 7) * 2) =
                            __float2bfloat16_rn(r[j]);
                }
            }
        }
        fence_async_smem();
        ok = cta_sync(sh, true);
    }

    // Empty sequence: the final state is the initial state.
    if (nchunks == 0 && p.ht) {
        const int d = tid;
        float* dst = p.ht + (((int64_t)n * p.HV + hv) * kHeadDim + d) * kHeadDim + v0;
        const float* src = p.h0 ? p.h0 + (((int64_t)n * p.HV + hv) * kHeadDim + d) * kHeadDim + v0 : nullptr;
        for (int j = 0; j < VS; j += 4)
            *reinterpret_cast<float4*>(dst + j) = src ? *reinterpret_cast<const float4*>(src + j) : make_float4(0, 0, 0, 0);
    }

    // Unwind after an abort: let every copy this CTA started land before the CTA exits.
    if (sh.abort && tid == 0) {
        for (int st = 0; st < 2; ++st)
            if (k_pend[st]) mbar_wait(&sh.bar_k[st], k_par[st], kSiteDrain);
        if (q_pend) mbar_wait(&sh.bar_q, q_par, kSiteDrain);
        if (v_pend) mbar_wait(&sh.bar_v, v_par, kSiteDrain);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tb, kTmemCols);
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 4-D map over [B, T, heads, 128] bf16 with element strides (sb, st, sh); box (64, 1, 64, 1).
static bool make_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t heads, int64_t sb, int64_t st,
                     int64_t sh) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)heads, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)st * 2, (cuuint64_t)sb * 2};
    cuuint32_t box[4] = {64, 1, 64, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int VS>
static int launch_vs(const ChunkParams& p, int64_t nseq, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(chunk_prefill_kernel<VS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Layout<VS>::SMEM) != cudaSuccess)
            return GDN_ERR_LAUNCH;
        configured = true;
    }
    dim3 grid((unsigned)(p.HV * (kHeadDim / VS)), (unsigned)nseq);
    chunk_prefill_kernel<VS><<<grid, 128, Layout<VS>::SMEM, s>>>(p);
    return launch_status();
}

int launch_chunk(const ChunkArgs& a, cudaStream_t s) {
    if (a.nseq == 0) return GDN_OK;
    ChunkParams p;
    memset(&p, 0, sizeof(p));
    if (!make_map(&p.tm_q, a.q, a.B, a.T, a.H, a.qsb, a.qst, a.qsh) ||
        !make_map(&p.tm_k, a.k, a.B, a.T, a.H, a.ksb, a.kst, a.ksh) ||
        !make_map(&p.tm_v, a.v, a.B, a.T, a.HV, a.vsb, a.vst, a.vsh))
        return GDN_ERR_LAUNCH;
    p.g = a.g;
    p.beta = a.beta;
    p.beta_f32 = a.beta_dtype == GDN_F32;
    p.h0 = a.h0;
    p.ht = a.ht;
    p.o = static_cast<bf16*>(a.o);
    p.cu_seqlens = a.cu_seqlens;
    p.T = a.T;
    p.HV = a.HV;
    p.rep = a.HV / a.H;
    p.scale = a.scale;
    int sms = 148;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    // Split the value columns when whole heads would leave SMs idle.
    if (a.nseq * a.HV >= 2 * sms) return launch_vs<128>(p, a.nseq, s);
    return launch_vs<64>(p, a.nseq, s);
}

}  // namespace gdn
