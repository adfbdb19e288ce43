// Chunked gated-delta-rule prefill on tcgen05 tensor cores (chunk 64, WY/UT form).
//
// Reference semantics: torch_chunk_gated_delta_rule, model/model.py:242-286 (fp32 eager;
// fla's chunk_gated_delta_rule on CUDA, model/model.py:289-294), with varlen packing
// through cu_seqlens as in fla 0.5.x.
//
// One CTA owns one (sequence, value head, slice of VS = 64 value columns) and walks the
// sequence's chunks in order with its fp32 state slice S [128 x VS] resident in TMEM.
// Per chunk of 64 tokens (gc = cumulative log decay, rk / rq = inverse L2 norms of the raw
// bf16 k / q rows, the q scale folded into rq):
//   KK = K K^T, QK = Q K^T                                 tcgen05, raw bf16 operands
//   A  = strict_lower(beta_i rk_i rk_j KK_ij e^{gc_i-gc_j}), P = rq_i rk_j QK_ij e^{..}, j <= i
//   X  = (I + A)^-1: 16x16 diagonal blocks and the 16->32 merge on CUDA cores in fp32,
//        the 32->64 merge as two tcgen05 products
//   W  = X diag(beta e^gc rk) K,  U = X diag(beta) V        (U accumulated in fp32 TMEM)
//   VN = U - W S,  O1 = Q S                                S as a bf16 operand
//   o  = rq e^gc O1 + P VN
//   S <- e^{g_last} S + K^T diag(rk e^{g_last-gc}) VN      VN split into bf16 hi + lo
// Rows past the end of a sequence get beta = 0 and g = 0, which makes them identity steps.
//
// Implementation notes:
//   * the intra-chunk output is folded into the inter-chunk accumulator: with
//     eq_i = rq_i e^{gc_i}, o_i = eq_i (Q S + P' VN)_i where P' = P / eq (row-wise), i.e.
//     P'_ij = rk_j QK_ij e^{-gc_j}; e^{gc_i - gc_j} is formed as e^{gc_i} e^{-gc_j} while the
//     chunk's decay stays above 2^-100 and element by element otherwise;
//   * the chain keeps its fp32 state rows in registers; each chunk's update K^T(...) lands in
//     a fresh TMEM accumulator and is added as S <- e^{g_last} S + dS.
//
// Warp roles (384 threads): warp 0 loads tiles (TMA) and gates; warps 4-7 ("prep") build the
// chunk-local factors P', X, W of chunk c+1 and issue their own MMAs, while warps 8-11
// ("chain") advance the state through chunk c and issue theirs. The roles hand buffers to
// each other through mbarriers; K/Q/V tiles, P', W and the chain's TMEM accumulators are
// double buffered by chunk parity.
//
// Every wait is bounded (sm100.cuh): a wait that gives up raises the device error word and
// the CTA's abort flag; every role then leaves its loop, the loader waits for the copies it
// started, the issuer for the MMAs it issued, TMEM is freed and the CTA returns.

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

constexpr int kVS = 64;                       // value columns per CTA
constexpr uint32_t kPanel = 64 * 128;         // one 128-byte panel of 64 rows
constexpr int kAfStride = 68;                 // fp32 row stride of the inverse workspace

// dynamic shared memory layout (byte offsets, 1024-aligned where TMA or MMA reads)
struct Smem {
    static constexpr uint32_t K = 0;                         // [2] K tiles: two d-panels each
    static constexpr uint32_t Q = K + 2 * 2 * kPanel;        // [2] Q tiles
    static constexpr uint32_t V = Q + 2 * 2 * kPanel;        // [2] V tiles: one panel each
    static constexpr uint32_t PM = V + 2 * kPanel;           // [2] P' (bf16, K-major)
    static constexpr uint32_t WB = PM + 2 * kPanel;          // [2] W (bf16, K-major, two d-panels)
    static constexpr uint32_t AU = WB + 2 * 2 * kPanel;      // X diag(beta); E32 during the inverse
    static constexpr uint32_t AW = AU + kPanel;              // X diag(cw); D32 during the inverse
    static constexpr uint32_t T2 = AW + kPanel;              // E32 D32 (bf16, MN-major)
    static constexpr uint32_t SB = T2 + kPanel;              // S^T [v][d] bf16, two d-panels
    static constexpr uint32_t VHI = SB + 2 * kPanel;         // hi(ce VN) [tok][v]
    static constexpr uint32_t VLO = VHI + kPanel;            // lo(ce VN)
    static constexpr uint32_t VBF = VLO + kPanel;            // VN [tok][v]
    static constexpr uint32_t AF = VBF + kPanel;             // fp32 [64][kAfStride]
    static constexpr uint32_t END = AF + 64 * kAfStride * 4;
    static constexpr uint32_t BYTES = END + 1024;            // + alignment slack
};

struct Bars {
    uint64_t kqv_full[2], kqv_empty[2], gates_full[2], gates_empty[2];
    uint64_t acc_kq, acc_t2, acc_x, acc_wu[2], acc_vn[2], acc_s, drain_prep, drain_chain;
    uint64_t wb_ready, o_free[2];
};

struct Shared {
    Bars bar;
    uint32_t tmem_base;
    int abort;
    // gates ring, written by the loader warp
    float graw[2][64];
    float braw[2][64];
    // prep scalars of the chunk being prepared
    float gcl[64];   // cumulative log2 decay
    float beta[64];
    float rk[64];    // 1/|k| (0 past the end)
    float rq[64];    // scale/|q|
    float rowA[64];  // beta rk 2^gcl
    float colS[64];  // rk 2^-gcl
    float cw[64];    // beta rk 2^gcl
    float mx[64];    // max(gcl, -100)
    float scan_carry;
    int fast;        // every gcl of the chunk is above -100: product-form decay
    // chain scalars per chunk parity
    float ce[2][64];  // rk 2^(glast - gcl)
    float eq[2][64];  // rq 2^mx
    float dec[2];     // 2^glast
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kDecayFloor = -100.f;     // log2 floor of the product-form decay factors
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColDS = 0;           // dS = K^T (hi + lo), all lanes, 64 columns
constexpr uint32_t kColR = 64;           // per-parity accumulators: 64 + 128 * parity
constexpr uint32_t kColKQ = 320;         // KK (lanes A) / QK (lanes B)
constexpr uint32_t kColT2 = 384;         // T2 (lanes A) / X_LL (lanes B)
constexpr uint32_t kHalfB = 16u << 16;   // lane offset of the second M=64 accumulator
// inside a parity region R: W[:, 0:64] lanes A and W[:, 64:128] lanes B at R; U -> VN lanes A
// and O = Q S + P' VN lanes B at R + 64.

enum : uint32_t { kBarPrep = 1, kBarChain = 2 };

// 8 fp32 values -> one 16-byte bf16 chunk of a swizzled panel row.
__device__ __forceinline__ void put_chunk(uint8_t* panel, uint32_t row, uint32_t chunk, const float* v) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(panel + sw128(row, chunk)) = raw;
}

__device__ __forceinline__ float sum_squares_row(const uint8_t* tile, uint32_t row) {
    float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int pnl = 0; pnl < 2; ++pnl)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 raw = *reinterpret_cast<const uint4*>(tile + pnl * kPanel + sw128(row, ch));
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(h[i]);
                ss[i] = fmaf(f.x, f.x, ss[i]);
                ss[i] = fmaf(f.y, f.y, ss[i]);
            }
        }
    return (ss[0] + ss[1]) + (ss[2] + ss[3]);
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__global__ void __launch_bounds__(384, 1) chunk_prefill_kernel(const __grid_constant__ ChunkParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ Shared sh;
    Bars& bar = sh.bar;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int kSlices = kHeadDim / kVS;
    const int hv = blockIdx.x / kSlices;
    const int v0 = (blockIdx.x % kSlices) * kVS;
    const int h = hv / p.rep;
    const int n = blockIdx.y;
    int64_t bos = 0, len = p.T, brow = n;
    if (p.cu_seqlens) {
        bos = p.cu_seqlens[n];
        len = p.cu_seqlens[n + 1] - bos;
        brow = 0;
    }
    const int nchunks = (int)((len + 63) / 64);
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;  // TMEM lane quarter of this warp
    const int half_row = 16 * (warp & 3) + (lane & 15);           // row of an M=64 accumulator
    const bool lanes_a = lane < 16;

    if (tid == 0) {
        sh.abort = 0;
        uint64_t* all = reinterpret_cast<uint64_t*>(&bar);
        for (uint32_t i = 0; i < sizeof(Bars) / sizeof(uint64_t); ++i) mbar_init(all + i, 1);
        fence_mbar_init();
        tma_prefetch_map(&p.tm_q);
        tma_prefetch_map(&p.tm_k);
        tma_prefetch_map(&p.tm_v);
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;
    auto wait = [&](uint64_t* b, uint32_t parity, int site) -> bool {
        return mbar_wait_or_abort(b, parity, site, &sh.abort);
    };
    auto fail = [&]() { atomicExch(&sh.abort, 1); };
    auto nvalid_of = [&](int c) -> int {
        const int64_t rest = len - 64 * (int64_t)c;
        return (int)(rest < 64 ? rest : 64);
    };

    if (warp == 0) {
        // ================================ loader ================================
        int issued[2] = {0, 0};
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1;
            if (c >= 2) {
                bool w = wait(&bar.kqv_empty[s], ((c >> 1) + 1) & 1, kSiteTmaLoad);
                w = w && wait(&bar.gates_empty[s], ((c >> 1) + 1) & 1, kSiteTmaLoad);
                if (!__all_sync(0xffffffffu, w)) {
                    fail();
                    break;
                }
            }
            const int t = (int)(bos + 64 * c);
            if (lane == 0) {
                mbar_arrive_expect_tx(&bar.kqv_full[s], 5 * kPanel);
                uint8_t* kt = sm + Smem::K + s * 2 * kPanel;
                uint8_t* qt = sm + Smem::Q + s * 2 * kPanel;
                tma_load_4d(kt, &p.tm_k, &bar.kqv_full[s], 0, h, t, (int)brow);
                tma_load_4d(kt + kPanel, &p.tm_k, &bar.kqv_full[s], 64, h, t, (int)brow);
                tma_load_4d(qt, &p.tm_q, &bar.kqv_full[s], 0, h, t, (int)brow);
                tma_load_4d(qt + kPanel, &p.tm_q, &bar.kqv_full[s], 64, h, t, (int)brow);
                tma_load_4d(sm + Smem::V + s * kPanel, &p.tm_v, &bar.kqv_full[s], v0, hv, t, (int)brow);
                issued[s] = c + 1;
            }
            const int nvalid = nvalid_of(c);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = 2 * lane + e;
                float gv = 0.f, bv = 0.f;
                if (j < nvalid) {
                    const int64_t gi = (brow * p.T + t + j) * p.HV + hv;
                    gv = p.g[gi];
                    bv = p.beta_f32 ? static_cast<const float*>(p.beta)[gi]
                                    : to_f32(static_cast<const bf16*>(p.beta)[gi]);
                }
                sh.graw[s][j] = gv;
                sh.braw[s][j] = bv;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar.gates_full[s]);
        }
        // let every tile this warp asked for land before the CTA can exit
        if (lane == 0)
            for (int s = 0; s < 2; ++s)
                if (issued[s]) mbar_wait(&bar.kqv_full[s], ((issued[s] - 1) >> 1) & 1, kSiteDrain);
    } else if (warp >= 4 && warp < 8) {
        // ================================ prep ================================
        const int pt = tid - 128;  // 0..127
        float* Af = reinterpret_cast<float*>(sm + Smem::AF);
        const uint32_t id_sq = make_idesc(64, 64, kFmtBF16, false, false);
        const uint32_t id_mn64 = make_idesc(64, 64, kFmtBF16, false, true);
        auto issue_kq = [&](int c) {
            const uint8_t* kt = sm + Smem::K + (c & 1) * 2 * kPanel;
            const uint8_t* qt = sm + Smem::Q + (c & 1) * 2 * kPanel;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t po = (kk >> 2) * kPanel, ko = (kk & 3) * 32;
                const uint64_t bd = sdesc_kmajor(kt + po, ko);
                mma_f16(tb + kColKQ, sdesc_kmajor(kt + po, ko), bd, id_sq, kk > 0);
                mma_f16(tb + kColKQ + kHalfB, sdesc_kmajor(qt + po, ko), bd, id_sq, kk > 0);
            }
            mma_commit(&bar.acc_kq);
        };
        bool issued_any = false;
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1;
            const uint32_t ph = c & 1, phs = (c >> 1) & 1;
            const int nvalid = nvalid_of(c);
            const uint8_t* kt = sm + Smem::K + s * 2 * kPanel;
            const uint8_t* qt = sm + Smem::Q + s * 2 * kPanel;
            bool ok = wait(&bar.gates_full[s], phs, kSiteTmaLoad) && wait(&bar.kqv_full[s], phs, kSiteTmaLoad);
            // the chain of chunk c-2 must be done with this parity's scalars and accumulators
            if (ok && c >= 2) ok = wait(&bar.o_free[s], ((c >> 1) + 1) & 1, kSiteMma);
            if (!named_sync_all(kBarPrep, 128, ok)) { fail(); break; }
            if (pt == 0) {  // KK, QK of this chunk; the norms below overlap them
                tc_fence_after();
                issue_kq(c);
                issued_any = true;
            }
            // ---- gates (scan in log2 units) and inverse norms
            float gsum = 0.f;
            if (pt < 64) {
                float x = sh.graw[s][pt] * kLog2e;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, x, o);
                    if (lane >= o) x += y;
                }
                gsum = x;
                if (pt == 31) sh.scan_carry = x;
                sh.beta[pt] = sh.braw[s][pt];
                const float inv = rsqrtf(sum_squares_row(kt, pt) + 1e-6f);
                sh.rk[pt] = pt < nvalid ? inv : 0.f;
            } else {
                const int r = pt - 64;
                sh.rq[r] = rsqrtf(sum_squares_row(qt, r) + 1e-6f) * p.scale;
            }
            named_sync(kBarPrep, 128);
            if (pt < 64) sh.gcl[pt] = pt >= 32 ? gsum + sh.scan_carry : gsum;
            named_sync(kBarPrep, 128);
            if (pt == 0) mbar_arrive(&bar.gates_empty[s]);
            if (pt < 64) {
                const float gl = sh.gcl[pt];
                const float glast = sh.gcl[63];
                const float rk = sh.rk[pt], bt = sh.beta[pt], rq = sh.rq[pt];
                const float mxv = fmaxf(gl, kDecayFloor);
                const float e_gl = exp2f(gl);
                sh.rowA[pt] = bt * rk * e_gl;
                sh.colS[pt] = rk * exp2f(-fmaxf(gl, kDecayFloor));
                sh.cw[pt] = bt * rk * e_gl;
                sh.mx[pt] = mxv;
                sh.ce[s][pt] = rk * exp2f(glast - gl);
                sh.eq[s][pt] = rq * exp2f(mxv);
                if (pt == 0) {
                    sh.dec[s] = exp2f(glast);
                    sh.fast = glast > kDecayFloor;
                }
            }
            named_sync(kBarPrep, 128);
            // ---- A (fp32 rows, from KK in lanes A) and P' (bf16 rows, from QK in lanes B)
            if (!named_sync_all(kBarPrep, 128, wait(&bar.acc_kq, ph, kSiteMma))) { fail(); break; }
            tc_fence_after();
            {
                const int i = half_row;
                const int lim = lanes_a ? i : i + 1;  // columns kept: j < lim
                const bool fast = sh.fast;
                const float rs_fast = lanes_a ? sh.rowA[i] : 1.f;
                const float gli = sh.gcl[i];
                const float rs_slow = lanes_a ? sh.beta[i] * sh.rk[i] : 1.f;
                const float shift = lanes_a ? 0.f : sh.mx[i];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float r[32];
                    tmem_ld32_wait(tb + kColKQ + lane_base + 32 * half, r);
                    if (fast) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            const float4 cs = ld4(&sh.colS[32 * half + j]);
                            r[j] *= rs_fast * cs.x;
                            r[j + 1] *= rs_fast * cs.y;
                            r[j + 2] *= rs_fast * cs.z;
                            r[j + 3] *= rs_fast * cs.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int col = 32 * half + j;
                            const float e = exp2f(fminf(gli - sh.gcl[col] - shift, 0.f));
                            r[j] *= rs_slow * sh.rk[col] * e;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = (32 * half + j) < lim ? r[j] : 0.f;
                    if (lanes_a) {
                        float* arow = Af + i * kAfStride + 32 * half;
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(arow + j) = make_float4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                    } else {
                        uint8_t* pm = sm + Smem::PM + s * kPanel;
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) put_chunk(pm, i, 4 * half + ch, r + 8 * ch);
                    }
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarPrep, 128);
            // ---- inverses of the four 16x16 diagonal blocks of I + A (two partial sums per row)
            {
                float x[16];
                const int b = pt >> 4, col = pt & 15;
                if (pt < 64) {
                    const float* blk = Af + 16 * b * kAfStride + 16 * b;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float a0 = 0.f, a1 = 0.f;
#pragma unroll
                        for (int j = 0; j < i; ++j) {
                            if (j & 1) a1 = fmaf(blk[i * kAfStride + j], x[j], a1);
                            else a0 = fmaf(blk[i * kAfStride + j], x[j], a0);
                        }
                        x[i] = (i == col) ? 1.f : (i > col ? -(a0 + a1) : 0.f);
                    }
                }
                named_sync(kBarPrep, 128);
                if (pt < 64) {
                    float* blk = Af + 16 * b * kAfStride + 16 * b;
#pragma unroll
                    for (int i = 0; i < 16; ++i) blk[i * kAfStride + col] = x[i];
                }
            }
            named_sync(kBarPrep, 128);
            // ---- 16 -> 32 merge inside each 32-block: X10 = -X11 (A10 X00)
            {
                const int blk = pt >> 6, e = pt & 63;
                const int i = e >> 2, j0 = (e & 3) * 4, r0 = 32 * blk;
                float t4[4] = {0.f, 0.f, 0.f, 0.f};
                const float* arow = Af + (r0 + 16 + i) * kAfStride + r0;
#pragma unroll
                for (int kx = 0; kx < 16; kx += 4) {
                    const float4 a = ld4(arow + kx);
                    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 xv = ld4(&Af[(r0 + kx + q) * kAfStride + r0 + j0]);
                        t4[0] = fmaf(av[q], xv.x, t4[0]); t4[1] = fmaf(av[q], xv.y, t4[1]);
                        t4[2] = fmaf(av[q], xv.z, t4[2]); t4[3] = fmaf(av[q], xv.w, t4[3]);
                    }
                }
                named_sync(kBarPrep, 128);
                *reinterpret_cast<float4*>(&Af[(r0 + 16 + i) * kAfStride + r0 + j0]) = make_float4(t4[0], t4[1], t4[2], t4[3]);
                named_sync(kBarPrep, 128);
                float x4[4] = {0.f, 0.f, 0.f, 0.f};
                const float* xrow = Af + (r0 + 16 + i) * kAfStride + r0 + 16;
#pragma unroll
                for (int kx = 0; kx < 16; kx += 4) {
                    const float4 a = ld4(xrow + kx);
                    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 tv = ld4(&Af[(r0 + 16 + kx + q) * kAfStride + r0 + j0]);
                        x4[0] = fmaf(av[q], tv.x, x4[0]); x4[1] = fmaf(av[q], tv.y, x4[1]);
                        x4[2] = fmaf(av[q], tv.z, x4[2]); x4[3] = fmaf(av[q], tv.w, x4[3]);
                    }
                }
                named_sync(kBarPrep, 128);
                *reinterpret_cast<float4*>(&Af[(r0 + 16 + i) * kAfStride + r0 + j0]) =
                    make_float4(-x4[0], -x4[1], -x4[2], -x4[3]);
            }
            named_sync(kBarPrep, 128);
            // ---- bf16 operands of the 32 -> 64 merge: E32 (lower-left block of A) and D32
            {
                const int i = pt & 63, hf = pt >> 6;  // two threads per row, 32 columns each
                const float* arow = Af + i * kAfStride + 32 * hf;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    float e8[8], d8[8];
                    const float4 a0 = ld4(arow + 8 * cc), a1 = ld4(arow + 8 * cc + 4);
                    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int j = 32 * hf + 8 * cc + q;
                        e8[q] = (i >= 32 && j < 32) ? av[q] : 0.f;
                        d8[q] = ((i >> 5) == (j >> 5) && j <= i) ? av[q] : 0.f;
                    }
                    put_chunk(sm + Smem::AU, i, 4 * hf + cc, e8);
                    put_chunk(sm + Smem::AW, i, 4 * hf + cc, d8);
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarPrep, 128);
            if (pt == 0) {  // T2 = E32 D32 (lanes A)
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16(tb + kColT2, sdesc_kmajor(sm + Smem::AU, kk * 32),
                            sdesc_mnmajor(sm + Smem::AW + kk * 2048, kPanel), id_mn64, kk > 0);
                mma_commit(&bar.acc_t2);
            }
            // ---- T2 -> bf16 operand
            if (!named_sync_all(kBarPrep, 128, wait(&bar.acc_t2, ph, kSiteMma))) { fail(); break; }
            tc_fence_after();
            {
                float r[64];
                tmem_ld64_wait(tb + kColT2 + lane_base, r);
                if (lanes_a)
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch) put_chunk(sm + Smem::T2, half_row, ch, r + 8 * ch);
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarPrep, 128);
            if (pt == 0) {  // X_LL = D32 T2 (lanes B)
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16(tb + kColT2 + kHalfB, sdesc_kmajor(sm + Smem::AW, kk * 32),
                            sdesc_mnmajor(sm + Smem::T2 + kk * 2048, kPanel), id_mn64, kk > 0);
                mma_commit(&bar.acc_x);
            }
            // ---- X = D32 - X_LL; two column-scaled bf16 copies feed U and W. Row i is shared
            // by lanes l (columns 32-63) and l + 16 (columns 0-31, whose TMEM lanes hold X_LL).
            if (!named_sync_all(kBarPrep, 128, wait(&bar.acc_x, ph, kSiteMma))) { fail(); break; }
            tc_fence_after();
            {
                const int i = half_row;
                const int cbase = lanes_a ? 32 : 0;
                float r[32];
                tmem_ld32_wait(tb + kColT2 + lane_base, r);  // lanes B: X_LL columns 0-31
                const float* arow = Af + i * kAfStride + cbase;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    float xu[8], xw[8];
                    const float4 a0 = ld4(arow + 8 * cc), a1 = ld4(arow + 8 * cc + 4);
                    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const float4 b0 = ld4(&sh.beta[cbase + 8 * cc]), b1 = ld4(&sh.beta[cbase + 8 * cc + 4]);
                    const float4 w0 = ld4(&sh.cw[cbase + 8 * cc]), w1 = ld4(&sh.cw[cbase + 8 * cc + 4]);
                    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int col = cbase + 8 * cc + q;
                        float xv;
                        if (col > i) xv = 0.f;
                        else if (!lanes_a && i >= 32) xv = -r[8 * cc + q];
                        else xv = av[q];
                        xu[q] = xv * bv[q];
                        xw[q] = xv * wv[q];
                    }
                    put_chunk(sm + Smem::AU, i, cbase / 8 + cc, xu);
                    put_chunk(sm + Smem::AW, i, cbase / 8 + cc, xw);
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarPrep, 128);
            if (pt == 0) {
                // W[:, 0:64] (lanes A) and W[:, 64:128] (lanes B) = (X diag(cw)) K; U = (X diag(beta)) V
                tc_fence_after();
                const uint32_t tR = tb + kColR + 128 * s;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = sdesc_kmajor(sm + Smem::AW, kk * 32);
                    mma_f16(tR, ad, sdesc_mnmajor(kt + kk * 2048, kPanel), id_mn64, kk > 0);
                    mma_f16(tR + kHalfB, ad, sdesc_mnmajor(kt + kPanel + kk * 2048, kPanel), id_mn64, kk > 0);
                    mma_f16(tR + 64, sdesc_kmajor(sm + Smem::AU, kk * 32),
                            sdesc_mnmajor(sm + Smem::V + s * kPanel + kk * 2048, kPanel), id_mn64, kk > 0);
                }
                mma_commit(&bar.acc_wu[s]);
            }
            // ---- W -> bf16 operand (lanes A: d 0-63, lanes B: d 64-127)
            if (!named_sync_all(kBarPrep, 128, wait(&bar.acc_wu[s], phs, kSiteMma))) { fail(); break; }
            tc_fence_after();
            {
                float r[64];
                tmem_ld64_wait(tb + kColR + 128 * s + lane_base, r);
                uint8_t* panel = sm + Smem::WB + s * 2 * kPanel + (lanes_a ? 0 : kPanel);
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) put_chunk(panel, half_row, ch, r + 8 * ch);
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarPrep, 128);
            if (pt == 0) mbar_arrive(&bar.wb_ready);
        }
        // every MMA this warpgroup issued is complete before TMEM can be freed
        if (pt == 0 && issued_any) {
            mma_commit(&bar.drain_prep);
            mbar_wait(&bar.drain_prep, 0, kSiteDrain);
        }
    } else if (warp >= 8) {
        // ================================ chain ================================
        const int ct = tid - 256;  // 0..127: the state row (and TMEM lane) of this thread
        const int d = ct;
        uint8_t* sbp = sm + Smem::SB + (d >> 6) * kPanel;
        const uint32_t sb_off = (d & 7) * 2;
        const uint32_t sb_chunk = (d & 63) >> 3;
        const int64_t state_row = (((int64_t)n * p.HV + hv) * kHeadDim + d) * kHeadDim + v0;
        const uint32_t id_vn = make_idesc(64, kVS, kFmtBF16, false, false, true);
        const uint32_t id_o1 = make_idesc(64, kVS, kFmtBF16, false, false);
        const uint32_t id_s = make_idesc(128, kVS, kFmtBF16, true, true);
        const uint32_t id_o2 = make_idesc(64, kVS, kFmtBF16, false, true);
        float S[kVS];
        if (p.h0) {
#pragma unroll
            for (int j = 0; j < kVS; j += 4) {
                const float4 x4 = ld4(p.h0 + state_row + j);
                S[j] = x4.x; S[j + 1] = x4.y; S[j + 2] = x4.z; S[j + 3] = x4.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < kVS; ++j) S[j] = 0.f;
        }
        if (nchunks == 0) {
            if (p.ht)
#pragma unroll
                for (int j = 0; j < kVS; j += 4)
                    *reinterpret_cast<float4*>(p.ht + state_row + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
        } else {
#pragma unroll
            for (int v = 0; v < kVS; ++v)
                *reinterpret_cast<bf16*>(sbp + sw128(v, sb_chunk) + sb_off) = __float2bfloat16_rn(S[v]);
        }
        fence_async_smem();
        named_sync(kBarChain, 128);
        bool issued_any = false;
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1;
            const uint32_t ph = c & 1, phs = (c >> 1) & 1;
            const uint32_t tR = tb + kColR + 128 * s;
            const uint8_t* kt = sm + Smem::K + s * 2 * kPanel;
            const uint8_t* qt = sm + Smem::Q + s * 2 * kPanel;
            const int64_t t0 = bos + 64 * (int64_t)c;
            const int nvalid = nvalid_of(c);
            // ---- VN = U - W S (lanes A, onto U); O = Q S (lanes B)
            if (!named_sync_all(kBarChain, 128, wait(&bar.wb_ready, ph, kSiteMma))) { fail(); break; }
            if (ct == 0) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t po = (kk >> 2) * kPanel, ko = (kk & 3) * 32;
                    const uint64_t bd = sdesc_kmajor(sm + Smem::SB + po, ko);
                    mma_f16(tR + 64, sdesc_kmajor(sm + Smem::WB + s * 2 * kPanel + po, ko), bd, id_vn, 1);
                    mma_f16(tR + 64 + kHalfB, sdesc_kmajor(qt + po, ko), bd, id_o1, kk > 0);
                }
                mma_commit(&bar.acc_vn[s]);
                issued_any = true;
            }
            if (!named_sync_all(kBarChain, 128, wait(&bar.acc_vn[s], phs, kSiteMma))) { fail(); break; }
            tc_fence_after();
            // ---- VN -> bf16 VN and the split ce VN
            {
                const int i = half_row;
                const float cei = sh.ce[s][i];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float r[32];
                    tmem_ld32_wait(tR + 64 + lane_base + 32 * half, r);  // lanes A: VN rows
                    if (lanes_a) {
#pragma unroll
                        for (int cc = 0; cc < 4; ++cc) {
                            float hi[8], lo[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const float x = cei * r[8 * cc + j];
                                hi[j] = round_bf16(x);
                                lo[j] = x - hi[j];
                            }
                            const int ch = 4 * half + cc;
                            put_chunk(sm + Smem::VBF, i, ch, r + 8 * cc);
                            put_chunk(sm + Smem::VHI, i, ch, hi);
                            put_chunk(sm + Smem::VLO, i, ch, lo);
                        }
                    }
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarChain, 128);
            if (ct == 0) {
                // dS = K^T hi + K^T lo (all lanes, fresh); O += P' VN (lanes B)
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = sdesc_mnmajor(kt + kk * 2048, kPanel);
                    mma_f16(tb + kColDS, ad, sdesc_mnmajor(sm + Smem::VHI + kk * 2048, kPanel), id_s, kk > 0);
                    mma_f16(tb + kColDS, ad, sdesc_mnmajor(sm + Smem::VLO + kk * 2048, kPanel), id_s, 1);
                    mma_f16(tR + 64 + kHalfB, sdesc_kmajor(sm + Smem::PM + s * kPanel, kk * 32),
                            sdesc_mnmajor(sm + Smem::VBF + kk * 2048, kPanel), id_o2, 1);
                }
                mma_commit(&bar.acc_s);
                mma_commit(&bar.kqv_empty[s]);
            }
            if (!named_sync_all(kBarChain, 128, wait(&bar.acc_s, ph, kSiteMma))) { fail(); break; }
            tc_fence_after();
            // ---- S <- 2^glast S + dS; o = eq O (32 columns at a time keeps the state in registers)
            {
                const float decay = sh.dec[s];
                const bool last = c + 1 == nchunks;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float r[32];
                    tmem_ld32_wait(tb + kColDS + lane_base + 32 * half, r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) S[32 * half + j] = fmaf(decay, S[32 * half + j], r[j]);
                }
                if (last) {
                    if (p.ht)
#pragma unroll
                        for (int j = 0; j < kVS; j += 4)
                            *reinterpret_cast<float4*>(p.ht + state_row + j) =
                                make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
                } else {
#pragma unroll
                    for (int v = 0; v < kVS; ++v)
                        *reinterpret_cast<bf16*>(sbp + sw128(v, sb_chunk) + sb_off) = __float2bfloat16_rn(S[v]);
                }
                const int i = half_row;
                const bool store = !lanes_a && i < nvalid;
                const float eqi = sh.eq[s][i];
                bf16* orow = p.o + ((brow * p.T + t0 + i) * p.HV + hv) * kHeadDim + v0;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float r[32];
                    tmem_ld32_wait(tR + 64 + lane_base + 32 * half, r);  // lanes B: O rows
                    if (store) {
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            uint4 raw;
                            __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                hh[j] = __floats2bfloat162_rn(eqi * r[8 * ch + 2 * j], eqi * r[8 * ch + 2 * j + 1]);
                            *reinterpret_cast<uint4*>(orow + 32 * half + 8 * ch) = raw;
                        }
                    }
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarChain, 128);
            if (ct == 0) mbar_arrive(&bar.o_free[s]);
        }
        if (ct == 0 && issued_any) {
            mma_commit(&bar.drain_chain);
            mbar_wait(&bar.drain_chain, 0, kSiteDrain);
        }
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
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(chunk_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Smem::BYTES) != cudaSuccess)
            return GDN_ERR_LAUNCH;
        configured = true;
    }
    dim3 grid((unsigned)(p.HV * (kHeadDim / kVS)), (unsigned)a.nseq);
    chunk_prefill_kernel<<<grid, 384, Smem::BYTES, s>>>(p);
    return launch_status();
}

}  // namespace gdn
