// Chunked gated-delta-rule prefill on tcgen05 tensor cores (chunk 64, WY/UT form).
//
// Reference semantics: torch_chunk_gated_delta_rule, model/model.py:242-286 (fp32 eager;
// fla's chunk_gated_delta_rule on CUDA, model/model.py:289-294), with varlen packing
// through cu_seqlens as in fla 0.5.x.
//
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
// The intra-chunk output is folded into the inter-chunk accumulator: with eq_i = rq_i e^{gc_i},
// o_i = eq_i (Q S + P' VN)_i where P'_ij = rk_j QK_ij e^{-gc_j}; e^{gc_i - gc_j} is formed as
// e^{gc_i} e^{-gc_j} while the chunk's decay stays above 2^-100 and element by element otherwise.
//
// Two kernels:
//   chunk_factor_kernel  one CTA per (value head, chunk), all chunks at once: everything that
//                        does not depend on the state (norms, gates, P', X, W) goes into a
//                        33 KB record per (value head, chunk) in a caller-provided workspace,
//                        laid out as the scan kernel's shared-memory stage.
//   chunk_scan_kernel    one CTA per (sequence, value head, 64-column slice of the state),
//                        walking the chunks in order with the fp32 state slice in registers.
//                        A loader warp streams K/Q/V tiles (TMA) and records (bulk copy); two
//                        chain warpgroups (one per 32-column half of the slice) run U,
//                        VN = U - W S, dS = K^T VN and the state update; an epilogue warpgroup
//                        drains O = Q S + P' VN to global memory. The chain's critical path per
//                        chunk is two MMA round trips (W S, then dS) and two half-width readouts;
//                        the output MMAs are committed after them and never waited on there.
//
// Every wait is bounded (sm100.cuh): a wait that gives up raises the device error word and
// the CTA's abort flag; every role then leaves its loop, the loader waits for the copies it
// started, the issuer for the MMAs it issued, TMEM is freed and the CTA returns.

#include "common.cuh"
#include "gates.cuh"
#include "launch.h"
#include "sm100.cuh"
#include "tensor_map.h"

namespace gdn {

using namespace sm100;

constexpr int kVS = 64;                       // value columns per scan CTA
constexpr int kSlices = kHeadDim / kVS;         // scan CTAs per (sequence, value head)
constexpr uint32_t kPanel = 64 * 128;         // one 128-byte-swizzled panel of 64 rows
constexpr int kAfStride = 68;                 // fp32 row stride of the inverse workspace

// ---- per-(value head, chunk) record, produced by the factor kernel, consumed by the scan kernel
struct RecScalars {
    float ce[64];  // rk 2^(glast - gcl)
    float eq[64];  // rq 2^max(gcl, -100)
    float dec;     // 2^glast
    float pad[127];
};
static_assert(sizeof(RecScalars) == 1024, "record scalars are one 1 KB block");

constexpr uint32_t kRecW = 0;               // W: bf16, K-major, two d-panels (rows = tokens)
constexpr uint32_t kRecXB = 2 * kPanel;     // X diag(beta): bf16, K-major
constexpr uint32_t kRecPM = 3 * kPanel;     // P': bf16, K-major
constexpr uint32_t kRecSc = 4 * kPanel;     // RecScalars
constexpr uint32_t kRecBytes = kRecSc + sizeof(RecScalars);

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kDecayFloor = -100.f;     // log2 floor of the product-form decay factors
constexpr uint32_t kHalfB = 16u << 16;    // lane offset of the second M=64 accumulator

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

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// =========================================================================================
// factor kernel
// =========================================================================================
struct FactorParams {
    CUtensorMap tm_q;  // 4-D (128, H, T, B) bf16, box (64, 1, 64, 1), 128-byte swizzle
    CUtensorMap tm_k;
    const float* g;    // [B, T, HV]
    const void* beta;  // [B, T, HV] bf16 or fp32
    int beta_f32;
    const int32_t* cu_seqlens;
    uint8_t* records;  // [slots, HV] records
    uint32_t* ready;   // [slots, HV] flags set once a record is written (fused launch), or null
    int64_t slots;
    int64_t T;
    int nseq, ncd;     // sequences; chunks per row of the dense layout
    int HV, rep;
    float scale;
    GateInputs gates;  // beta and g from the raw projections when gates.b is set
};

struct FSmem {
    static constexpr uint32_t K = 0;                   // K tile (two d-panels); W staging at the end
    static constexpr uint32_t Q = K + 2 * kPanel;      // Q tile; P' and T2 once KK / QK are done
    static constexpr uint32_t PM = Q;
    static constexpr uint32_t T2 = Q + kPanel;         // E32 D32 (bf16, MN-major)
    static constexpr uint32_t AU = Q + 2 * kPanel;     // X diag(beta); E32 during the inverse
    static constexpr uint32_t AW = AU + kPanel;        // X diag(cw); D32 during the inverse
    static constexpr uint32_t AF = AW + kPanel;        // fp32 [64][kAfStride]
    static constexpr uint32_t END = AF + 64 * kAfStride * 4;
    static constexpr uint32_t BYTES = END + 1024;      // + alignment slack
};

struct FShared {
    uint64_t tma, acc_kq, acc_t2, acc_x, acc_w, drain;
    uint32_t tmem_base;
    // read with 16-byte vector loads: every array starts on a 16-byte boundary
    alignas(16) float graw[64];
    alignas(16) float braw[64];
    alignas(16) float gcl[64];   // cumulative log2 decay
    alignas(16) float beta[64];
    alignas(16) float rk[64];    // 1/|k| (0 past the end)
    alignas(16) float rq[64];    // scale/|q|
    alignas(16) float rowA[64];  // beta rk 2^gcl
    alignas(16) float colS[64];  // rk 2^-max(gcl, -100)
    alignas(16) float cw[64];    // beta rk 2^gcl
    alignas(16) float mx[64];    // max(gcl, -100)
    float scan_carry;
    int fast;        // every gcl of the chunk is above -100: product-form decay
    alignas(128) RecScalars rs;
};
static_assert(offsetof(FShared, colS) % 16 == 0 && offsetof(FShared, beta) % 16 == 0 &&
                  offsetof(FShared, cw) % 16 == 0 && offsetof(FShared, rs) % 16 == 0,
              "vector-loaded arrays are 16-byte aligned");

constexpr uint32_t kFactorTmemCols = 128;
constexpr uint32_t kColKQ = 0;    // KK (lanes A) / QK (lanes B); W halves (lanes A / B) later
constexpr uint32_t kColT2 = 64;   // T2 (lanes A) / X_LL (lanes B)
enum : uint32_t { kBarFactor = 1, kBarChain = 2, kBarEpi = 3 };

// Release / acquire of a record's ready flag between the factor and the scan roles of the fused
// launch (the record itself moves through the async proxy: bulk stores, then bulk loads).
__device__ __forceinline__ void flag_release(uint32_t* flag) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(1u) : "memory");
}

__device__ __forceinline__ uint32_t flag_acquire(const uint32_t* flag) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    return v;
}

// One factor unit, i.e. one (value head, chunk slot), run by the 128 threads of one warpgroup
// (pt = 0..127, named barrier `bar`). The barriers in `sh` are initialised once per warpgroup
// and complete once per unit: `ph` is this unit's phase parity. Result: 1 when the unit ran
// (its barrier phases completed), 0 for a slot no chunk maps to, -1 once a bounded wait has
// given up (the device error word is set; the warpgroup then stops).
//
// The slot of chunk c of sequence n: n * ncd + c for the dense layout; cu[n] / 64 + n + c for
// a packed batch. Slots of different sequences never collide because a sequence of length L
// starting at token b has at most floor((b + L) / 64) - floor(b / 64) + 1 chunks.
__device__ __forceinline__ int factor_unit(const FactorParams& p, int64_t unit, FShared& sh, uint8_t* sm, uint32_t tb,
                                           uint32_t bar, int pt, uint32_t ph) {
    const int warp = pt >> 5, lane = pt & 31;
    const int hv = (int)(unit % p.HV);
    const int64_t slot = unit / p.HV;
    const int h = hv / p.rep;
    int64_t bos = 0, len = p.T, brow = 0, c = 0;
    if (p.cu_seqlens == nullptr) {
        brow = slot / p.ncd;
        c = slot % p.ncd;
    } else {
        int lo = 0, hi = p.nseq - 1;  // last sequence whose first slot is <= slot
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.cu_seqlens[mid] / 64 + (int64_t)mid <= slot) lo = mid;
            else hi = mid - 1;
        }
        bos = p.cu_seqlens[lo];
        len = p.cu_seqlens[lo + 1] - bos;
        c = slot - (bos / 64 + lo);
        if (c < 0 || 64 * c >= len) return 0;  // a slot no chunk maps to (uniform over the warpgroup)
    }
    const int t = (int)(bos + 64 * c);
    const int nvalid = (int)(len - 64 * c < 64 ? len - 64 * c : 64);
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const int half_row = 16 * warp + (lane & 15);
    const bool lanes_a = lane < 16;
    uint8_t* kt = sm + FSmem::K;
    uint8_t* qt = sm + FSmem::Q;
    float* Af = reinterpret_cast<float*>(sm + FSmem::AF);

    if (pt == 0) {
        mbar_arrive_expect_tx(&sh.tma, 4 * kPanel);
        tma_load_4d(kt, &p.tm_k, &sh.tma, 0, h, t, (int)brow);
        tma_load_4d(kt + kPanel, &p.tm_k, &sh.tma, 64, h, t, (int)brow);
        tma_load_4d(qt, &p.tm_q, &sh.tma, 0, h, t, (int)brow);
        tma_load_4d(qt + kPanel, &p.tm_q, &sh.tma, 64, h, t, (int)brow);
    }
    if (pt < 64) {
        float gv = 0.f, bv = 0.f;
        if (pt < nvalid) {
            const int64_t gi = (brow * p.T + t + pt) * p.HV + hv;
            if (p.gates.b) {
                delta_gate(p.gates, brow * p.T + t + pt, hv, bv, gv);
            } else {
                gv = p.g[gi];
                bv = p.beta_f32 ? static_cast<const float*>(p.beta)[gi] : to_f32(static_cast<const bf16*>(p.beta)[gi]);
            }
        }
        sh.graw[pt] = gv;
        sh.braw[pt] = bv;
    }
    named_sync(bar, 128);
    const uint32_t id_sq = make_idesc(64, 64, kFmtBF16, false, false);
    const uint32_t id_mn64 = make_idesc(64, 64, kFmtBF16, false, true);
    bool tiles_landed = false, mma_issued = false;

    do {
        tiles_landed = named_sync_all(bar, 128, mbar_wait(&sh.tma, ph, kSiteTmaLoad));
        if (!tiles_landed) break;
        // shared-memory descriptors, built once: each MMA below only adds a byte offset
        const uint64_t dK = sdesc_kmajor(kt, 0), dQ = sdesc_kmajor(qt, 0);
        const uint64_t dKmn = sdesc_mnmajor(kt, kPanel);
        const uint64_t dAU = sdesc_kmajor(sm + FSmem::AU, 0), dAW = sdesc_kmajor(sm + FSmem::AW, 0);
        const uint64_t dAWmn = sdesc_mnmajor(sm + FSmem::AW, kPanel), dT2mn = sdesc_mnmajor(sm + FSmem::T2, kPanel);
        if (pt == 0) {  // KK, QK; the norms below overlap them
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t off = (kk >> 2) * kPanel + (kk & 3) * 32;
                const uint64_t bd = sdesc_add(dK, off);
                mma_f16(tb + kColKQ, bd, bd, id_sq, kk > 0);
                mma_f16(tb + kColKQ + kHalfB, sdesc_add(dQ, off), bd, id_sq, kk > 0);
            }
            mma_commit(&sh.acc_kq);
            mma_issued = true;
        }
        // ---- gates (scan in log2 units) and inverse norms
        float gsum = 0.f;
        if (pt < 64) {
            float x = sh.graw[pt] * kLog2e;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            gsum = x;
            if (pt == 31) sh.scan_carry = x;
            sh.beta[pt] = sh.braw[pt];
            const float inv = rsqrtf(sum_squares_row(kt, pt) + 1e-6f);
            sh.rk[pt] = pt < nvalid ? inv : 0.f;
        } else {
            const int r = pt - 64;
            sh.rq[r] = rsqrtf(sum_squares_row(qt, r) + 1e-6f) * p.scale;
        }
        named_sync(bar, 128);
        if (pt < 64) sh.gcl[pt] = pt >= 32 ? gsum + sh.scan_carry : gsum;
        named_sync(bar, 128);
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
            sh.rs.ce[pt] = rk * exp2f(glast - gl);
            sh.rs.eq[pt] = rq * exp2f(mxv);
            if (pt == 0) {
                sh.rs.dec = exp2f(glast);
                sh.fast = glast > kDecayFloor;
            }
        }
        named_sync(bar, 128);
        // ---- A (fp32 rows, from KK in lanes A) and P' (bf16 rows, from QK in lanes B)
        if (!named_sync_all(bar, 128, mbar_wait(&sh.acc_kq, ph, kSiteMma))) break;
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
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) put_chunk(sm + FSmem::PM, i, 4 * half + ch, r + 8 * ch);
                }
            }
        }
        tc_fence_before();
        named_sync(bar, 128);
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
            named_sync(bar, 128);
            if (pt < 64) {
                float* blk = Af + 16 * b * kAfStride + 16 * b;
#pragma unroll
                for (int i = 0; i < 16; ++i) blk[i * kAfStride + col] = x[i];
            }
        }
        named_sync(bar, 128);
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
            named_sync(bar, 128);
            *reinterpret_cast<float4*>(&Af[(r0 + 16 + i) * kAfStride + r0 + j0]) = make_float4(t4[0], t4[1], t4[2], t4[3]);
            named_sync(bar, 128);
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
            named_sync(bar, 128);
            *reinterpret_cast<float4*>(&Af[(r0 + 16 + i) * kAfStride + r0 + j0]) =
                make_float4(-x4[0], -x4[1], -x4[2], -x4[3]);
        }
        named_sync(bar, 128);
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
                put_chunk(sm + FSmem::AU, i, 4 * hf + cc, e8);
                put_chunk(sm + FSmem::AW, i, 4 * hf + cc, d8);
            }
        }
        fence_async_smem();
        tc_fence_before();
        named_sync(bar, 128);
        if (pt == 0) {  // T2 = E32 D32 (lanes A)
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_f16(tb + kColT2, sdesc_add(dAU, kk * 32), sdesc_add(dAWmn, kk * 2048), id_mn64, kk > 0);
            mma_commit(&sh.acc_t2);
        }
        // ---- T2 -> bf16 operand
        if (!named_sync_all(bar, 128, mbar_wait(&sh.acc_t2, ph, kSiteMma))) break;
        tc_fence_after();
        {
            float r[64];
            tmem_ld64_wait(tb + kColT2 + lane_base, r);
            if (lanes_a)
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) put_chunk(sm + FSmem::T2, half_row, ch, r + 8 * ch);
        }
        fence_async_smem();
        tc_fence_before();
        named_sync(bar, 128);
        if (pt == 0) {  // X_LL = D32 T2 (lanes B)
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_f16(tb + kColT2 + kHalfB, sdesc_add(dAW, kk * 32), sdesc_add(dT2mn, kk * 2048), id_mn64, kk > 0);
            mma_commit(&sh.acc_x);
        }
        // ---- X = D32 - X_LL; two column-scaled bf16 copies: X diag(beta) (record) and X diag(cw)
        // (W product). Row i is shared by lanes l (columns 32-63) and l + 16 (columns 0-31, whose
        // TMEM lanes hold X_LL).
        if (!named_sync_all(bar, 128, mbar_wait(&sh.acc_x, ph, kSiteMma))) break;
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
                put_chunk(sm + FSmem::AU, i, cbase / 8 + cc, xu);
                put_chunk(sm + FSmem::AW, i, cbase / 8 + cc, xw);
            }
        }
        fence_async_smem();
        tc_fence_before();
        named_sync(bar, 128);
        if (pt == 0) {  // W[:, 0:64] (lanes A) and W[:, 64:128] (lanes B) = (X diag(cw)) K
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = sdesc_add(dAW, kk * 32);
                mma_f16(tb + kColKQ, ad, sdesc_add(dKmn, kk * 2048), id_mn64, kk > 0);
                mma_f16(tb + kColKQ + kHalfB, ad, sdesc_add(dKmn, kPanel + kk * 2048), id_mn64, kk > 0);
            }
            mma_commit(&sh.acc_w);
        }
        // ---- W -> bf16 (lanes A: d 0-63, lanes B: d 64-127) into the dead K tile, then the
        // record goes out with four bulk stores
        if (!named_sync_all(bar, 128, mbar_wait(&sh.acc_w, ph, kSiteMma))) break;
        tc_fence_after();
        {
            float r[64];
            tmem_ld64_wait(tb + kColKQ + lane_base, r);
            uint8_t* panel = kt + (lanes_a ? 0 : kPanel);
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) put_chunk(panel, half_row, ch, r + 8 * ch);
        }
        fence_async_smem();
        named_sync(bar, 128);
        if (pt == 0) {
            uint8_t* rec = p.records + ((int64_t)slot * p.HV + hv) * (int64_t)kRecBytes;
            bulk_store(rec + kRecW, kt, 2 * kPanel);
            bulk_store(rec + kRecXB, sm + FSmem::AU, kPanel);
            bulk_store(rec + kRecPM, sm + FSmem::PM, kPanel);
            bulk_store(rec + kRecSc, &sh.rs, sizeof(RecScalars));
            bulk_commit();
            bulk_wait_all();
            if (p.ready) flag_release(p.ready + slot * p.HV + hv);
        }
        tc_fence_before();
        named_sync(bar, 128);  // the next unit reuses the shared memory and TMEM
        return 1;
    } while (false);

    // a wait gave up: let this unit's copies and products finish before the caller frees TMEM
    if (pt == 0) {
        if (!tiles_landed) mbar_wait(&sh.tma, ph, kSiteDrain);
        if (mma_issued) {
            mma_commit(&sh.drain);
            mbar_wait(&sh.drain, 0, kSiteDrain);
        }
    }
    return -1;
}

// Units of the fused launch in chunk-major order: u -> (chunk c, sequence n, value head hv), so
// that chunk c of every sequence comes before any chunk c + 1. Returns the (slot * HV + hv) unit,
// or -1 where sequence n has no chunk c. u runs below ncd * nseq * HV.
__device__ __forceinline__ int64_t chunk_major_unit(const FactorParams& p, int64_t u) {
    const int64_t per_chunk = (int64_t)p.nseq * p.HV;
    const int64_t c = u / per_chunk;
    const int64_t r = u - c * per_chunk;
    const int n = (int)(r / p.HV), hv = (int)(r - (int64_t)n * p.HV);
    int64_t slot = (int64_t)n * p.ncd + c;
    if (p.cu_seqlens) {
        const int64_t bos = p.cu_seqlens[n], len = p.cu_seqlens[n + 1] - bos;
        if (64 * c >= len) return -1;
        slot = bos / 64 + n + c;
    }
    return slot * p.HV + hv;
}

// One warpgroup working through units first, first + stride, ... below total, in order (in
// chunk-major order when `chunk_major`, else u is the unit itself). `relinquish` gives up the
// CTA's right to allocate more TMEM once this warpgroup has its columns, so that the next CTA
// on the SM can allocate without waiting; a CTA whose other warpgroups still allocate passes
// false.
__device__ __forceinline__ void factor_worker(const FactorParams& p, FShared& sh, uint8_t* sm, uint32_t bar, int pt,
                                              int64_t first, int64_t stride, int64_t total, bool relinquish,
                                              bool chunk_major) {
    if (pt == 0) {
        mbar_init(&sh.tma, 1);
        mbar_init(&sh.acc_kq, 1);
        mbar_init(&sh.acc_t2, 1);
        mbar_init(&sh.acc_x, 1);
        mbar_init(&sh.acc_w, 1);
        mbar_init(&sh.drain, 1);
        fence_mbar_init();
    }
    if (pt < 32) {
        tmem_alloc(&sh.tmem_base, kFactorTmemCols);
        if (relinquish) tmem_relinquish();
    }
    tc_fence_before();
    named_sync(bar, 128);
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;
    uint32_t ph = 0;
    for (int64_t u = first; u < total; u += stride) {
        const int64_t unit = chunk_major ? chunk_major_unit(p, u) : u;
        if (unit < 0) continue;
        const int r = factor_unit(p, unit, sh, sm, tb, bar, pt, ph);
        if (r < 0) break;
        ph ^= (uint32_t)r;
    }
    tc_fence_before();
    named_sync(bar, 128);
    if (pt < 32) tmem_dealloc(tb, kFactorTmemCols);
}

__global__ void __launch_bounds__(128, 3) chunk_factor_kernel(const __grid_constant__ FactorParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ FShared sh;
    factor_worker(p, sh, align1024(smem_raw), kBarFactor, threadIdx.x, blockIdx.x, gridDim.x, (int64_t)gridDim.x, true,
                  false);
}

// =========================================================================================
// scan kernel
// =========================================================================================
struct ScanParams {
    CUtensorMap tm_q;  // 4-D (128, H, T, B) bf16, box (64, 1, 64, 1), 128-byte swizzle
    CUtensorMap tm_k;
    CUtensorMap tm_v;  // 4-D (128, HV, T, B)
    const float* h0;   // [N, HV, 128, 128] or null
    float* ht;         // [N, HV, 128, 128] or null
    bf16* o;           // [B, T, HV, 128]
    const int32_t* cu_seqlens;
    const uint8_t* records;
    const uint32_t* ready;  // per-record flags to wait for (fused launch), or null
    const int32_t* order;   // packed batch: sequences longest first (grid row -> sequence), or null
    int64_t T;
    int ncd;
    int HV, rep;
};

// Waits (bounded, backing off) until the factor role has published a record.
__device__ __forceinline__ bool wait_ready(const uint32_t* flag, const int* abort) {
    uint32_t sleep_ns = 32;
    const long long start = clock64();
    while (!flag_acquire(flag)) {
        if (*reinterpret_cast<const volatile int*>(abort)) return false;
        if (clock64() - start > kWaitCycles) {
            raise_device_error(kSiteReady);
            return false;
        }
        __nanosleep(sleep_ns);
        sleep_ns = sleep_ns < 1024 ? 2 * sleep_ns : 1024;
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the bulk loads below read the record
    return true;
}

// One pipeline stage (81 KB). Three 128-row K-major operands stack two 64-row factors each, so
// that one M=128 product serves both the state update and the output:
//   WQ = [W; Q] per d-panel  (W from the record, Q from the q tile)
//   XZ = [X diag(beta); 0]   ZP = [0; P']   (the zero panel is shared by both)
// A stage fills as two parts with their own barriers: part A (W, Q, X diag(beta), V) is free
// again as soon as the chain's [W; Q] S product is done, so the next-but-one chunk's part A
// streams in early; part B (P', scalars, K) once the chain's dS and the helper's output
// product are done (the epilogue reads its row scales from the record in global memory).
struct SStage {
    static constexpr uint32_t WQ = 0;                 // [W0][Q0][W1][Q1], 8 KB each
    static constexpr uint32_t XZ = 4 * kPanel;        // X diag(beta), then the zero panel
    static constexpr uint32_t ZP = 5 * kPanel;        // the zero panel, then P'
    static constexpr uint32_t SC = 7 * kPanel;        // RecScalars
    static constexpr uint32_t K = SC + 1024;          // K tile (two d-panels)
    static constexpr uint32_t V = K + 2 * kPanel;     // V slice (one panel)
    static constexpr uint32_t BYTES = V + kPanel;
    static constexpr uint32_t TX_A = 4 * kPanel + kPanel + kPanel;   // W, Q, X diag(beta), V
    static constexpr uint32_t TX_B = kPanel + 1024 + 2 * kPanel;     // P', scalars, K
};

struct SSmem {
    static constexpr uint32_t ST = 0;                         // [2] stages
    static constexpr uint32_t SB = 2 * SStage::BYTES;         // S [d][v] bf16, MN-major, 128 rows
    static constexpr uint32_t VHI = SB + 2 * kPanel;          // hi(ce VN) [tok][v]
    static constexpr uint32_t VLO = VHI + kPanel;             // lo(ce VN)
    static constexpr uint32_t VBF = VLO + kPanel;             // VN [tok][v]
    static constexpr uint32_t END = VBF + kPanel;
    static constexpr uint32_t BYTES = END + 1024;             // + alignment slack
};
static_assert(SStage::BYTES % 1024 == 0 && SStage::K % 1024 == 0 && SSmem::SB % 1024 == 0, "swizzle atoms");
static_assert(SSmem::VLO == SSmem::VHI + kPanel, "hi and lo are one two-panel B operand of the dS product");

struct SShared {
    uint64_t full_a[2], full_b[2], empty_a[2], empty_b[2];
    uint64_t u_done[2], acc_vn[2], ds_issued[2], acc_o[2], o_free[2], acc_s;
    uint64_t drain_chain, drain_helper;
    uint32_t tmem_base;
    int abort;
};

constexpr int kScanThreads = 512;  // warp 0 loader, 1 MMA helper, 6-7 epilogue, 8-15 chain
constexpr int kChainThreads = 256;
constexpr int kEpiThreads = 64;
constexpr uint32_t kScanTmemCols = 256;
constexpr uint32_t kColD = 0;     // per parity (64 * parity): VN in lanes 0-63, -O in lanes 64-127
constexpr uint32_t kColDS = 128;  // [K^T hi | K^T lo]: one N = 128 product, 128 columns

// One scan CTA: (bx, by) = (value head * slices + slice, sequence).
__device__ __forceinline__ void scan_cta(const ScanParams& p, int bx, int by) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ SShared sh;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3;                                   // TMEM lane quarter of this warp
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
    const int hv = bx / kSlices;
    const int v0 = (bx % kSlices) * kVS;
    const int h = hv / p.rep;
    const int n = p.order ? p.order[by] : by;
    int64_t bos = 0, len = p.T, brow = n, slot0 = (int64_t)n * p.ncd;
    if (p.cu_seqlens) {
        bos = p.cu_seqlens[n];
        len = p.cu_seqlens[n + 1] - bos;
        brow = 0;
        slot0 = bos / 64 + n;
    }
    const int nchunks = (int)((len + 63) / 64);

    if (tid == 0) {
        sh.abort = 0;
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sh.full_a[s], 1);
            mbar_init(&sh.full_b[s], 1);
            mbar_init(&sh.empty_a[s], 1);  // the chain's [W; Q] S product
            mbar_init(&sh.empty_b[s], 2);  // the chain's dS and the helper's output product
            mbar_init(&sh.u_done[s], 1);
            mbar_init(&sh.acc_vn[s], 1);
            mbar_init(&sh.ds_issued[s], 1);
            mbar_init(&sh.acc_o[s], 1);
            mbar_init(&sh.o_free[s], 1);
        }
        mbar_init(&sh.acc_s, 1);
        mbar_init(&sh.drain_chain, 1);
        mbar_init(&sh.drain_helper, 1);
        fence_mbar_init();
        tma_prefetch_map(&p.tm_q);
        tma_prefetch_map(&p.tm_k);
        tma_prefetch_map(&p.tm_v);
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, kScanTmemCols);
        tmem_relinquish();
    }
    // the zero panel of both stages (never written by a copy)
    for (int i = tid; i < 2 * (int)(kPanel / 16); i += kScanThreads) {
        const int s = i / (int)(kPanel / 16), j = i % (int)(kPanel / 16);
        reinterpret_cast<uint4*>(sm + SSmem::ST + s * SStage::BYTES + SStage::ZP)[j] = make_uint4(0, 0, 0, 0);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;
    auto wait = [&](uint64_t* b, uint32_t parity, int site) -> bool {
        return mbar_wait_or_abort(b, parity, site, &sh.abort);
    };
    auto spin = [&](uint64_t* b, uint32_t parity, int site) -> bool {  // the chain's critical waits
        return mbar_wait_or_abort(b, parity, site, &sh.abort, false);
    };
    auto fail = [&]() { atomicExch(&sh.abort, 1); };
    auto nvalid_of = [&](int c) -> int {
        const int64_t rest = len - 64 * (int64_t)c;
        return (int)(rest < 64 ? rest : 64);
    };
    auto stage = [&](int s) -> uint8_t* { return sm + SSmem::ST + s * SStage::BYTES; };
    const uint32_t id_pos = make_idesc(128, kVS, kFmtBF16, false, true);        // D (+)= A B
    const uint32_t id_neg = make_idesc(128, kVS, kFmtBF16, false, true, true);  // D += -A B
    const uint32_t id_s = make_idesc(128, 2 * kVS, kFmtBF16, true, true);  // B = [hi | lo], two panels

    if (warp == 0) {
        // ================================ loader ================================
        int issued[2] = {0, 0};  // 1 + chunk of the last copy started per stage; negative: both parts
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1;
            const int t = (int)(bos + 64 * c);
            uint8_t* st = stage(s);
            const uint8_t* rec = p.records + ((slot0 + c) * p.HV + hv) * (int64_t)kRecBytes;
            if (c >= 2) {
                const bool w = wait(&sh.empty_a[s], ((c >> 1) + 1) & 1, kSiteTmaLoad);
                if (!__all_sync(0xffffffffu, w)) {
                    fail();
                    break;
                }
            }
            const bool ready = !(p.ready && lane == 0) || wait_ready(p.ready + (slot0 + c) * p.HV + hv, &sh.abort);
            if (!__all_sync(0xffffffffu, ready)) {
                fail();
                break;
            }
            if (lane == 0) {
                uint64_t* bar = &sh.full_a[s];
                mbar_arrive_expect_tx(bar, SStage::TX_A);
                bulk_load(st + SStage::WQ, rec + kRecW, kPanel, bar);
                bulk_load(st + SStage::WQ + 2 * kPanel, rec + kRecW + kPanel, kPanel, bar);
                tma_load_4d(st + SStage::WQ + kPanel, &p.tm_q, bar, 0, h, t, (int)brow);
                tma_load_4d(st + SStage::WQ + 3 * kPanel, &p.tm_q, bar, 64, h, t, (int)brow);
                bulk_load(st + SStage::XZ, rec + kRecXB, kPanel, bar);
                tma_load_4d(st + SStage::V, &p.tm_v, bar, v0, hv, t, (int)brow);
                issued[s] = c + 1;
            }
            if (c >= 2) {
                const bool w = wait(&sh.empty_b[s], ((c >> 1) + 1) & 1, kSiteTmaLoad);
                if (!__all_sync(0xffffffffu, w)) {
                    fail();
                    break;
                }
            }
            if (lane == 0) {
                uint64_t* bar = &sh.full_b[s];
                mbar_arrive_expect_tx(bar, SStage::TX_B);
                bulk_load(st + SStage::ZP + kPanel, rec + kRecPM, kPanel, bar);
                bulk_load(st + SStage::SC, rec + kRecSc, 1024, bar);
                tma_load_4d(st + SStage::K, &p.tm_k, bar, 0, h, t, (int)brow);
                tma_load_4d(st + SStage::K + kPanel, &p.tm_k, bar, 64, h, t, (int)brow);
                issued[s] = -(c + 1);
            }
            __syncwarp();
        }
        // let every copy this warp started land before the CTA can exit
        if (lane == 0)
            for (int s = 0; s < 2; ++s) {
                const int c = (issued[s] < 0 ? -issued[s] : issued[s]) - 1;
                if (c < 0) continue;
                mbar_wait(&sh.full_a[s], (c >> 1) & 1, kSiteDrain);
                if (issued[s] < 0) mbar_wait(&sh.full_b[s], (c >> 1) & 1, kSiteDrain);
            }
    } else if (warp == 1) {
        // ============================== MMA helper ==============================
        // Issues the products off the chain's critical path. U(c+1) = [X diag(beta); 0] V goes
        // into the accumulator of parity (c+1) & 1 as soon as the chain's [W; Q] S product of
        // chunk c is done (so it never delays it) and its inputs have landed; the output part
        // -[0; P'] VN of chunk c queues behind the chain's dS. Ordering with the chain's MMAs
        // goes through mbarriers.
        if (lane == 0 && nchunks > 0) {
            const uint64_t dVBF = sdesc_mnmajor(sm + SSmem::VBF, kPanel);
            auto issue_u = [&](int c) {
                const int s = c & 1;
                const uint64_t a = sdesc_kmajor(stage(s) + SStage::XZ, 0), b = sdesc_mnmajor(stage(s) + SStage::V, kPanel);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16(tb + kColD + 64 * s, sdesc_add(a, kk * 32), sdesc_add(b, kk * 2048), id_pos, kk > 0);
                mma_commit(&sh.u_done[s]);
            };
            bool issued_any = false;
            if (wait(&sh.full_a[0], 0, kSiteTmaLoad)) {
                tc_fence_after();
                issue_u(0);
                issued_any = true;
                for (int c = 0; c < nchunks; ++c) {
                    const int s = c & 1;
                    const uint32_t phs = (c >> 1) & 1;
                    if (c + 1 < nchunks) {
                        bool ok = wait(&sh.acc_vn[s], phs, kSiteMma);
                        if (ok) ok = wait(&sh.full_a[s ^ 1], ((c + 1) >> 1) & 1, kSiteTmaLoad);
                        if (ok && c >= 1) ok = wait(&sh.o_free[s ^ 1], ((c - 1) >> 1) & 1, kSiteMma);
                        if (!ok) { fail(); break; }
                        tc_fence_after();
                        issue_u(c + 1);
                    }
                    if (!wait(&sh.ds_issued[s], phs, kSiteMma)) { fail(); break; }
                    tc_fence_after();
                    const uint64_t a = sdesc_kmajor(stage(s) + SStage::ZP, 0);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16(tb + kColD + 64 * s, sdesc_add(a, kk * 32), sdesc_add(dVBF, kk * 2048), id_neg, 1);
                    mma_commit(&sh.acc_o[s]);
                    mma_commit(&sh.empty_b[s]);
                }
            } else {
                fail();
            }
            if (issued_any) {
                mma_commit(&sh.drain_helper);
                mbar_wait(&sh.drain_helper, 0, kSiteDrain);
            }
        }
    } else if (warp == 6 || warp == 7) {
        // =============================== epilogue ===============================
        // -O sits in TMEM lanes 64-127 (rows 0-63 of the lower half of the M=128 accumulator).
        const int et = tid - 192;        // 0..63
        const int row = et;              // output row of this thread (lane quarter 2 or 3)
        const float* eq_rec = reinterpret_cast<const float*>(p.records + kRecSc + offsetof(RecScalars, eq)) + row;
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1;
            const uint32_t phs = (c >> 1) & 1;
            const uint32_t tD = tb + kColD + 64 * s;
            if (!named_sync_all(kBarEpi, kEpiThreads, wait(&sh.acc_o[s], phs, kSiteMma))) {
                fail();
                break;
            }
            // the record of chunk c has been read by this CTA's products, so it is written
            const float neg_eq = -eq_rec[(((slot0 + c) * p.HV + hv) * (int64_t)kRecBytes) / 4];
            tc_fence_after();
            const bool store = row < nvalid_of(c);
            bf16* orow = p.o + ((brow * p.T + bos + 64 * (int64_t)c + row) * p.HV + hv) * kHeadDim + v0;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float r[32];
                tmem_ld32_wait(tD + lane_base + 32 * half, r);
                if (store) {
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) {
                        uint4 raw;
                        __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            hh[j] = __floats2bfloat162_rn(neg_eq * r[8 * ch + 2 * j], neg_eq * r[8 * ch + 2 * j + 1]);
                        *reinterpret_cast<uint4*>(orow + 32 * half + 8 * ch) = raw;
                    }
                }
            }
            tc_fence_before();
            named_sync(kBarEpi, kEpiThreads);
            if (et == 0) mbar_arrive(&sh.o_free[s]);
        }
    } else if (warp >= 8) {
        // ================================ chain ================================
        const int ct = tid - 256;       // 0..255
        const int d = ct & 127;         // the state row (and TMEM lane) of this thread
        const int cg = ct >> 7;         // column half of the slice: columns 32 cg .. 32 cg + 31
        const bool vn_rows = quarter < 2;  // lanes 0-63 hold VN: token row 32 quarter + lane
        const int vrow = 32 * quarter + lane;
        const int64_t state_row = (((int64_t)n * p.HV + hv) * kHeadDim + d) * kHeadDim + v0 + 32 * cg;
        float S[32];
        if (p.h0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 x4 = ld4(p.h0 + state_row + j);
                S[j] = x4.x; S[j + 1] = x4.y; S[j + 2] = x4.z; S[j + 3] = x4.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) S[j] = 0.f;
        }
        if (nchunks == 0) {
            if (p.ht)
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(p.ht + state_row + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
        } else {
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) put_chunk(sm + SSmem::SB, d, 4 * cg + ch, S + 8 * ch);
        }
        fence_async_smem();
        named_sync(kBarChain, kChainThreads);
        const uint64_t dSB = sdesc_mnmajor(sm + SSmem::SB, kPanel);
        const uint64_t dVHI = sdesc_mnmajor(sm + SSmem::VHI, kPanel);
        bool issued_any = false;
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1;
            const uint32_t ph = c & 1, phs = (c >> 1) & 1;
            const uint32_t tD = tb + kColD + 64 * s;
            uint8_t* st = stage(s);
            const bool landed = spin(&sh.full_a[s], phs, kSiteTmaLoad) && spin(&sh.full_b[s], phs, kSiteTmaLoad) &&
                                spin(&sh.u_done[s], phs, kSiteMma);
            if (!named_sync_all(kBarChain, kChainThreads, landed)) {
                fail();
                break;
            }
            // the stage can be refilled once the MMAs below are done: read its scalars now
            const RecScalars* rs = reinterpret_cast<const RecScalars*>(st + SStage::SC);
            const float cei = rs->ce[vrow & 63];
            const float decay = rs->dec;
            // ---- D -= [W; Q] S: VN = U - W S (lanes 0-63), -Q S (lanes 64-127)
            if (ct == 0) {
                tc_fence_after();
                const uint64_t a = sdesc_kmajor(st + SStage::WQ, 0);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_f16(tD, sdesc_add(a, (kk >> 2) * 2 * kPanel + (kk & 3) * 32), sdesc_add(dSB, kk * 2048), id_neg, 1);
                mma_commit(&sh.acc_vn[s]);
                mma_commit(&sh.empty_a[s]);
                issued_any = true;
            }
            // VN is read out once the previous chunk's output product is done with VBF
            bool ready = spin(&sh.acc_vn[s], phs, kSiteMma);
            if (ready && c >= 1) ready = spin(&sh.acc_o[s ^ 1], ((c - 1) >> 1) & 1, kSiteMma);
            if (!named_sync_all(kBarChain, kChainThreads, ready)) {
                fail();
                break;
            }
            tc_fence_after();
            // ---- VN -> bf16 VN and the split ce VN, this warpgroup's 32 columns
            if (vn_rows) {
                float r[32];
                tmem_ld32_wait(tD + lane_base + 32 * cg, r);
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    float hi[8], lo[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float x = cei * r[8 * cc + j];
                        hi[j] = round_bf16(x);
                        lo[j] = x - hi[j];
                    }
                    const int ch = 4 * cg + cc;
                    put_chunk(sm + SSmem::VBF, vrow, ch, r + 8 * cc);
                    put_chunk(sm + SSmem::VHI, vrow, ch, hi);
                    put_chunk(sm + SSmem::VLO, vrow, ch, lo);
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarChain, kChainThreads);
            if (ct == 0) {
                // [K^T hi | K^T lo] (all lanes, fresh; hi and lo are adjacent panels, so one N = 128
                // product per k step); the helper's output product queues behind it
                tc_fence_after();
                const uint64_t ak = sdesc_mnmajor(st + SStage::K, kPanel);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = sdesc_add(ak, kk * 2048);
                    mma_f16(tb + kColDS, ad, sdesc_add(dVHI, kk * 2048), id_s, kk > 0);
                }
                mma_commit(&sh.acc_s);
                mma_commit(&sh.empty_b[s]);
                mbar_arrive(&sh.ds_issued[s]);
            }
            if (!named_sync_all(kBarChain, kChainThreads, spin(&sh.acc_s, ph, kSiteMma))) {
                fail();
                break;
            }
            tc_fence_after();
            // ---- S <- 2^glast S + (K^T hi + K^T lo), this warpgroup's 32 columns
#pragma unroll
            for (int h16 = 0; h16 < 2; ++h16) {
                float rh[16], rl[16];
                const uint32_t col = tb + kColDS + lane_base + 32 * cg + 16 * h16;
                tmem_ld16x2_wait(col, col + kVS, rh, rl);
#pragma unroll
                for (int j = 0; j < 16; ++j) S[16 * h16 + j] = fmaf(decay, S[16 * h16 + j], rh[j] + rl[j]);
            }
            if (c + 1 == nchunks) {
                if (p.ht)
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(p.ht + state_row + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
            } else {
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) put_chunk(sm + SSmem::SB, d, 4 * cg + ch, S + 8 * ch);
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(kBarChain, kChainThreads);
        }
        if (ct == 0 && issued_any) {
            mma_commit(&sh.drain_chain);
            mbar_wait(&sh.drain_chain, 0, kSiteDrain);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tb, kScanTmemCols);
}

__global__ void __launch_bounds__(kScanThreads, 1) chunk_scan_kernel(const __grid_constant__ ScanParams p) {
    pdl_launch_dependents();  // a gated norm launched after this kernel may stage its z early
    scan_cta(p, blockIdx.x, blockIdx.y);
}

// =========================================================================================
// fused launch: when the scan leaves SMs idle (few sequences times heads), one cooperative
// launch runs the scan CTAs and, on the remaining SMs, three factor warpgroups per CTA that
// produce the records in chunk order; each record carries a ready flag the scan's loader waits
// for. The factor role never waits for the scan role, and a cooperative launch keeps every
// CTA resident, so the waits always end.
// =========================================================================================
constexpr int kFusedFactorGroups = 3;
constexpr int kMinFactorCtas = 16;
constexpr uint32_t kFusedSmemBytes =
    (SSmem::BYTES > kFusedFactorGroups * FSmem::END + 1024) ? SSmem::BYTES : kFusedFactorGroups * FSmem::END + 1024;
static_assert(FSmem::END % 1024 == 0, "factor warpgroup regions stay 1024-aligned");

__global__ void __launch_bounds__(kScanThreads, 1) chunk_fused_kernel(const __grid_constant__ FactorParams f,
                                                                       const __grid_constant__ ScanParams sp, int nscan,
                                                                       int scan_gx) {
    pdl_launch_dependents();  // a gated norm launched after this kernel may stage its z early
    if ((int)blockIdx.x < nscan) {
        scan_cta(sp, (int)blockIdx.x % scan_gx, (int)blockIdx.x / scan_gx);
        return;
    }
    const int g = threadIdx.x >> 7;
    if (g >= kFusedFactorGroups) return;
    extern __shared__ uint8_t smem_raw[];
    __shared__ FShared fsh[kFusedFactorGroups];
    const int64_t ctas = (int64_t)(gridDim.x - nscan);
    factor_worker(f, fsh[g], align1024(smem_raw) + g * FSmem::END, 1 + g, threadIdx.x & 127,
                  (int64_t)(blockIdx.x - nscan) * kFusedFactorGroups + g, ctas * kFusedFactorGroups,
                  (int64_t)f.ncd * f.nseq * f.HV, false, true);
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
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

int64_t chunk_workspace_slots(int64_t B, int64_t T, int64_t nseq, bool packed) {
    const int64_t ncd = (T + 63) / 64;
    return packed ? ncd + nseq : B * ncd;
}

// Workspace: the records, then one ready flag per record (used by the fused launch).
static size_t ready_offset(int64_t slots, int64_t HV) { return (size_t)slots * (size_t)HV * kRecBytes; }

size_t chunk_workspace_bytes(int64_t B, int64_t T, int64_t nseq, bool packed, int64_t HV) {
    const int64_t slots = chunk_workspace_slots(B, T, nseq, packed);
    const size_t flags = ((size_t)slots * (size_t)HV * sizeof(uint32_t) + 255) & ~size_t(255);
    const size_t order = packed ? (((size_t)nseq * sizeof(int32_t) + 255) & ~size_t(255)) : 0;
    return ready_offset(slots, HV) + flags + order;
}

// Packed batches: the scan's grid rows take the sequences longest first, so that the longest
// sequences do not start in the last wave of CTAs. Rank of sequence n = the number of sequences
// that are longer, or as long with a smaller index; one thread per sequence.
constexpr int kMaxOrderedSeqs = 1024;

__global__ void seq_order_kernel(const int32_t* __restrict__ cu, int nseq, int32_t* __restrict__ order) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= nseq) return;
    const int32_t len = cu[n + 1] - cu[n];
    int rank = 0;
    for (int m = 0; m < nseq; ++m) {
        const int32_t lm = cu[m + 1] - cu[m];
        rank += (lm > len || (lm == len && m < n)) ? 1 : 0;
    }
    order[rank] = n;
}

// Per-device launch facts, looked up once: SM count, cooperative launch support and the
// shared-memory opt-ins of the three kernels.
struct ChunkDevice {
    bool ready = false, ok = false, fused = false;
    int sms = 0;
};

static const ChunkDevice& chunk_device() {
    static ChunkDevice devices[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        static ChunkDevice none;
        return none;
    }
    ChunkDevice& d = devices[dev];
    if (!d.ready) {
        int coop = 0, active = 0;
        d.ok = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
               cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess &&
               cudaFuncSetAttribute(chunk_factor_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)FSmem::BYTES) == cudaSuccess &&
               cudaFuncSetAttribute(chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)SSmem::BYTES) == cudaSuccess &&
               cudaFuncSetAttribute(chunk_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kFusedSmemBytes) == cudaSuccess &&
               cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, chunk_fused_kernel, kScanThreads,
                                                             kFusedSmemBytes) == cudaSuccess;
        d.fused = d.ok && coop && active >= 1;
        d.ready = true;
    }
    return d;
}

// After the chunk kernels: the launch status, then the output-gated RMSNorm of o when asked for.
static int finish_chunk(const ChunkArgs& a, cudaStream_t s) {
    const int st = launch_status();
    if (st != GDN_OK || a.y == nullptr) return st;
    // a programmatic dependent of the chunk kernel: its CTAs load z and the weight (inputs of the call,
    // which the chunk kernel does not write) while the scan ends, and read o after griddepcontrol.wait
    return launch_gated_rmsnorm(a.o, a.z, a.norm_w, a.y, a.B * a.T * a.HV, kHeadDim, a.eps, s, true);
}

int launch_chunk(const ChunkArgs& a, cudaStream_t s) {
    if (a.nseq == 0) return GDN_OK;
    const bool packed = a.cu_seqlens != nullptr;
    const int64_t slots = chunk_workspace_slots(a.B, a.T, a.nseq, packed);
    if (slots * a.HV > INT32_MAX) return GDN_ERR_SHAPE;
    if (a.workspace == nullptr || a.workspace_bytes < chunk_workspace_bytes(a.B, a.T, a.nseq, packed, a.HV))
        return GDN_ERR_WORKSPACE;
    const ChunkDevice& dev = chunk_device();
    if (!dev.ok) return GDN_ERR_LAUNCH;
    FactorParams f;
    ScanParams sp;
    memset(&f, 0, sizeof(f));
    memset(&sp, 0, sizeof(sp));
    if (!make_map(&f.tm_q, a.q, a.B, a.T, a.H, a.qsb, a.qst, a.qsh) ||
        !make_map(&f.tm_k, a.k, a.B, a.T, a.H, a.ksb, a.kst, a.ksh) ||
        !make_map(&sp.tm_v, a.v, a.B, a.T, a.HV, a.vsb, a.vst, a.vsh))
        return GDN_ERR_LAUNCH;
    sp.tm_q = f.tm_q;
    sp.tm_k = f.tm_k;
    const int ncd = (int)((a.T + 63) / 64);
    f.g = a.g;
    f.beta = a.beta;
    f.gates = a.gates;
    f.beta_f32 = a.beta_dtype == GDN_F32;
    f.cu_seqlens = a.cu_seqlens;
    f.records = static_cast<uint8_t*>(a.workspace);
    f.slots = slots;
    f.T = a.T;
    f.nseq = (int)a.nseq;
    f.ncd = ncd;
    f.HV = a.HV;
    f.rep = a.HV / a.H;
    f.scale = a.scale;
    sp.h0 = a.h0;
    sp.ht = a.ht;
    sp.o = static_cast<bf16*>(a.o);
    sp.cu_seqlens = a.cu_seqlens;
    sp.records = static_cast<const uint8_t*>(a.workspace);
    sp.T = a.T;
    sp.ncd = ncd;
    sp.HV = a.HV;
    sp.rep = f.rep;
    const int scan_gx = a.HV * (kHeadDim / kVS);
    const int64_t nscan = (int64_t)scan_gx * a.nseq;
    if (dev.fused && slots > 0 && nscan + kMinFactorCtas <= dev.sms) {
        uint32_t* ready = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a.workspace) + ready_offset(slots, a.HV));
        if (cudaMemsetAsync(ready, 0, (size_t)slots * a.HV * sizeof(uint32_t), s) != cudaSuccess)
            return GDN_ERR_LAUNCH;
        f.ready = ready;
        sp.ready = ready;
        int ns = (int)nscan, gx = scan_gx;
        void* args[] = {&f, &sp, &ns, &gx};
        if (cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(chunk_fused_kernel), dim3((unsigned)dev.sms),
                                        dim3(kScanThreads), args, kFusedSmemBytes, s) != cudaSuccess)
            return GDN_ERR_LAUNCH;
        return finish_chunk(a, s);
    }
    if (slots > 0) {
        chunk_factor_kernel<<<(unsigned)(slots * a.HV), 128, FSmem::BYTES, s>>>(f);
        const int st = launch_status();
        if (st != GDN_OK) return st;
    }
    if (packed && a.nseq > 1 && a.nseq <= kMaxOrderedSeqs) {
        const size_t flags = ((size_t)slots * a.HV * sizeof(uint32_t) + 255) & ~size_t(255);
        int32_t* order = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(a.workspace) + ready_offset(slots, a.HV) + flags);
        seq_order_kernel<<<(unsigned)((a.nseq + 127) / 128), 128, 0, s>>>(a.cu_seqlens, (int)a.nseq, order);
        const int st = launch_status();
        if (st != GDN_OK) return st;
        sp.order = order;
    }
    dim3 grid((unsigned)scan_gx, (unsigned)a.nseq);
    chunk_scan_kernel<<<grid, kScanThreads, SSmem::BYTES, s>>>(sp);
    return finish_chunk(a, s);
}

}  // namespace gdn
