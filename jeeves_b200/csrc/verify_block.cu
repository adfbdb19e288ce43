// Block verify on tcgen05 tensor cores: the outputs and update vectors of T <= 8 drafted tokens
// from one read of each (row, value head) state, for the verify that keeps its update vectors
// (gdn_recurrent_deltas; the engine's delta_outputs, inference/engine.py:249-252, and its
// delta_commit, :254-258, as gdn_delta_commit).
//
// The token recurrence (torch_recurrent_gated_delta_rule, model/model.py:221-239),
//   delta_t = beta_t (v_t - d_t S_{t-1}^T kn_t),  o_t = d_t S_{t-1}^T qn_t + (qn_t . kn_t) delta_t,
//   S_t = d_t S_{t-1} + kn_t delta_t^T,           d_t = e^{g_t}, kn / qn the normalised k / q rows,
// unrolls over the block with D_t = d_0 ... d_t and P(u, t) = d_{u+1} ... d_t into
//   S_{t-1}^T kn_t = D_{t-1} S_0^T kn_t + sum_{u<t}  P(u, t-1) (kn_t . kn_u) delta_u,
//   o_t            = D_t     S_0^T qn_t + sum_{u<=t} P(u, t)   (qn_t . kn_u) delta_u,
// so one product of the state with the 2T raw k and q rows, R = S_0^T [k_0 .. k_{T-1} q_0 .. q_{T-1}]
// (128 x 2T), and the Gram products of those rows give every output; the rest is O(T^2) per
// column. R runs on the tensor cores (kind::f16) with the state split into two bf16 parts,
// S = hi + lo + r with hi = bf16(S), lo = bf16(S - hi), |r| <= 2^-18 |S| element by element,
// against the bf16 k and q rows (exact), accumulated in fp32.
//
// Two persistent CTAs per SM walk the (row, value head) pairs. Their threads load each pair's 64 KB
// state into registers one pair ahead (every load of a warp one whole state row) and split it into
// the two bf16 operands of A = S^T in shared memory (MN-major, 128-byte swizzle: the state rows
// are A's K). One thread then issues the products: first the Gram products of the k / q rows,
// committed on their own so that warp 0 forms the pair's coefficients while the tensor cores go
// on with hi and lo into two accumulators. Warps 0-3 drain R, one state column each (TMEM lane =
// column), while warps 4-7 put the next pair's rows, v and gates in place (also loaded one pair
// ahead). Every wait is bounded; a wait that gives up raises the device error word, the CTA stops
// taking pairs, waits for the products it started and frees its TMEM.

#include <type_traits>

#include "common.cuh"
#include "launch.h"
#include "norm.cuh"
#include "sm100.cuh"

namespace gdn {
namespace vblock {

using namespace sm100;

constexpr int kThreads = 256;
constexpr int kIssuer = 224;       // lane 0 of warp 7 issues the products: the Gram first, then hi and lo
constexpr int kMaxT = 8;
constexpr uint32_t kPanel = 128 * 128;              // 128 rows x 128 bytes (64 bf16 columns or K elements)
constexpr uint32_t kVA = 4 * kPanel;                // after hi (2 panels) and lo (2 panels): the MN-major operands
constexpr uint32_t kSmem = kVA + 2 * kPanel + 1024; // the k / q rows, K-major in 128-row panels + alignment slack
constexpr uint32_t kTmemCols = 64;                  // R from hi in columns 0-15, from lo in 16-31, the Gram in 32-47
constexpr int kRowsPerThread = 16;                  // state rows w + 8 k of one 4-column group a thread holds
enum : uint32_t { kBarDrain = 1 };                  // named barrier of the drain's warps 0-3

enum : int { kSiteProduct = 0x302, kSiteGram = 0x303 };

struct Params {
    const float* state;  // [pairs, 128, 128] fp32
    const bf16* q;
    const bf16* k;
    const bf16* v;
    const float* g;
    const void* beta;
    int beta_f32;
    bf16* o;          // [rows, T, HV, 128], or null when the gated norm is fused (y)
    float* deltas;    // [rows, T, HV, 128]
    // the output-gated RMSNorm fused into the drain, when y is set: y = norm(o) * w * silu(z)
    const bf16* z;       // [rows, T, HV, 128]
    const bf16* norm_w;  // [128]
    bf16* y;             // [rows, T, HV, 128]
    float eps;
    int64_t qsb, qst, qsh, ksb, kst, ksh, vsb, vst, vsh;
    int HV, rep, pairs;
    float scale;
};

// Per-slot coefficients of the pair in flight (see the header: Ck[t][u] = P(u, t-1) (kn_t . kn_u),
// Cq[t][u] = P(u, t) (qn_t . kn_u), Dk[t] = D_{t-1}, Dq[t] = D_t).
struct Coef {
    float ck[kMaxT][kMaxT], cq[kMaxT][kMaxT];
    float dk[kMaxT], dq[kMaxT], dec[kMaxT], beta[kMaxT], rk[kMaxT], rq[kMaxT];
    float gram[2 * kMaxT][2 * kMaxT];  // raw row products: [a][b] = row a . row b (k rows, then q rows)
};

// The fused norm's buffers (only in the kernels that fuse it): z one pair ahead (two buffers), the
// outputs as bf16 values and each token's 1 / sqrt(mean square + eps).
struct NormBufs {
    alignas(16) bf16 z[2][kMaxT][kHeadDim];
    float xs[kMaxT][kHeadDim];
    float inv[kMaxT];
};
struct NoNorm {};

// The pair's inputs besides the state and the rows, deposited one pair ahead (two buffers).
struct Aux {
    alignas(16) bf16 v[kMaxT][kHeadDim];
    float g[kMaxT], beta[kMaxT];
};

struct Shared {
    uint64_t acc, acc_gram;
    uint32_t tmem_base;
    int abort;
    Coef coef;
    Aux aux[2];
};

// What warps 4-7 (thread lt = 0 .. 127 of them) load one pair ahead: row chunks lt and lt + 128
// of the 2T x 16 chunks of k and q, chunk lt of the T x 16 chunks of v, and one gate value
// (lt < T: g_lt; T <= lt < 2T: beta_{lt - T}).
struct Prefetch {
    uint4 rows[2];
    uint4 vch, zch;
    float gb;
};

template <int T, bool NORM>
__device__ __forceinline__ void prefetch(const Params& p, int pair, int lt, Prefetch& f) {
    const int64_t b = pair / p.HV;
    const int hv = pair % p.HV;
    const int h = hv / p.rep;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int it = lt + 128 * r, n = it >> 4, ch = it & 15;
        if (it < 2 * T * 16) {
            const bf16* src = n < T ? p.k + b * p.ksb + (int64_t)n * p.kst + h * p.ksh
                                    : p.q + b * p.qsb + (int64_t)(n - T) * p.qst + h * p.qsh;
            f.rows[r] = *reinterpret_cast<const uint4*>(src + 8 * ch);
        }
    }
    if (lt < T * 16) {
        f.vch = *reinterpret_cast<const uint4*>(p.v + b * p.vsb + (int64_t)(lt >> 4) * p.vst + hv * p.vsh + 8 * (lt & 15));
        if (NORM)
            f.zch = *reinterpret_cast<const uint4*>(p.z + ((b * T + (lt >> 4)) * p.HV + hv) * kHeadDim + 8 * (lt & 15));
    }
    if (lt < 2 * T) {
        const int t = lt < T ? lt : lt - T;
        const int64_t gi = (b * T + t) * p.HV + hv;
        f.gb = lt < T ? p.g[gi]
                      : (p.beta_f32 ? static_cast<const float*>(p.beta)[gi]
                                    : __bfloat162float(static_cast<const bf16*>(p.beta)[gi]));
    }
}

// Puts a prefetched pair into the bf16 K-major row operand (chunk ch of row n at its swizzled
// place in K-panel ch / 8 of 128 rows) and into an Aux buffer.
template <int T>
__device__ __forceinline__ void deposit(const Prefetch& f, uint8_t* vb, Aux& aux, int lt, bf16 (*zdst)[kHeadDim]) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int it = lt + 128 * r, n = it >> 4, ch = it & 15;
        if (it < 2 * T * 16) *reinterpret_cast<uint4*>(vb + (ch >> 3) * kPanel + sw128(n, ch & 7)) = f.rows[r];
    }
    if (lt < T * 16) {
        *reinterpret_cast<uint4*>(&aux.v[lt >> 4][8 * (lt & 15)]) = f.vch;
        if (zdst) *reinterpret_cast<uint4*>(&zdst[lt >> 4][8 * (lt & 15)]) = f.zch;
    }
    if (lt < T) aux.g[lt] = f.gb;
    else if (lt < 2 * T) aux.beta[lt - T] = f.gb;
}

__device__ __forceinline__ bf16 (*z_buffer(NormBufs& nb, int i))[kHeadDim] { return nb.z[i]; }
__device__ __forceinline__ bf16 (*z_buffer(NoNorm&, int))[kHeadDim] { return nullptr; }

template <int T, bool NORM>
__global__ void __launch_bounds__(kThreads, 2) verify_block_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ Shared sh;
    __shared__ typename std::conditional<NORM, NormBufs, NoNorm>::type nb;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int first = blockIdx.x, stride = gridDim.x;
    const int npairs = first < p.pairs ? (p.pairs - first + stride - 1) / stride : 0;
    auto pair_of = [&](int j) { return first + j * stride; };
    uint8_t* const vb = sm + kVA;
    Coef& cf = sh.coef;

    if (tid == 0) {
        sh.abort = 0;
        mbar_init(&sh.acc, 1);
        mbar_init(&sh.acc_gram, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    // rows 2T .. 127 of the row operand stay zero
    for (int i = tid; i < 128 * 16; i += kThreads) {
        const int n = i >> 4, ch = i & 15;
        if (n >= 2 * T) *reinterpret_cast<uint4*>(vb + (ch >> 3) * kPanel + sw128(n, ch & 7)) = make_uint4(0, 0, 0, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // The state lives in registers between its load and its split: thread (warp w, lane l) holds
    // columns 4 l .. 4 l + 3 of state rows w, w + 8, ..., w + 120 (every load of a warp is one
    // whole 512-byte row), loaded one pair ahead.
    float4 sv[kRowsPerThread];
    auto load_state = [&](int j) {
        const float* src = p.state + (int64_t)pair_of(j) * (kHeadDim * kHeadDim) + warp * kHeadDim + 4 * lane;
#pragma unroll
        for (int k = 0; k < kRowsPerThread; ++k) sv[k] = ldg_stream(reinterpret_cast<const float4*>(src + 8 * k * kHeadDim));
    };
    // One thread of warp 1 asks L2 for the state of the pair after next (one bulk prefetch of its
    // 64 KB): the register loads one pair ahead then find it there, and DRAM keeps streaming while
    // the pair in registers goes through its serial chain (128 rows x 5 tokens 77 -> 70.5 us).
    auto prefetch_state = [&](int j) {
        if (tid == 32 && j < npairs) {
            const float* src = p.state + (int64_t)pair_of(j) * (kHeadDim * kHeadDim);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src),
                         "r"((uint32_t)(kHeadDim * kHeadDim * sizeof(float)))
                         : "memory");
        }
    };
    if (npairs > 0) load_state(0);
    // As a programmatic dependent of the verify layer's conv step, the set-up and the first state
    // loads above overlap that kernel; the rows, v, gates and z are read only past this point.
    pdl_wait();
    Prefetch pf;
    if (warp >= 4 && npairs > 0) {
        prefetch<T, NORM>(p, pair_of(0), tid - 128, pf);
        deposit<T>(pf, vb, sh.aux[0], tid - 128, z_buffer(nb, 0));
    }
    __syncthreads();
    const uint32_t tb = sh.tmem_base;
    const uint32_t idesc = make_idesc(128, 16, kFmtBF16, true, false);
    int computing = -1;  // the issuer: the parity of the products in flight, or -1

    for (int j = 0; j < npairs; ++j) {
        const int pair = pair_of(j);
        const Aux& aux = sh.aux[j & 1];
        // a gated norm launched as this kernel's dependent may stage its z during the last pairs
        if (j + 1 == npairs) pdl_launch_dependents();
        prefetch_state(j + 2);
        // the next pair's rows, v and gates start loading now and land during this pair
        if (warp >= 4 && j + 1 < npairs) prefetch<T, NORM>(p, pair_of(j + 1), tid - 128, pf);
        // ---- the split: this thread's 16 x 4 state values into bf16 hi and lo (MN-major operands,
        // hi panels 0-1, lo panels 2-3; 8-byte halves of the swizzled 16-byte chunks)
        {
            const int col = 4 * lane;
            const uint32_t pan = (col >> 6) * kPanel, chunk = (col & 63) >> 3, half = (col & 7) * 2;
#pragma unroll
            for (int k = 0; k < kRowsPerThread; ++k) {
                const int row = warp + 8 * k;
                const float4 x = sv[k];
                const __nv_bfloat162 h01 = __floats2bfloat162_rn(x.x, x.y), h23 = __floats2bfloat162_rn(x.z, x.w);
                const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
                const __nv_bfloat162 l01 = __floats2bfloat162_rn(x.x - f01.x, x.y - f01.y);  // exact differences
                const __nv_bfloat162 l23 = __floats2bfloat162_rn(x.z - f23.x, x.w - f23.y);
                const uint32_t off = pan + sw128(row, chunk) + half;
                *reinterpret_cast<uint2*>(sm + off) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
                *reinterpret_cast<uint2*>(sm + 2 * kPanel + off) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
            }
        }
        if (j + 1 < npairs) load_state(j + 1);  // lands while this pair is multiplied and drained
        fence_async_smem();
        __syncthreads();
        if (tid == kIssuer) {
            // ---- the Gram product G = [k | q]^T [k | q] of the rows (M = 64: rows 0-63 of the
            // zero-padded operand, row r of G in TMEM lane r for r < 16), committed on its own so
            // that warp 0 forms the coefficients while the tensor cores go on with
            // R = hi^T [k | q] + lo^T [k | q] (8 steps of K = 16 state rows for each part)
            tc_fence_after();
            const uint32_t gdesc = make_idesc(64, 16, kFmtBF16, false, false);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint64_t rows = sdesc_kmajor(vb + (ks >> 2) * kPanel, (ks & 3) * 32);
                mma_f16(tb + 32, rows, rows, gdesc, ks > 0);
            }
            mma_commit(&sh.acc_gram);
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint64_t a = sdesc_mnmajor(sm + part * 2 * kPanel, kPanel);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_f16(tb + 16 * part, sdesc_add(a, ks * 2048),
                            sdesc_kmajor(vb + (ks >> 2) * kPanel, (ks & 3) * 32), idesc, ks > 0);
            }
            mma_commit(&sh.acc);
            computing = j & 1;
        } else if (warp == 0) {
            // ---- meanwhile: the Gram rows (TMEM lanes 0 .. 2T-1), then the pair's coefficients
            // lane 0 polls, backing off, so that the wait takes no shared-memory bandwidth from the products
            const bool gok = __shfl_sync(0xffffffffu, lane != 0 || mbar_wait_or_abort(&sh.acc_gram, j & 1, kSiteGram, &sh.abort), 0);
            if (!gok && lane == 0) atomicExch(&sh.abort, 1);
            if (gok) {
                tc_fence_after();
                float gr[16];
                tmem_ld16_wait(tb + 32, gr);  // lane r: row r . rows 0 .. 15
                if (lane < 2 * T) {
#pragma unroll
                    for (int b = 0; b < 2 * T; ++b) cf.gram[lane][b] = gr[b];
                }
                __syncwarp();
                // lane t < T: its token's decay and norms, then its rows of the coefficients
                const int t = lane < T ? lane : 0;
                const float dect = expf(aux.g[t]);
                const float rkt = rsqrtf(cf.gram[t][t] + 1e-6f);
                float dec[T], rk[T];
#pragma unroll
                for (int u = 0; u < T; ++u) {
                    dec[u] = __shfl_sync(0xffffffffu, dect, u);
                    rk[u] = __shfl_sync(0xffffffffu, rkt, u);
                }
                if (lane < T) {
                    float dprev = 1.f;
#pragma unroll
                    for (int u = 0; u < T; ++u) dprev = u < t ? dprev * dec[u] : dprev;
                    const float rqt = rsqrtf(cf.gram[T + t][T + t] + 1e-6f) * p.scale;
                    cf.dk[t] = dprev;
                    cf.dq[t] = dprev * dect;
                    cf.dec[t] = dect;
                    cf.rk[t] = rkt;
                    cf.rq[t] = rqt;
                    cf.beta[t] = aux.beta[t];
                    // P(u, t) and P(u, t - 1) for u = t, t - 1, ..., 0
                    float pt = 1.f, pt1 = 1.f;
#pragma unroll
                    for (int u = T - 1; u >= 0; --u) {
                        if (u > t) continue;
                        cf.cq[t][u] = pt * cf.gram[T + t][u] * rqt * rk[u];
                        if (u < t) {
                            cf.ck[t][u] = pt1 * cf.gram[t][u] * rkt * rk[u];
                            pt1 *= dec[u];
                        }
                        pt *= dec[u];
                    }
                }
            }
        }
        // ---- the products are done: the operands may take the next pair
        // (warp 0 has waited for the Gram product; a failed wait there raised the abort flag)
        const bool done = tid != 0 ||
                          (!*reinterpret_cast<volatile int*>(&sh.abort) &&
                           mbar_wait_or_abort(&sh.acc, j & 1, kSiteProduct, &sh.abort));
        if (!__syncthreads_and(done)) {
            atomicExch(&sh.abort, 1);
            break;
        }
        tc_fence_after();
        computing = -1;
        if (warp < 4) {
            // ---- epilogue: thread c holds column c of R = R_hi + R_lo (TMEM lane c)
            const int c = tid;
            const int64_t b = pair / p.HV;
            const int hv = pair % p.HV;
            float rh[16], rl[16];
            tmem_ld16x2_wait(tb + ((uint32_t)(32 * warp) << 16), tb + 16 + ((uint32_t)(32 * warp) << 16), rh, rl);
            float vv[T];
#pragma unroll
            for (int t = 0; t < T; ++t) vv[t] = __bfloat162float(aux.v[t][c]);
            float dl[T];
#pragma unroll
            for (int t = 0; t < T; ++t) {
                float a = cf.dk[t] * ((rh[t] + rl[t]) * cf.rk[t]);
#pragma unroll
                for (int u = 0; u < t; ++u) a = __fmaf_rn(cf.ck[t][u], dl[u], a);
                dl[t] = cf.beta[t] * __fmaf_rn(-cf.dec[t], a, vv[t]);
                float ot = cf.dq[t] * ((rh[T + t] + rl[T + t]) * cf.rq[t]);
#pragma unroll
                for (int u = 0; u <= t; ++u) ot = __fmaf_rn(cf.cq[t][u], dl[u], ot);
                const int64_t gi = (b * T + t) * p.HV + hv;
                p.deltas[gi * kHeadDim + c] = dl[t];
                if constexpr (NORM) nb.xs[t][c] = round_bf16(ot);
                else p.o[gi * kHeadDim + c] = __float2bfloat16_rn(ot);
            }
            if constexpr (NORM) {
                // The output-gated RMSNorm of each token's row of 128 (GatedRMSNorm.forward,
                // model/model.py:150-158) in the standalone norm kernel's order: lane l of a 16-lane
                // group sums the squares of elements 8 l .. 8 l + 7, the group adds by xor shuffles.
                named_sync(kBarDrain, 128);
                {
                    const int t = c >> 4 < T ? c >> 4 : 0, l = c & 15;
                    float xs8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) xs8[e] = nb.xs[t][8 * l + e];
                    float sq = sum_squares8(xs8);
#pragma unroll
                    for (int off = 8; off > 0; off >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, off));
                    if (l == 0 && (c >> 4) < T) nb.inv[t] = gated_norm_inv(sq, p.eps);
                }
                named_sync(kBarDrain, 128);
                const float wc = __bfloat162float(p.norm_w[c]);
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    const float normed = round_bf16(nb.xs[t][c] * nb.inv[t]);
                    const float weighted = round_bf16(wc * normed);
                    const float yv = weighted * silu_f32(__bfloat162float(nb.z[j & 1][t][c]));
                    p.y[((b * T + t) * p.HV + hv) * kHeadDim + c] = __float2bfloat16_rn(yv);
                }
            }
        } else if (j + 1 < npairs) {
            // ---- warps 4-7: the next pair's prefetched inputs (the products that read the rows are done)
            deposit<T>(pf, vb, sh.aux[(j + 1) & 1], tid - 128, z_buffer(nb, (j + 1) & 1));
        }
        tc_fence_before();
        __syncthreads();
    }
    // products still in flight (after a wait gave up) end before the CTA leaves
    if (tid == kIssuer && computing >= 0) {
        mbar_wait(&sh.acc_gram, (uint32_t)computing, kSiteGram);
        mbar_wait(&sh.acc, (uint32_t)computing, kSiteProduct);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tb, kTmemCols);
}

}  // namespace vblock

int launch_verify_block(const VerifyBlockArgs& a, cudaStream_t s) {
    using namespace vblock;
    if (a.rows == 0 || a.T == 0) return GDN_OK;
    if (a.T > kMaxT || a.T < 1) return GDN_ERR_UNSUPPORTED;
    static bool ready[64] = {false};
    static int sms[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_LAUNCH;
    if (!ready[dev]) {
        bool ok = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms[dev] > 0;
#define GDN_VB_ATTR(TT)                                                                                          \
        ok = ok &&                                                                                               \
             cudaFuncSetAttribute(verify_block_kernel<TT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                  (int)kSmem) == cudaSuccess &&                                                  \
             cudaFuncSetAttribute(verify_block_kernel<TT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                  (int)kSmem) == cudaSuccess;
        GDN_VB_ATTR(1) GDN_VB_ATTR(2) GDN_VB_ATTR(3) GDN_VB_ATTR(4) GDN_VB_ATTR(5) GDN_VB_ATTR(6) GDN_VB_ATTR(7)
        GDN_VB_ATTR(8)
#undef GDN_VB_ATTR
        if (!ok) return GDN_ERR_LAUNCH;
        ready[dev] = true;
    }
    const int64_t pairs = a.rows * a.HV;
    if (pairs > INT32_MAX) return GDN_ERR_SHAPE;
    Params p;
    memset(&p, 0, sizeof(p));
    p.state = a.state_in;
    p.q = static_cast<const bf16*>(a.q);
    p.k = static_cast<const bf16*>(a.k);
    p.v = static_cast<const bf16*>(a.v);
    p.g = a.g;
    p.beta = a.beta;
    p.beta_f32 = a.beta_dtype == GDN_F32;
    p.o = static_cast<bf16*>(a.o);
    p.deltas = a.deltas;
    p.z = static_cast<const bf16*>(a.z);
    p.norm_w = static_cast<const bf16*>(a.norm_w);
    p.y = static_cast<bf16*>(a.y);
    p.eps = a.eps;
    p.qsb = a.qsb; p.qst = a.qst; p.qsh = a.qsh;
    p.ksb = a.ksb; p.kst = a.kst; p.ksh = a.ksh;
    p.vsb = a.vsb; p.vst = a.vst; p.vsh = a.vsh;
    p.HV = a.HV;
    p.rep = a.HV / a.H;
    p.pairs = (int)pairs;
    p.scale = a.scale;
    const int64_t slots = 2 * (int64_t)sms[dev];  // two CTAs an SM: one's serial phases overlap the other's
    const int grid = (int)(pairs < slots ? pairs : slots);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.dependent ? 1 : 0;
    cudaError_t err;
    switch (a.T) {
#define GDN_VB_CASE(TT)                                                                                   \
        case TT:                                                                                          \
            err = a.y ? cudaLaunchKernelEx(&cfg, verify_block_kernel<TT, true>, p)                        \
                      : cudaLaunchKernelEx(&cfg, verify_block_kernel<TT, false>, p);                      \
            break;
        GDN_VB_CASE(1) GDN_VB_CASE(2) GDN_VB_CASE(3) GDN_VB_CASE(4) GDN_VB_CASE(5) GDN_VB_CASE(6) GDN_VB_CASE(7)
        GDN_VB_CASE(8)
#undef GDN_VB_CASE
        default: return GDN_ERR_UNSUPPORTED;
    }
    return err == cudaSuccess ? launch_status() : GDN_ERR_LAUNCH;
}

// The engine's verify branch of a delta layer (conv_step, delta_outputs, norm;
// inference/engine.py:427-435) in one call. The block verify is a programmatic dependent of the
// conv step: the conv does not write the states, so the block's CTAs set up, allocate TMEM and load
// their first states while the conv runs. For few states the gated norm runs in the block's drain;
// otherwise the block writes its outputs into y and the standalone norm normalises y in place, as
// a programmatic dependent of the block.
int launch_verify_layer(const VerifyLayerArgs& a, cudaStream_t s) {
    if (a.B == 0 || a.T == 0) return GDN_OK;  // nothing launched, so nothing may depend on a launch
    if (a.T > vblock::kMaxT) return GDN_ERR_UNSUPPORTED;
    const int64_t key_dim = (int64_t)a.H * kHeadDim, value_dim = (int64_t)a.HV * kHeadDim;
    // (the conv launched as a programmatic dependent of the previous layer's last kernel measured
    // slower at 16 rows, 0.791 -> 0.810 ms a config-4 step, and equal above)
    int st = launch_conv_step(a.conv_state, a.qkv, a.qkv_sb, a.qkv_st, a.conv_w, a.ext, a.q, a.k, a.v, a.B, a.T,
                              a.taps, a.K, key_dim, value_dim, kHeadDim, kHeadDim, s);
    if (st != GDN_OK) return st;
    VerifyBlockArgs b{};
    b.q = a.q; b.k = a.k; b.v = a.v;
    b.g = a.g; b.beta = a.beta; b.beta_dtype = a.beta_dtype;
    b.state_in = a.state;
    b.deltas = a.deltas;
    b.rows = a.B; b.T = a.T;
    b.H = a.HV; b.HV = a.HV;  // q and k come repeat-interleaved to the value heads
    const int64_t tok = value_dim;
    b.qsb = b.ksb = b.vsb = a.T * tok;
    b.qst = b.kst = b.vst = tok;
    b.qsh = b.ksh = b.vsh = kHeadDim;
    b.scale = a.scale;
    b.dependent = true;
    const bool fused = a.B * a.HV < kVerifyFusedNormStates;
    if (fused) {
        b.z = a.z; b.norm_w = a.norm_w; b.y = a.y; b.eps = a.eps;
    } else {
        b.o = a.y;
    }
    st = launch_verify_block(b, s);
    if (st != GDN_OK || fused) return st;
    return launch_gated_rmsnorm(a.y, a.z, a.norm_w, a.y, a.B * a.T * a.HV, kHeadDim, a.eps, s, true);
}

}  // namespace gdn
