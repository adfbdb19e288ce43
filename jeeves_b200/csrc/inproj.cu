// The gated-delta layer's merged input projection with the causal conv fused into the GEMM's
// epilogue (tcgen05). The prefill branch of GatedDeltaNet.forward computes qkv = in_proj_qkv(x)
// and, beside it, z, b and a (model/model.py:459-462; on CUDA the engine runs the projections that
// read one input as one GEMM, inference/engine.py:155-166, :376), then keeps the last pre-conv rows
// as the conv state and applies qkv = silu(causal_conv1d(qkv)) (model/model.py:469-470, :478-479). Here
// one call computes Y = X W^T for the merged weight W = [W_qkv; W_rest] ([N, K], nn.Linear
// layout) and writes
//   out[t, c] = silu(conv_c(Y_bf16[t-3..t, c]))   for c < C (the qkv channels),
//   out[t, c] = Y_bf16[t, c]                       for c >= C,
// with Y rounded to bf16 first and the conv output rounded to bf16 before the SiLU, as the two
// eager steps do (the conv in fp32 fused multiply-adds in tap order, the SiLU with the hardware
// exponential and reciprocal: within one bf16 unit of the conv kernel's exact rounding). With
// cu_seqlens the window restarts at every sequence. Optionally the last `taps` pre-conv rows of
// each sequence go to conv_tail [nseq, C, taps] (the conv state the cache keeps,
// model/model.py:469, :478).
//
// The product is computed transposed, Y^T = W X^T, so that a tile's accumulator holds 128
// channels in the TMEM lanes and `bn` consecutive tokens in its columns: the thread that owns a
// channel's lane walks its tokens in order and keeps the conv window in registers, with no
// shared-memory staging. A tile's columns are tokens t0 - 3 .. t0 + bn - 4 (the three before t0
// recomputed for the window; TMA fills rows before 0 and past T with zeros), and it writes the
// bn - 3 tokens from t0 on. Without conv channels (the decode-time projections and the output
// projection) there is no window: a tile's bn columns are tokens t0 .. t0 + bn - 1.
//
// The kernel is persistent (one CTA per SM, tiles strided by the grid, tokens fastest so that the
// CTAs running at once share the activations and a few weight panels in L2). Warp 8 streams
// 64-wide K slices of W and X with TMA (128-byte swizzle) through as many stages as fit (four at
// the widest tile, up to eight for narrow ones); warp 9 issues
// tcgen05.mma (M = 128, N = bn, K = 16) into one of two 256-column accumulators, so that the
// products of the next tile run while warps 0-7 drain the previous one (warp w reads TMEM lane
// quadrant w % 4 and half w / 4 of the columns).

#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"
#include "tensor_map.h"

namespace gdn {
namespace inproj {

using namespace sm100;

constexpr int kBM = 128;                 // channels per tile (the MMA's M)
constexpr int kHalo = 3;                 // tokens before the tile's outputs (taps - 1 of a 4-tap conv)
constexpr int kMaxBN = 256;              // tokens per tile at most (the MMA's N)
constexpr int kBK = 64;                  // K per stage (one 128-byte swizzle panel)
constexpr int kMaxStages = 8;             // single-CTA stages: as many as fit (4 at the widest tile)
constexpr uint32_t kSmemLimit = 232448 - 1024;  // 227 KB a CTA, less room for the static variables
constexpr uint32_t kAStage = kBM * 128;     // 16 KB of W
constexpr int kEpilogueWarps = 8;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 32 * (kEpilogueWarps + 2);
constexpr int kConvertWarps = 4;  // fp8 weights: warps 10-13 turn e4m3 codes into the fp16 operand
constexpr int kFp8Threads = kThreads + 32 * kConvertWarps;
// fp8 stages: the fp16 weight operand (16 KB), the activation rows (up to 32 KB), the raw codes
// that TMA brings (128 rows x 64 codes, 8 KB)
constexpr uint32_t kRawStage = kBM * kBK;

constexpr uint32_t kAccCols = 256;       // columns of one accumulator; two of them fill TMEM
constexpr int kChunk = 16;               // accumulator columns per TMEM load

struct Params {
    CUtensorMap tm_w;  // 2-D (K, N), box (64, 128); fp8: the codes, uint8, no swizzle
    CUtensorMap tm_x;  // 2-D (K, T), box (64, bn)
    CUtensorMap tm_out;  // split K with out_tma: 2-D (N, T) bf16 over out, box (32, 16)
    const bf16* conv_w;  // [C, 4]
    const int32_t* cu_seqlens;  // [nseq + 1] or null (one sequence of T tokens)
    bf16* out;           // [T, N], row stride ldo
    bf16* conv_tail;     // [nseq, C, 4] or null
    int64_t ldo;
    int T, N, C, K, nseq;
    int bn;              // tokens per tile, a multiple of 32 in [64, 256]
    int halo;            // leading columns recomputed for the conv window: kHalo with a conv, else 0
    int tiles_t, tiles;  // token tiles, all tiles
    int stages;          // single-CTA kernel: pipeline stages (as many as fit, at most 8)
    int ksplit;          // single-CTA kernel: CTAs of a cluster that split K (1: no split)
    int out_tma;         // split K: the owners store their outputs with tm_out
    uint32_t stage_bytes;  // single-CTA kernel: W (16 KB) + X (bn x 128 B) [+ raw codes (8 KB)]
    // fp8 weights (the single-CTA kernel with FP8 = true): e4m3 codes [N, K] (row stride ldc
    // bytes) with one fp32 scale per row, and the activations as fp16 rows with a power-of-two
    // scale per row (tm_x then maps those fp16 rows)
    const uint8_t* codes;
    int64_t ldc;
    const float* w_scale;
    const float* row_scale;
};

struct Shared {
    uint64_t full[kMaxStages], empty[kMaxStages], acc_full[2], acc_empty[2], mma_done;
    uint64_t codes_full[kMaxStages];  // fp8: the raw codes of a stage have landed
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// SiLU of a bf16-valued input with the hardware exponential and reciprocal: x / (1 + 2^(-x log2 e)).
// The epilogue's arithmetic runs beside the tensor cores and slows them (it shares the SM's power
// budget), so it takes the short form; against the exact quotient the bf16 result differs by at
// most one unit in the last place, and rarely. x below about -88 gives -0 (the divisor is
// infinite), 0 gives 0, NaN stays NaN.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// The sequence of token t of a packed batch: its first token, its end and its index.
__device__ __forceinline__ void find_sequence(const int32_t* cu, int nseq, int t, int& start, int& end, int& id) {
    int lo = 0, hi = nseq - 1;  // the last sequence that starts at or before t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(cu + mid) <= t) lo = mid;
        else hi = mid - 1;
    }
    id = lo;
    start = __ldg(cu + lo);
    end = __ldg(cu + lo + 1);
}

}  // namespace inproj
}  // namespace gdn

namespace gdn {
namespace inproj {

// Stores a lane's 16 values of one channel, tokens tb .. tb + 15 (column j of the tile first),
// skipping the halo columns and the tokens past T unless the whole chunk is known to be inside.
__device__ __forceinline__ void store_chunk(bf16* out_c, int64_t ldo, int tb, int j, int T, int halo, bool whole,
                                            const float (&v)[kChunk]) {
    bf16* q = out_c + (int64_t)tb * ldo;
    if (whole) {
#pragma unroll
        for (int e = 0; e < kChunk; ++e) q[e * ldo] = __float2bfloat16_rn(v[e]);
    } else {
#pragma unroll
        for (int e = 0; e < kChunk; ++e)
            if (j + e >= halo && tb + e < T) q[e * ldo] = __float2bfloat16_rn(v[e]);
    }
}

// Drains one warp's share of a finished accumulator: channel c (this lane's TMEM lane of quadrant
// `acc`), columns col0 .. col0 + ncols - 1, where column j is token row0 + j. The window carries
// the bf16-rounded pre-conv values of the three tokens before the current one; the drain of the
// second half of the columns starts it from the last three columns of the first half.
template <bool VARLEN, bool SCALED = false>
__device__ __forceinline__ void drain(const Params& p, uint32_t acc, int col0, int ncols, int row0, int c, int lane) {
    const bool in_n = c < p.N, conv = c < p.C;
    // fp8 weights: y = (acc x row scale) x weight scale, the order of the reference's fp8 GEMM
    const float ws = SCALED && in_n ? __ldg(p.w_scale + c) : 1.f;
    float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f;
    if (conv) {
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p.conv_w + (int64_t)c * 4));
        const bf16* h = reinterpret_cast<const bf16*>(&raw);
        w0 = to_f32(h[0]);
        w1 = to_f32(h[1]);
        w2 = to_f32(h[2]);
        w3 = to_f32(h[3]);
    }
    float x1 = 0.f, x2 = 0.f, x3 = 0.f;  // pre-conv values of tokens t - 3, t - 2, t - 1
    if (col0 > 0) {
        float v[kChunk];
        tmem_ld16_wait(acc + col0 - kChunk, v);
        if (SCALED) {
            const int t0 = row0 + col0 - kChunk;
#pragma unroll
            for (int e = kChunk - 3; e < kChunk; ++e)
                v[e] = v[e] * __ldg(p.row_scale + min(max(t0 + e, 0), p.T - 1)) * ws;
        }
        x1 = round_bf16(v[kChunk - 3]);
        x2 = round_bf16(v[kChunk - 2]);
        x3 = round_bf16(v[kChunk - 1]);
    }
    bf16* out_c = p.out + c;
#pragma unroll 1
    for (int j = col0; j < col0 + ncols; j += kChunk) {
        float v[kChunk];
        tmem_ld16_wait(acc + j, v);
        const int tb = row0 + j;  // token of column j
        int s_start = 0, s_end = p.T, s_id = 0;
        if (VARLEN) {
            const int t = tb + (lane & (kChunk - 1));
            if (t >= 0 && t < p.T) find_sequence(p.cu_seqlens, p.nseq, t, s_start, s_end, s_id);
        }
        float y[kChunk], pre[kChunk], res[kChunk];
#pragma unroll
        for (int e = 0; e < kChunk; ++e) {
            if (SCALED) v[e] = v[e] * __ldg(p.row_scale + min(max(tb + e, 0), p.T - 1)) * ws;
            y[e] = round_bf16(v[e]);
            float a1 = x1, a2 = x2, a3 = x3;
            if (VARLEN) {  // the window restarts at the token's sequence start
                const int t = tb + e, st = __shfl_sync(0xffffffffu, s_start, e);
                a1 = t - 3 >= st ? a1 : 0.f;
                a2 = t - 2 >= st ? a2 : 0.f;
                a3 = t - 1 >= st ? a3 : 0.f;
            }
            float s = w0 * a1;  // fused multiply-adds in tap order
            s = fmaf(w1, a2, s);
            s = fmaf(w2, a3, s);
            s = fmaf(w3, y[e], s);
            pre[e] = round_bf16(s);
            x1 = x2;
            x2 = x3;
            x3 = y[e];
        }
        if (conv) {
#pragma unroll
            for (int e = 0; e < kChunk; ++e) res[e] = silu_fast(pre[e]);
        }
        // a chunk past the halo and inside the tokens stores without per-token checks (warp-uniform)
        const bool whole = j >= p.halo && tb + kChunk <= p.T;
        if (conv) store_chunk(out_c, p.ldo, tb, j, p.T, p.halo, whole, res);
        else if (in_n) store_chunk(out_c, p.ldo, tb, j, p.T, p.halo, whole, y);
        if (conv && p.conv_tail) {  // the last four pre-conv tokens of each sequence (the cache's conv state)
#pragma unroll
            for (int e = 0; e < kChunk; ++e) {
                const int t = tb + e;
                const int end = VARLEN ? __shfl_sync(0xffffffffu, s_end, e) : p.T;
                const int id = VARLEN ? __shfl_sync(0xffffffffu, s_id, e) : 0;
                if (j + e >= p.halo && t < p.T && t >= end - 4)
                    p.conv_tail[((int64_t)id * p.C + c) * 4 + (4 - (end - t))] = __float2bfloat16_rn(y[e]);
            }
        }
    }
}

}  // namespace inproj
}  // namespace gdn

namespace gdn {
namespace inproj {

// Two e4m3 codes (the low 16 bits) as an fp16 pair: exact, every e4m3 value is an fp16 value.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t codes) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)(codes & 0xFFFFu)));
    return r;
}

// ---- split K (decode-sized batches without conv channels): the ks CTAs of a cluster compute one
// tile's partial products over consecutive K ranges, then sum them through distributed shared
// memory. The tile's token columns, in chunks of 16 (nch = bn / 16 of them), are dealt out in
// contiguous blocks to 2 ks workers: worker j = 2 x CTA + warp half (warps 4-7 are half 1) owns
// chunks [ceil(j nch / 2ks), ceil((j + 1) nch / 2ks)), so that every warp of every CTA sends and
// sums about the same share (warp w reads TMEM lane quadrant w % 4, i.e. 32 channels). A sender writes its partial of a chunk into a
// 2 KB slot of the owner's freed stage memory (32 lanes x 16 columns fp32, four columns per lane
// per 16-byte store, 512 contiguous bytes a warp store); the owner adds the ks partials in rank
// order (the same bits whichever CTA owns the chunk), rounds to bf16 into a [16 tokens][32
// channels] box and stores it with one TMA copy (or, when the output's layout does not allow a
// tensor map, with 2-byte stores per channel).
struct SplitLayout {
    int nch, maxown;  // chunks of 16 columns in the tile; chunks a CTA owns at most
    __device__ __forceinline__ SplitLayout(const Params& p)
        : nch(p.bn >> 4), maxown((nch + p.ksplit - 1) / p.ksplit) {}
    // first chunk of worker j = 2 x CTA + warp half (worker j covers [begin(j), begin(j + 1)))
    __device__ __forceinline__ int begin(const Params& p, int j) const { return (j * nch + 2 * p.ksplit - 1) / (2 * p.ksplit); }
    // slot of the owner's local chunk li of lane quadrant q from sender s, in the owner's memory
    __device__ __forceinline__ uint32_t slot(const Params& p, int q, int li, int s) const {
        return (uint32_t)(((q * maxown + li) * p.ksplit + s) * 2048);
    }
    __device__ __forceinline__ uint32_t box(const Params& p, int q, int li) const {
        return (uint32_t)(4 * maxown * p.ksplit * 2048 + (q * maxown + li) * 1024);
    }
};

__device__ __forceinline__ void split_send(const Params& p, uint8_t* sm, uint32_t tb, int w, int lane, int kr) {
    const SplitLayout L(p);
    const int q = w & 3, h = w >> 2;
    const uint32_t acc = tb + ((uint32_t)(32 * q) << 16);
    for (int o = 0; o < p.ksplit; ++o) {
        if (o == kr) continue;
        const int first = L.begin(p, 2 * o), u0 = L.begin(p, 2 * o + h), u1 = L.begin(p, 2 * o + h + 1);
        const uint32_t dst = mapa_shared(sm + L.slot(p, q, u0 - first, kr), (uint32_t)o);
        for (int u = u0; u < u1; ++u) {
            float v[kChunk];
            tmem_ld16_wait(acc + 16 * u, v);
            const uint32_t d = dst + (uint32_t)((u - u0) * p.ksplit * 2048);
#pragma unroll
            for (int i = 0; i < kChunk / 4; ++i)
                asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(d + (uint32_t)((i * 32 + lane) * 16)),
                             "f"(v[4 * i]), "f"(v[4 * i + 1]), "f"(v[4 * i + 2]), "f"(v[4 * i + 3])
                             : "memory");
        }
    }
}

template <bool SCALED>
__device__ __forceinline__ void split_finish(const Params& p, uint8_t* sm, uint32_t tb, int tile, int w, int lane, int kr) {
    if (tile >= p.tiles) return;
    const SplitLayout L(p);
    const int ks = p.ksplit, q = w & 3, h = w >> 2;
    const int first = L.begin(p, 2 * kr), u0 = L.begin(p, 2 * kr + h), u1 = L.begin(p, 2 * kr + h + 1);
    const int n0 = (tile / p.tiles_t) * kBM, t0 = (tile % p.tiles_t) * p.bn;
    const uint32_t acc = tb + ((uint32_t)(32 * q) << 16);
    const int c = n0 + 32 * q + lane;
    const float ws = SCALED && c < p.N ? __ldg(p.w_scale + c) : 1.f;
    for (int u = u0; u < u1; ++u) {
        const int li = u - first;
        float sum[kChunk];
        tmem_ld16_wait(acc + 16 * u, sum);  // this CTA's own partial
        float own[kChunk];
#pragma unroll
        for (int e = 0; e < kChunk; ++e) own[e] = sum[e];
        const uint8_t* slot = sm + L.slot(p, q, li, 0) + lane * 16;
        for (int s = 0; s < ks; ++s, slot += 2048) {  // rank order p_0 + p_1 + ..., whichever CTA owns the chunk
#pragma unroll
            for (int i = 0; i < kChunk / 4; ++i) {
                float4 f = make_float4(own[4 * i], own[4 * i + 1], own[4 * i + 2], own[4 * i + 3]);
                if (s != kr) f = *reinterpret_cast<const float4*>(slot + i * 512);
                if (s == 0) {
                    sum[4 * i] = f.x;
                    sum[4 * i + 1] = f.y;
                    sum[4 * i + 2] = f.z;
                    sum[4 * i + 3] = f.w;
                } else {
                    sum[4 * i] += f.x;
                    sum[4 * i + 1] += f.y;
                    sum[4 * i + 2] += f.z;
                    sum[4 * i + 3] += f.w;
                }
            }
        }
        const int tu = t0 + 16 * u;  // token of the chunk's first column
#pragma unroll
        for (int e = 0; e < kChunk; ++e) {
            if (SCALED) sum[e] = sum[e] * __ldg(p.row_scale + min(tu + e, p.T - 1)) * ws;
            sum[e] = round_bf16(sum[e]);
        }
        if (p.out_tma) {
            uint8_t* box = sm + L.box(p, q, li) + lane * 2;
#pragma unroll
            for (int e = 0; e < kChunk; ++e) *reinterpret_cast<bf16*>(box + e * 64) = __float2bfloat16_rn(sum[e]);
        } else if (c < p.N) {
            store_chunk(p.out + c, p.ldo, tu, 0, p.T, 0, tu + kChunk <= p.T, sum);
        }
    }
    if (p.out_tma && u1 > u0) {
        fence_async_smem();  // the boxes' generic-proxy stores become visible to the copy engine
        __syncwarp();
        if (lane == 0) {
            for (int u = u0; u < u1; ++u) tma_store_2d(&p.tm_out, sm + L.box(p, q, u - first), n0 + 32 * q, t0 + 16 * u);
            bulk_commit();
            bulk_wait_all();  // the boxes are read (and written out) before the CTA's memory goes away
        }
        __syncwarp();
    }
}

// The single-CTA kernel. FP8: the weight operand comes from e4m3 codes, which TMA brings into a
// raw area of each stage (128 rows x 64 codes) and warps 10-13 convert to fp16 in the 128-byte
// swizzled layout that TMA would have produced for bf16; the products are fp16 x fp16 (kind::f16)
// against the fp16 activation rows, and the drain applies the row and weight scales.
// NP: 64-wide K panels per stage. With fp8 codes two (K a multiple of 128): the codes of a stage
// then arrive as one box of 128-byte rows (128 codes of each of the 128 weight rows) instead of
// 64-byte rows, so that each copy request carries a whole line and a stage covers twice the K.
// A stage holds [NP weight panels][NP activation panels][raw codes: 128 rows x 64 NP bytes].
template <bool FP8, int NP = 1>
__global__ void __launch_bounds__(FP8 ? kFp8Threads : kThreads, 1) in_proj_conv_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    const int S = p.stages;
    const uint32_t xpanel = (uint32_t)p.bn * 128;
    const uint32_t stride = p.stage_bytes, x_off = NP * kAStage, raw_off = NP * (kAStage + xpanel);
    __shared__ Shared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kblocks = p.K / (kBK * NP);  // stages' worth of K
    // split K: the CTAs of a cluster share one tile, CTA kr taking K blocks [kb0, kb1); otherwise
    // the CTA walks the tiles with stride gridDim.x over all K blocks
    const int ks = p.ksplit;
    const int kr = ks > 1 ? (int)cluster_rank() : 0;
    const int kb0 = kblocks * kr / ks, kb1 = kblocks * (kr + 1) / ks;
    const int tfirst = ks > 1 ? (int)blockIdx.x / ks : (int)blockIdx.x;
    const int tstep = ks > 1 ? (int)gridDim.x / ks : (int)gridDim.x;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&sh.full[s], FP8 ? 1 + kConvertWarps : 1);  // the producer (+ the converters)
            mbar_init(&sh.empty[s], 1);
            mbar_init(&sh.codes_full[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sh.acc_full[b], 1);
            mbar_init(&sh.acc_empty[b], kEpilogueWarps);
        }
        mbar_init(&sh.mma_done, 1);
        sh.abort = 0;
        fence_mbar_init();
        tma_prefetch_map(&p.tm_w);
        tma_prefetch_map(&p.tm_x);
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, 2 * kAccCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;
    // Split-K launches are programmatic dependents of the previous kernel in the stream: the set-up
    // above (barriers, TMEM, tensor-map prefetch) overlaps that kernel's end; nothing in global
    // memory is read before this wait (a no-op for an ordinary launch).
    pdl_wait();

    if (warp == kProducerWarp) {
        // ============================== producer ==============================
        if (lane == 0) {
            const uint32_t bytes = NP * ((FP8 ? 0u : kAStage) + xpanel);
            int it = 0, s = 0;
            uint32_t ph = 0;  // parity of stage s's current use (the index and parity advance by steps:
                              // no division by the run-time stage count on these threads)
            bool ok = true;
            for (int tile = tfirst; ok && tile < p.tiles; tile += tstep) {
                const int n0 = (tile / p.tiles_t) * kBM;
                const int row0 = (tile % p.tiles_t) * (p.bn - p.halo) - p.halo;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    if (it >= S && !mbar_wait_or_abort(&sh.empty[s], ph ^ 1u, kSiteTmaLoad, &sh.abort, false)) {
                        atomicExch(&sh.abort, 1);
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm + s * stride;
                    mbar_arrive_expect_tx(&sh.full[s], bytes);
                    if (FP8) {
                        mbar_arrive_expect_tx(&sh.codes_full[s], NP * kRawStage);
                        tma_load_2d(st + raw_off, &p.tm_w, &sh.codes_full[s], kb * NP * kBK, n0);
                    } else {
#pragma unroll
                        for (int i = 0; i < NP; ++i)
                            tma_load_2d(st + i * kAStage, &p.tm_w, &sh.full[s], (kb * NP + i) * kBK, n0);
                    }
#pragma unroll
                    for (int i = 0; i < NP; ++i)
                        tma_load_2d(st + x_off + i * xpanel, &p.tm_x, &sh.full[s], (kb * NP + i) * kBK, row0);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            // the copies in flight land before the CTA's shared memory can go away
            for (int i = it > S ? it - S : 0; i < it; ++i) {
                if (FP8) mbar_wait(&sh.codes_full[i % S], (uint32_t)(i / S) & 1, kSiteDrain);
                mbar_wait(&sh.full[i % S], (uint32_t)(i / S) & 1, kSiteDrain);
            }
        }
    } else if (warp == kMmaWarp) {
        // ============================== MMA issuer ==============================
        if (lane == 0) {
            const uint32_t idesc = make_idesc(kBM, (uint32_t)p.bn, FP8 ? kFmtF16 : kFmtBF16, false, false);
            int lt = 0, s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int tile = tfirst; ok && tile < p.tiles; tile += tstep, ++lt) {
                const int b = lt & 1;
                const uint32_t acc = tb + b * kAccCols;
                if (lt >= 2 && !mbar_wait_or_abort(&sh.acc_empty[b], (uint32_t)((lt >> 1) - 1) & 1, kSiteReady,
                                                   &sh.abort, false)) {
                    atomicExch(&sh.abort, 1);
                    break;
                }
                tc_fence_after();
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait_or_abort(&sh.full[s], ph, kSiteTmaLoad, &sh.abort, false)) {
                        atomicExch(&sh.abort, 1);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t* st = sm + s * stride;
#pragma unroll
                    for (int i = 0; i < NP; ++i) {
                        const uint64_t da = sdesc_kmajor(st + i * kAStage, 0), db = sdesc_kmajor(st + x_off + i * xpanel, 0);
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk)
                            mma_f16(acc, sdesc_add(da, kk * 32), sdesc_add(db, kk * 32), idesc,
                                    (kb != kb0 || i != 0 || kk != 0) ? 1u : 0u);
                    }
                    mma_commit(&sh.empty[s]);  // the stage is free once these products have read it
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                mma_commit(&sh.acc_full[b]);  // also after a failed wait, so that no drain waits in vain
            }
            mma_commit(&sh.mma_done);
            mbar_wait(&sh.mma_done, 0, kSiteMma);  // every product issued is done before TMEM goes away
        }
    } else if (warp < kEpilogueWarps && ks > 1) {
        // split K: the one accumulator is complete; the sums across the cluster follow below
        if (!mbar_wait_or_abort(&sh.acc_full[0], 0, kSiteMma, &sh.abort)) atomicExch(&sh.abort, 1);
    } else if (warp < kEpilogueWarps) {
        // ================================ epilogue ================================
        const int q = warp & 3, half = p.bn >> 1, col0 = (warp >> 2) * half;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++lt) {
            const int b = lt & 1;
            if (!mbar_wait_or_abort(&sh.acc_full[b], (uint32_t)(lt >> 1) & 1, kSiteMma, &sh.abort)) {
                atomicExch(&sh.abort, 1);
                break;
            }
            if (*reinterpret_cast<volatile int*>(&sh.abort)) break;
            tc_fence_after();
            const int n0 = (tile / p.tiles_t) * kBM;
            const int row0 = (tile % p.tiles_t) * (p.bn - p.halo) - p.halo;
            const uint32_t acc = tb + b * kAccCols + ((uint32_t)(32 * q) << 16);
            const int c = n0 + 32 * q + lane;
            if (p.cu_seqlens) drain<true, FP8>(p, acc, col0, half, row0, c, lane);
            else drain<false, FP8>(p, acc, col0, half, row0, c, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.acc_empty[b]);  // the MMA may overwrite this accumulator
        }
    } else if constexpr (FP8) {
        // ============================ e4m3 -> fp16 converters ============================
        constexpr int kPer = NP * kBM * kBK / 16 / (32 * kConvertWarps);  // 16-code pieces per thread: 4 NP
        const int ct = tid - 32 * (kEpilogueWarps + 2);              // 0 .. 127
        const int my_tiles = tfirst < p.tiles ? (p.tiles - tfirst + tstep - 1) / tstep : 0;
        const int total = my_tiles * (kb1 - kb0);
        int s = 0;
        uint32_t ph = 0;
        for (int it = 0; it < total; ++it) {
            if (!mbar_wait_or_abort(&sh.codes_full[s], ph, kSiteTmaLoad, &sh.abort, false)) {
                atomicExch(&sh.abort, 1);
                break;
            }
            uint8_t* st = sm + s * stride;
            const uint8_t* raw = st + raw_off;  // row r of the codes at r * 64 NP
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                // piece (row, part): codes 16 part .. 16 part + 15 of the row, into panel part / 4
                const int id = ct + 32 * kConvertWarps * i, row = id / (4 * NP), part = id % (4 * NP);
                uint8_t* dst = st + (part / 4) * kAStage;
                const uint4 w = *reinterpret_cast<const uint4*>(raw + row * (kBK * NP) + part * 16);
                const uint4 lo = make_uint4(e4m3x2_to_f16x2(w.x), e4m3x2_to_f16x2(w.x >> 16), e4m3x2_to_f16x2(w.y),
                                            e4m3x2_to_f16x2(w.y >> 16));
                const uint4 hi = make_uint4(e4m3x2_to_f16x2(w.z), e4m3x2_to_f16x2(w.z >> 16), e4m3x2_to_f16x2(w.w),
                                            e4m3x2_to_f16x2(w.w >> 16));
                *reinterpret_cast<uint4*>(dst + sw128(row, 2 * (part % 4))) = lo;
                *reinterpret_cast<uint4*>(dst + sw128(row, 2 * (part % 4) + 1)) = hi;
            }
            fence_async_smem();  // the generic-proxy stores become visible to the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.full[s]);
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
    }
    if (ks > 1) {
        __syncwarp();
        tc_fence_before();
        cluster_sync();  // every CTA of the cluster is done with its products: its stages are free
        tc_fence_after();
        if (warp < kEpilogueWarps) split_send(p, sm, tb, warp, lane, kr);
        cluster_sync();  // the partial sums have landed
        if (warp < kEpilogueWarps) split_finish<FP8>(p, sm, tb, tfirst, warp, lane, kr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tb, 2 * kAccCols);
    }
}

// Activation rows for the fp8 GEMM: each bf16 row scaled by a power of two that puts its largest
// magnitude in [2^13, 2^14) (the exponent at most 126 down), converted to fp16, with the scale
// kept per row; the scaled bf16 values are exact in fp16 down to 2^-30 of the row's largest
// (the activation conversion of inference/fp8.py:30-52, FP16_TOP_EXPONENT = 13).
__global__ void __launch_bounds__(256) fp16_rows_kernel(const bf16* __restrict__ x, int64_t ldx, int K,
                                                        __half* __restrict__ xh, float* __restrict__ row_scale) {
    // the GEMM behind this kernel (a programmatic dependent when K is split) may start its set-up
    // now; it reads these rows only after its griddepcontrol.wait, i.e. after this grid completes
    pdl_launch_dependents();
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    const bf16* xr = x + row * ldx;
    float amax = 0.f;
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + k);
        const bf16* h = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(to_f32(h[e])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
    const int exponent = (int)((__float_as_uint(amax) >> 23) & 0xFFu) - 127;
    const int shift = max(exponent - 13, -126);
    const float down = __uint_as_float((uint32_t)(127 - shift) << 23);  // 2^-shift
    __half* out = xh + row * K;
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + k);
        const bf16* h = reinterpret_cast<const bf16*>(&raw);
        uint4 o;
        __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            o2[e] = __halves2half2(__float2half_rn(to_f32(h[2 * e]) * down), __float2half_rn(to_f32(h[2 * e + 1]) * down));
        *reinterpret_cast<uint4*>(out + k) = o;
    }
    if (threadIdx.x == 0) row_scale[row] = __uint_as_float((uint32_t)(shift + 127) << 23);
}

// The e4m3 codes [N, K] (row stride ldc bytes) as fp16 [N, K] (exact): the fp8 path's weight
// operand for the CTA-pair kernel at prefill sizes, where each weight panel is read by many token
// tiles and converting it once beats converting it in every tile. 16 codes a thread.
__global__ void __launch_bounds__(256) codes_to_f16_kernel(const uint8_t* __restrict__ codes, int64_t ldc,
                                                           __half* __restrict__ w16, int64_t N, int K) {
    const int64_t per_row = K / 16, total = N * per_row;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / per_row, k = (i % per_row) * 16;
        const uint4 w = *reinterpret_cast<const uint4*>(codes + row * ldc + k);
        const uint4 lo = make_uint4(e4m3x2_to_f16x2(w.x), e4m3x2_to_f16x2(w.x >> 16), e4m3x2_to_f16x2(w.y),
                                    e4m3x2_to_f16x2(w.y >> 16));
        const uint4 hi = make_uint4(e4m3x2_to_f16x2(w.z), e4m3x2_to_f16x2(w.z >> 16), e4m3x2_to_f16x2(w.w),
                                    e4m3x2_to_f16x2(w.w >> 16));
        uint4* dst = reinterpret_cast<uint4*>(w16 + row * K + k);
        dst[0] = lo;
        dst[1] = hi;
    }
}

// ------------------------------------------------------------------------------------------
// The CTA-pair form: a cluster of two CTAs computes a 256-channel x bn-token tile with
// tcgen05.mma.cta_group::2 (M = 256). Each CTA stages its own 128 weight rows and half of the
// tile's tokens (32 KB a stage instead of 48 KB), so that each SM reads two thirds of the bytes
// per product from L2 and from its shared memory; the leader's thread 320 issues the products
// into both SMs' accumulators, and each CTA drains its own 128 channels as above.
// ------------------------------------------------------------------------------------------
constexpr int kPairStages = 6;
constexpr uint32_t kPairStageBytes = kAStage + (kMaxBN / 2) * 128;  // 32 KB
constexpr uint32_t kPairSmemBytes = kPairStages * kPairStageBytes + 1024;
constexpr int kPairBM = 2 * kBM;  // channels per pair tile

struct PairShared {
    uint64_t full[kPairStages], empty[kPairStages], acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    int abort;
};

// Raises the abort flag of both CTAs of the pair, so that the other's waits give up too.
__device__ __forceinline__ void pair_abort(int* abort, uint32_t rank) {
    atomicExch(abort, 1);
    asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(abort, rank ^ 1u)), "r"(1)
                 : "memory");
}

// F16: fp16 operands (the fp8 path's fp16 activation rows against an fp16 copy of the weights
// that codes_to_f16_kernel made), and the drain applies the row and weight scales.
template <bool F16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    in_proj_conv_pair_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ PairShared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();  // 0: the leader, which issues the products
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int kblocks = p.K / kBK;
    const int half_bn = p.bn >> 1;

    if (tid == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sh.acc_full[b], 1);
            mbar_init(&sh.acc_empty[b], 2 * kEpilogueWarps);  // the drains of both CTAs
        }
        mbar_init(&sh.mma_done, 1);
        sh.abort = 0;
        fence_mbar_init();
        tma_prefetch_map(&p.tm_w);
        tma_prefetch_map(&p.tm_x);
    }
    if (warp == 0) {
        tmem_alloc_pair(&sh.tmem_base, 2 * kAccCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;

    if (warp == kProducerWarp) {
        // ============================== producers (both CTAs) ==============================
        if (lane == 0) {
            const uint32_t bytes = 2 * (kAStage + (uint32_t)half_bn * 128);  // both CTAs' copies
            int it = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < p.tiles; tile += npairs) {
                const int tt = tile % p.tiles_t, nn = tile / p.tiles_t;
                // this CTA's weight rows and token rows; a start past the matrix is moved back
                // inside it (those rows feed only channels or tokens that are not written)
                int n0 = nn * kPairBM + kBM * (int)rank;
                int r0 = tt * (p.bn - p.halo) - p.halo + (int)rank * half_bn;
                if (n0 >= p.N) n0 = max(p.N - kBM, 0);
                if (r0 >= p.T) r0 = p.T - 1;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (it >= kPairStages &&
                        !mbar_wait_or_abort(&sh.empty[s], (uint32_t)(it / kPairStages - 1) & 1, kSiteTmaLoad,
                                            &sh.abort, false, kWaitCycles, true)) {
                        pair_abort(&sh.abort, rank);
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm + s * kPairStageBytes;
                    if (rank == 0) mbar_arrive_expect_tx(&sh.full[s], bytes);
                    const uint32_t bar = mapa_shared(&sh.full[s], 0);
                    tma_load_2d_pair(st, &p.tm_w, bar, kb * kBK, n0);
                    tma_load_2d_pair(st + kAStage, &p.tm_x, bar, kb * kBK, r0);
                }
            }
            if (rank == 0)  // the copies in flight land before the shared memory can go away
                for (int i = it > kPairStages ? it - kPairStages : 0; i < it; ++i)
                    mbar_wait(&sh.full[i % kPairStages], (uint32_t)(i / kPairStages) & 1, kSiteDrain);
        }
    } else if (warp == kMmaWarp) {
        // ============================== MMA issuer (leader) ==============================
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = make_idesc(kPairBM, (uint32_t)p.bn, F16 ? kFmtF16 : kFmtBF16, false, false);
            int it = 0, lt = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < p.tiles; tile += npairs, ++lt) {
                const int b = lt & 1;
                const uint32_t acc = tb + b * kAccCols;
                if (lt >= 2 && !mbar_wait_or_abort(&sh.acc_empty[b], (uint32_t)((lt >> 1) - 1) & 1, kSiteReady,
                                                   &sh.abort, false, kWaitCycles, true)) {
                    pair_abort(&sh.abort, rank);
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (!mbar_wait_or_abort(&sh.full[s], (uint32_t)(it / kPairStages) & 1, kSiteTmaLoad, &sh.abort,
                                            false, kWaitCycles, true)) {
                        pair_abort(&sh.abort, rank);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t* st = sm + s * kPairStageBytes;
                    const uint64_t da = sdesc_kmajor(st, 0), db = sdesc_kmajor(st + kAStage, 0);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_f16_pair(acc, sdesc_add(da, kk * 32), sdesc_add(db, kk * 32), idesc,
                                     (kb | kk) != 0 ? 1u : 0u);
                    mma_commit_pair(&sh.empty[s], 3);  // both CTAs' stages are free once read
                }
                mma_commit_pair(&sh.acc_full[b], 3);  // also after a failed wait
            }
            mma_commit_pair(&sh.mma_done, 1);
            mbar_wait(&sh.mma_done, 0, kSiteMma);  // every product issued is done before TMEM goes away
        }
    } else {
        // ================================ epilogue (both CTAs) ================================
        const int q = warp & 3, half = p.bn >> 1, col0 = (warp >> 2) * half;
        int lt = 0;
        for (int tile = pair; tile < p.tiles; tile += npairs, ++lt) {
            const int b = lt & 1;
            if (!mbar_wait_or_abort(&sh.acc_full[b], (uint32_t)(lt >> 1) & 1, kSiteMma, &sh.abort, true, kWaitCycles,
                                    true)) {
                pair_abort(&sh.abort, rank);
                break;
            }
            if (*reinterpret_cast<volatile int*>(&sh.abort)) break;
            tc_fence_after();
            const int tt = tile % p.tiles_t, nn = tile / p.tiles_t;
            const int row0 = tt * (p.bn - p.halo) - p.halo;
            const uint32_t acc = tb + b * kAccCols + ((uint32_t)(32 * q) << 16);
            const int c = nn * kPairBM + kBM * (int)rank + 32 * q + lane;
            if (p.cu_seqlens) drain<true, F16>(p, acc, col0, half, row0, c, lane);
            else drain<false, F16>(p, acc, col0, half, row0, c, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&sh.acc_empty[b], 0));  // the leader may overwrite it
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no CTA frees its TMEM or leaves while the other may still signal it
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tb, 2 * kAccCols);
    }
}

// 2-D map over a [rows, K] 16-bit matrix (bf16, or fp16 for the fp8 path's activation rows) with
// row stride ld (elements), box (64, box_rows).
static bool make_map2(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld, uint32_t box_rows,
                      CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over the bf16 output [T, N] (row stride ld elements) for the split-K owners' stores:
// box (32 channels, box_rows tokens), no swizzle; the copies clip at T and N.
static bool make_out_map(CUtensorMap* map, void* base, int64_t T, int64_t N, int64_t ld, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {32, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over the e4m3 codes [rows, K] (row stride ld bytes), box (64 np, 128), rows kept as they are.
static bool make_codes_map(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld, int np) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld};
    cuuint32_t box[2] = {(cuuint32_t)(kBK * np), (cuuint32_t)kBM};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tokens per tile: the candidate with the shortest estimated makespan, counted as rounds of tiles
// over the persistent CTAs (or CTA pairs) times the tile's columns plus a fixed cost per tile
// (pipeline fill and drain, in columns); ties go to the wider tile, which reads fewer bytes per
// product.
static int choose_bn(int64_t T, int64_t N, int ctas, int tile_channels, int halo) {
    static const int kCandidates[] = {256, 224, 192, 160, 128, 96, 64};
    constexpr int64_t kTileCost = 288;  // fitted to the measured times of the widths at T = 4096
    const int64_t tiles_n = (N + tile_channels - 1) / tile_channels;
    int best = 256;
    int64_t best_cost = INT64_MAX;
    for (int bn : kCandidates) {
        const int64_t tiles = (T + bn - halo - 1) / (bn - halo) * tiles_n;
        const int64_t grid = tiles < ctas ? tiles : ctas;
        const int64_t cost = (tiles + grid - 1) / grid * (bn + kTileCost);
        if (cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

// Clusters of `ks` single CTAs (one per SM at the largest stage ring) that can be resident at once.
static int max_split_clusters(int dev, bool fp8, int ks) {
    static int cache[64][2][4];  // [device][fp8][log2 ks - 1], 0 = not asked yet, -1 = none
    const int li = ks == 2 ? 0 : ks == 4 ? 1 : 2;
    int& slot = cache[dev][fp8 ? 1 : 0][li];
    if (slot == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)ks);
        cfg.blockDim = dim3((unsigned)(fp8 ? kFp8Threads : kThreads));
        cfg.dynamicSmemBytes = kSmemLimit;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)ks;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        const cudaError_t e = fp8 ? cudaOccupancyMaxActiveClusters(&n, in_proj_conv_kernel<true>, &cfg)
                                  : cudaOccupancyMaxActiveClusters(&n, in_proj_conv_kernel<false>, &cfg);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
        }
        slot = n > 0 ? n : -1;
    }
    return slot;
}

}  // namespace inproj

size_t in_proj_fp8_workspace_bytes(int64_t T, int64_t K) {
    return ((size_t)T * K * 2 + 255) / 256 * 256 + (size_t)T * 4;
}

// Offset of the fp16 weight copy in an fp8 workspace (after the rows and their scales).
static size_t fp8_w16_offset(int64_t T, int64_t K) { return (in_proj_fp8_workspace_bytes(T, K) + 255) / 256 * 256; }

size_t in_proj_fp8_pair_workspace_bytes(int64_t T, int64_t K, int64_t N) {
    return fp8_w16_offset(T, K) + (size_t)N * K * 2;
}

namespace inproj {

// The kernels' shared-memory limits and the device's SM count, once per device.
static int device_sms(int& dev) {
    static bool ready[64] = {false};
    static int sms[64] = {0};
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (!ready[dev]) {
        if (cudaFuncSetAttribute(in_proj_conv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemLimit) != cudaSuccess ||
            cudaFuncSetAttribute(in_proj_conv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemLimit) != cudaSuccess ||
            cudaFuncSetAttribute(in_proj_conv_kernel<true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemLimit) != cudaSuccess ||
            cudaFuncSetAttribute(in_proj_conv_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kPairSmemBytes) != cudaSuccess ||
            cudaFuncSetAttribute(in_proj_conv_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kPairSmemBytes) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms[dev] < 1)
            return 0;
        ready[dev] = true;
    }
    return sms[dev];
}

// How a shape runs: K split over clusters of ks CTAs (decode-sized batches without conv
// channels), CTA pairs with bn_pair-token tiles (when the pair tiles fill every pair of SMs; with
// fp8 weights only if `fp8_pair`, i.e. the workspace holds an fp16 copy of the weights), or single
// CTAs.
struct Plan {
    int ks = 1, bn_pair = 0, halo = 0;
    bool use_pair = false;
    int64_t pair_tiles = 0;
};

static Plan plan_shape(int64_t T, int64_t N, int64_t K, int64_t C, bool fp8, bool fp8_pair, int dev, int sms) {
    Plan pl;
    const int pairs = sms / 2;
    // without conv channels no tile needs the window's leading tokens
    pl.halo = C > 0 ? kHalo : 0;
    pl.bn_pair = choose_bn(T, N, pairs, kPairBM, pl.halo);
    pl.pair_tiles = (T + pl.bn_pair - pl.halo - 1) / (pl.bn_pair - pl.halo) * ((N + kPairBM - 1) / kPairBM);
    // Decode-sized batches without conv channels: all tokens in one tile, and K split over a
    // cluster of ks CTAs so that the tiles (one per 128 weight rows) cover the SMs; each CTA then
    // streams 1 / ks of its weight rows (the stage ring's copies, not the products, bound these
    // shapes). A split needs at least 4 K blocks a CTA and every cluster resident at once.
    if (C == 0 && T <= kMaxBN && K % kBK == 0) {
        const int64_t tiles_n = (N + kBM - 1) / kBM;
        for (int cand = 8; cand >= 2; cand >>= 1)
            if (tiles_n * cand <= sms && K / kBK >= 4 * cand && max_split_clusters(dev, fp8, cand) >= tiles_n) {
                pl.ks = cand;
                break;
            }
    }
    pl.use_pair = pl.ks == 1 && (!fp8 || fp8_pair) && pairs >= 1 && pl.pair_tiles >= pairs;
    return pl;
}

}  // namespace inproj

size_t in_proj_fp8_prefill_workspace_bytes(int64_t T, int64_t K, int64_t N, int64_t C) {
    using namespace inproj;
    int dev = 0;
    const int sms = device_sms(dev);
    const size_t base = in_proj_fp8_workspace_bytes(T, K);
    if (sms < 1) return base;
    return plan_shape(T, N, K, C, true, true, dev, sms).use_pair ? in_proj_fp8_pair_workspace_bytes(T, K, N) : base;
}

int launch_in_proj_conv(const InProjArgs& a, cudaStream_t s) {
    using namespace inproj;
    if (a.T == 0 || a.N == 0) return GDN_OK;
    int dev = 0;
    const int nsm = device_sms(dev);
    if (nsm < 1) return GDN_ERR_LAUNCH;
    const bool fp8 = a.codes != nullptr;
    // fp8 weights run on CTA pairs too when the workspace also holds an fp16 copy of the weights
    // (gdn_in_proj_fp8_prefill_workspace_size): one conversion pass, then fp16 x fp16 products
    const bool fp8_pair = fp8 && a.workspace_bytes >= in_proj_fp8_pair_workspace_bytes(a.T, a.K, a.N);
    const Plan pl = plan_shape(a.T, a.N, a.K, a.C, fp8, fp8_pair, dev, nsm);
    const int ks = pl.ks, halo = pl.halo, bn_pair = pl.bn_pair, pairs = nsm / 2;
    const bool use_pair = pl.use_pair;
    Params p;
    memset(&p, 0, sizeof(p));
    p.ksplit = ks;
    p.bn = ks > 1 ? (int)((a.T + 31) / 32 * 32) : use_pair ? bn_pair : choose_bn(a.T, a.N, nsm, kBM, halo);
    p.halo = halo;
    // fp8 with K split at up to 32 rows: stages of two K panels, the codes in 128-byte rows (as
    // many K blocks in flight as eight one-panel stages; measured 21.0 -> 19.1-19.8 us at 32 rows).
    // Wider token tiles keep one panel: their two-panel stages fit only twice (256 rows 29.0 -> 31.8).
    const int np = fp8 && ks > 1 && p.bn <= 32 && a.K % (2 * kBK) == 0 ? 2 : 1;
    __half* xh = nullptr;
    if (fp8) {
        if (!a.workspace || a.workspace_bytes < in_proj_fp8_workspace_bytes(a.T, a.K)) return GDN_ERR_WORKSPACE;
        xh = static_cast<__half*>(a.workspace);
        p.codes = static_cast<const uint8_t*>(a.codes);
        p.ldc = a.ldc;
        p.w_scale = a.w_scale;
        p.row_scale = reinterpret_cast<const float*>(static_cast<uint8_t*>(a.workspace) +
                                                     ((size_t)a.T * a.K * 2 + 255) / 256 * 256);
        if (use_pair) {
            __half* w16 = reinterpret_cast<__half*>(static_cast<uint8_t*>(a.workspace) + fp8_w16_offset(a.T, a.K));
            if (!make_map2(&p.tm_x, xh, a.T, a.K, a.K, (uint32_t)(p.bn / 2), CU_TENSOR_MAP_DATA_TYPE_FLOAT16) ||
                !make_map2(&p.tm_w, w16, a.N, a.K, a.K, kBM, CU_TENSOR_MAP_DATA_TYPE_FLOAT16))
                return GDN_ERR_LAUNCH;
        } else if (!make_map2(&p.tm_x, xh, a.T, a.K, a.K, (uint32_t)p.bn, CU_TENSOR_MAP_DATA_TYPE_FLOAT16) ||
                   !make_codes_map(&p.tm_w, a.codes, a.N, a.K, a.ldc, np)) {
            return GDN_ERR_LAUNCH;
        }
    } else if (!make_map2(&p.tm_w, a.w, a.N, a.K, a.ldw, kBM) ||
               !make_map2(&p.tm_x, a.x, a.T, a.K, a.ldx, (uint32_t)(use_pair ? p.bn / 2 : p.bn))) {
        return GDN_ERR_LAUNCH;
    }
    p.conv_w = static_cast<const bf16*>(a.conv_w);
    p.cu_seqlens = a.cu_seqlens;
    p.out = static_cast<bf16*>(a.out);
    p.conv_tail = static_cast<bf16*>(a.conv_tail);
    p.ldo = a.ldo;
    p.T = (int)a.T;
    p.N = (int)a.N;
    p.C = (int)a.C;
    p.K = (int)a.K;
    p.nseq = (int)a.nseq;
    const int tile_channels = use_pair ? kPairBM : kBM;
    const int64_t tiles_t = (a.T + p.bn - halo - 1) / (p.bn - halo);
    const int64_t tiles = tiles_t * ((a.N + tile_channels - 1) / tile_channels);
    if (tiles > INT32_MAX) return GDN_ERR_SHAPE;
    p.tiles_t = (int)tiles_t;
    p.tiles = (int)tiles;
    if (a.conv_tail &&
        cudaMemsetAsync(a.conv_tail, 0, (size_t)a.nseq * a.C * 4 * sizeof(bf16), s) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    p.stage_bytes = (uint32_t)np * (kAStage + (uint32_t)p.bn * 128 + (fp8 ? kRawStage : 0u));
    p.stages = (int)((kSmemLimit - 1024) / p.stage_bytes);
    if (p.stages > kMaxStages) p.stages = kMaxStages;
    const uint32_t single_smem = (uint32_t)p.stages * p.stage_bytes + 1024;
    if (fp8)
        fp16_rows_kernel<<<(unsigned)a.T, 256, 0, s>>>(static_cast<const bf16*>(a.x), a.ldx, (int)a.K, xh,
                                                         const_cast<float*>(p.row_scale));
    if (ks > 1) {
        // the partial sums' slots (4 lane quadrants x the chunks a CTA owns at most x ks senders x
        // 2 KB) and the owners' output boxes (1 KB a chunk) reuse the stage ring after the products
        const uint32_t maxown = (uint32_t)((p.bn / 16 + ks - 1) / ks);
        if (4u * maxown * ((uint32_t)ks * 2048u + 1024u) > (uint32_t)p.stages * p.stage_bytes) return GDN_ERR_LAUNCH;
        p.out_tma = (reinterpret_cast<uintptr_t>(a.out) % 16 == 0 && (a.ldo * 2) % 16 == 0 &&
                     make_out_map(&p.tm_out, a.out, a.T, a.N, a.ldo, 16u))
                        ? 1
                        : 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(tiles * ks));
        cfg.blockDim = dim3((unsigned)(fp8 ? kFp8Threads : kThreads));
        cfg.dynamicSmemBytes = single_smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)ks;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        const cudaError_t e = fp8 ? (np == 2 ? cudaLaunchKernelEx(&cfg, in_proj_conv_kernel<true, 2>, p)
                                             : cudaLaunchKernelEx(&cfg, in_proj_conv_kernel<true>, p))
                                  : cudaLaunchKernelEx(&cfg, in_proj_conv_kernel<false>, p);
        return e == cudaSuccess ? launch_status() : GDN_ERR_LAUNCH;
    }
    if (use_pair) {
        const int grid = 2 * (int)(tiles < pairs ? tiles : pairs);
        if (fp8) {
            __half* w16 = reinterpret_cast<__half*>(static_cast<uint8_t*>(a.workspace) + fp8_w16_offset(a.T, a.K));
            const int64_t pieces = a.N * (a.K / 16);
            const int cgrid = (int)((pieces + 255) / 256 < 8 * nsm ? (pieces + 255) / 256 : 8 * nsm);
            codes_to_f16_kernel<<<cgrid, 256, 0, s>>>(static_cast<const uint8_t*>(a.codes), a.ldc, w16, a.N, (int)a.K);
            in_proj_conv_pair_kernel<true><<<grid, kThreads, kPairSmemBytes, s>>>(p);
        } else {
            in_proj_conv_pair_kernel<false><<<grid, kThreads, kPairSmemBytes, s>>>(p);
        }
    } else if (fp8) {
        const int grid = (int)(tiles < nsm ? tiles : nsm);
        in_proj_conv_kernel<true><<<grid, kFp8Threads, single_smem, s>>>(p);
    } else {
        const int grid = (int)(tiles < nsm ? tiles : nsm);
        in_proj_conv_kernel<false><<<grid, kThreads, single_smem, s>>>(p);
    }
    return launch_status();
}

}  // namespace gdn
