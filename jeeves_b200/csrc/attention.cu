// Decode attention over a KV cache on tcgen05 (decode_attention, model/model.py:354-361; the
// reference's CUDA kernel is model/triton_kernels.py:117-211): the drafter's mask-row queries over
// the delta layers' key cache (inference/engine.py:436-437, R = K(K-1) rows, G = 1, D = 128) and
// the attention layers' candidate + mask rows (G = 4, D = 256).
//
// o[b, r, h] = softmax_n(scale * q[b, r, h] . k[b, n, h / G] + mask[b, 0, r, n]) v[b, n, h / G]
// over keys n < L. One CTA per (batch row, key head, range of key blocks); with at least as many
// (batch row, key head) pairs as SMs there is one range, else the keys are split so that every SM
// gets work. The query rows of the key head (R * G <= 64, row rq = r * G + g, padded to 64) stay in
// shared memory; key blocks of NK keys stream through two K / V stages with TMA (128-byte swizzle,
// 64-element d-panels), block j + 2 loading while block j + 1 is computed:
//   S = Q K^T   two M=64 accumulators (keys 0..NK/2-1 at TMEM lane offset 0, the rest at +16),
//               so that each of the 4 warps reads 16 rows x 2 key halves;
//   online softmax per row: m' = max(m, max_n s), p = exp2(s - m') with s = S scale log2 e +
//       mask log2 e (m' = -inf shifts by 0 so that p = 0), alpha = exp2(m - m'), l' = l alpha +
//       sum p; p goes to shared memory in bf16 as the operand of the next product;
//   O_blk = P V one M=64 accumulator per 64-wide d-panel (panels 2j and 2j + 1 share columns at
//               lane offsets 0 and +16); each thread keeps its row's O = O alpha + O_blk in
//               registers.
// With one range the CTA writes o = O / l in bf16 (0 for a row with every key masked); otherwise
// it writes O / l and lse = m + log2 l (or -inf) in fp32 and decode_attention_combine_kernel
// weights the ranges by exp2(lse - max lse), as the reference's second kernel does.

#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"
#include "tensor_map.h"

namespace gdn {
namespace attn {

using namespace sm100;

constexpr int kRows = 64;                        // query rows per CTA (the MMA's M)
constexpr uint32_t kPanelRow = 128;              // bytes per 64-element bf16 panel row
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Tile {
    static constexpr int NK = 64;                                    // keys per block
    static constexpr int DP = D / 64;                                // d-panels
    static constexpr uint32_t Q = 0;                                 // DP panels of 64 rows
    static constexpr uint32_t QPanel = kRows * kPanelRow;            // 8 KB
    static constexpr uint32_t KPanel = NK * kPanelRow;
    static constexpr uint32_t KV = Q + DP * QPanel;                  // two stages of K then V panels
    static constexpr uint32_t Stage = 2 * DP * KPanel;               // 64 KB
    static constexpr uint32_t P = KV + 2 * Stage;                    // NK / 64 panels of 64 rows
    static constexpr uint32_t END = P + (NK / 64) * QPanel;
    static constexpr uint32_t BYTES = END + 1024;                    // + alignment slack
    static constexpr uint32_t COL_S = 0;                             // NK columns
    static constexpr uint32_t COL_O = 64;                            // 128 columns
    static constexpr uint32_t TMEM_COLS = 256;
    static_assert(NK == 64 && NK <= COL_O, "keys per block");
    static_assert(D != 128 || 2 * BYTES <= 227 * 1024, "two CTAs per SM at D = 128");
};

struct Params {
    CUtensorMap tm_q;  // 4-D (D, H, R, B), box (64, G, R, 1)
    CUtensorMap tm_k;  // 4-D (D, Hkv, Lc, Bc), box (64, 1, NK, 1)
    CUtensorMap tm_v;
    const bf16* mask;  // [B, 1, R, L] additive, element strides (smb, smr), keys contiguous
    int64_t smb, smr;
    bf16* o;           // [B, R, H, D] contiguous (one range)
    float* part_o;     // [B * Hkv * splits * 64, D] (several ranges)
    float* part_lse;   // [B * Hkv * splits * 64]
    int R, G, Hkv, L, splits, blocks_per_split;
    float scale_log2e;
};

struct Shared {
    uint64_t qbar, full[2], s_done, o_done;
    uint32_t tmem_base;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// 8 fp32 values -> one 16-byte bf16 chunk of row `row` of a 128-byte-swizzled panel.
__device__ __forceinline__ void put_chunk8(uint8_t* panel, uint32_t row, uint32_t chunk, const float* v) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(panel + sw128(row, chunk)) = raw;
}

template <int D>
__global__ void __launch_bounds__(128) decode_attention_kernel(const __grid_constant__ Params p) {
    using TL = Tile<D>;
    constexpr int NK = TL::NK, DP = TL::DP;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ Shared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int rows = p.R * p.G;
    const int blocks_total = (p.L + NK - 1) / NK;
    const int j0 = split * p.blocks_per_split;
    const int nb = min(p.blocks_per_split, blocks_total - j0);  // key blocks of this CTA (>= 1)

    if (tid == 0) {
        mbar_init(&sh.qbar, 1);
        mbar_init(&sh.full[0], 1);
        mbar_init(&sh.full[1], 1);
        mbar_init(&sh.s_done, 1);
        mbar_init(&sh.o_done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, TL::TMEM_COLS);
        tmem_relinquish();
    }
    // query rows past R * G: zeros (TMA writes rows 0 .. R * G - 1 of each panel)
    for (int c = rows * 8 + tid; c < kRows * 8; c += 128) {
#pragma unroll
        for (int dp = 0; dp < DP; ++dp)
            *reinterpret_cast<uint4*>(sm + TL::Q + dp * TL::QPanel + (c >> 3) * kPanelRow + ((c & 7) << 4)) =
                make_uint4(0, 0, 0, 0);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;

    auto load_block = [&](int j) {  // thread 0: keys and values of block j0 + j into stage j & 1
        uint8_t* st = sm + TL::KV + (j & 1) * TL::Stage;
        const int n0 = (j0 + j) * NK;
        mbar_arrive_expect_tx(&sh.full[j & 1], TL::Stage);
#pragma unroll
        for (int dp = 0; dp < DP; ++dp) {
            tma_load_4d(st + dp * TL::KPanel, &p.tm_k, &sh.full[j & 1], 64 * dp, kvh, n0, b);
            tma_load_4d(st + (DP + dp) * TL::KPanel, &p.tm_v, &sh.full[j & 1], 64 * dp, kvh, n0, b);
        }
    };
    // the thread that issues the copies and the products: with at most 16 query rows warps 1-3
    // hold no rows (see warp_live below), so a lane of warp 1 takes the role and warp 0, the only
    // one with softmax work, never waits for an issue
    const int issuer = rows <= 16 ? 32 : 0;
    int loaded = 0;  // (issuer) blocks whose copies were issued
    if (tid == issuer) {
        mbar_arrive_expect_tx(&sh.qbar, (uint32_t)(DP * rows) * kPanelRow);
#pragma unroll
        for (int dp = 0; dp < DP; ++dp)
            tma_load_4d(sm + TL::Q + dp * TL::QPanel, &p.tm_q, &sh.qbar, 64 * dp, kvh * p.G, 0, b);
        for (; loaded < 2 && loaded < nb; ++loaded) load_block(loaded);
    }

    // S (M=64, N=64) and O (M=64, N=128: d 0..127 at lane offset 0, d 128..255 at +16): row i of
    // an M=64 accumulator sits in lane i % 16 of quarter i / 16, so lanes 0-15 of each warp hold
    // the softmax rows, and at D = 256 lanes 16-31 hold the second half of O.
    // S as two M = 64, N = 32 products: keys 0-31 at TMEM lane offset 0, keys 32-63 at +16, so
    // that lanes l and l + 16 of a warp hold the two key halves of row i and split its softmax
    const uint32_t id_s = make_idesc(kRows, NK / 2, kFmtBF16, false, false);
    const int kh = lane >> 4;                       // this lane's key half of row i
    const uint32_t id_o = make_idesc(kRows, 128, kFmtBF16, false, true);
    const int i = 16 * warp + (lane & 15);
    const bool owner = lane < 16;                   // holds row i of S
    const bool row_ok = i < rows;
    const bool holds_o = D == 256 || owner;         // holds 128 values of O
    // A warp whose 16 rows all lie past R * G (the padding of the MMA's M = 64) skips the softmax,
    // the P rows and the O update: those rows only feed O rows that are never stored, and the
    // skipped work would take issue slots from the other CTA on the SM (the drafter's 12 mask rows
    // leave warps 1-3 idle).
    const bool warp_live = 16 * warp < rows;
    const int r = row_ok ? i / p.G : 0;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const bf16* mrow = p.mask + (int64_t)b * p.smb + (int64_t)r * p.smr;
    float m = -INFINITY, l = 0.f;  // the row's running max and sum, the same in both key-half lanes
    float acc[128];
#pragma unroll
    for (int e = 0; e < 128; ++e) acc[e] = 0.f;
    bool ok = mbar_wait(&sh.qbar, 0, kSiteTmaLoad);
    int s_issued = 0, o_issued = 0;  // (issuer) products issued, for the drain after a failed wait

    for (int j = 0; j < nb && __syncthreads_and(ok); ++j) {
        const int st = j & 1;
        const uint8_t* stage = sm + TL::KV + st * TL::Stage;
        const int n0 = (j0 + j) * NK;
        if (tid == issuer) {
            ok = mbar_wait(&sh.full[st], (uint32_t)(j >> 1) & 1, kSiteTmaLoad);
            if (ok) {  // S = Q K^T
                tc_fence_after();
                const uint64_t dq = sdesc_kmajor(sm + TL::Q, 0), dk = sdesc_kmajor(stage, 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t a = sdesc_add(dq, (kk >> 2) * TL::QPanel + (kk & 3) * 32);
                    const uint32_t kb = (kk >> 2) * TL::KPanel + (kk & 3) * 32;
                    mma_f16(tb + TL::COL_S, a, sdesc_add(dk, kb), id_s, kk > 0);
                    mma_f16(tb + TL::COL_S + (16u << 16), a, sdesc_add(dk, kb + (NK / 2) * kPanelRow), id_s, kk > 0);
                }
                mma_commit(&sh.s_done);
                ++s_issued;
            }
        }
        // the mask of this row's keys (bf16, kept packed), loaded while the product runs; keys past L
        // and rows past R * G read as -inf
        uint4 mraw[NK / 16];
        const bool live = row_ok;
#pragma unroll
        for (int c = 0; c < NK / 16; ++c) {
            const int n = n0 + (NK / 2) * kh + 8 * c;
            if (live && n + 8 <= p.L) {
                mraw[c] = *reinterpret_cast<const uint4*>(mrow + n);
            } else {
                __nv_bfloat162 h2[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const bf16 lo = (live && n + 2 * e < p.L) ? mrow[n + 2 * e] : __float2bfloat16_rn(-INFINITY);
                    const bf16 hi = (live && n + 2 * e + 1 < p.L) ? mrow[n + 2 * e + 1] : __float2bfloat16_rn(-INFINITY);
                    h2[e] = __halves2bfloat162(lo, hi);
                }
                mraw[c] = *reinterpret_cast<const uint4*>(h2);
            }
        }
        ok = __syncthreads_and(ok) && mbar_wait(&sh.s_done, (uint32_t)j & 1, kSiteMma);
        if (!__syncthreads_and(ok)) break;
        tc_fence_after();
        float sv[NK / 2];
        float alpha = 0.f;
        if (warp_live) {  // warp-uniform: both halves of every row, combined with shuffles
            tmem_ld32_wait(tb + TL::COL_S + lane_base, sv);
            float mb = -INFINITY;
#pragma unroll
            for (int c = 0; c < NK / 16; ++c) {
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&mraw[c]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(h2[e]);
                    const int k0 = 8 * c + 2 * e;
                    sv[k0] = sv[k0] * p.scale_log2e + f.x * kLog2e;
                    sv[k0 + 1] = sv[k0 + 1] * p.scale_log2e + f.y * kLog2e;
                    mb = fmaxf(mb, fmaxf(sv[k0], sv[k0 + 1]));
                }
            }
            mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 16));
            const float m_new = fmaxf(m, mb);
            const float shift = m_new == -INFINITY ? 0.f : m_new;  // a row with every key masked keeps p = 0
            alpha = exp2f(m - shift);
            float ls = 0.f;
#pragma unroll
            for (int e = 0; e < NK / 2; ++e) {
                sv[e] = exp2f(sv[e] - shift);
                ls += sv[e];
            }
            ls += __shfl_xor_sync(0xffffffffu, ls, 16);
            l = l * alpha + ls;
            m = m_new;
            // P (bf16) as the K-major A operand of O_blk = P V: one 64-key panel, row i, this half
#pragma unroll
            for (int c = 0; c < NK / 16; ++c) put_chunk8(sm + TL::P, i, (NK / 16) * kh + c, sv + 8 * c);
        }
        alpha = __shfl_sync(0xffffffffu, alpha, lane & 15);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == issuer) {  // O_blk = P V
            tc_fence_after();
            const uint64_t dpn = sdesc_kmajor(sm + TL::P, 0);
#pragma unroll
            for (int h = 0; h < DP / 2; ++h) {  // d 128 h .. 128 h + 127 (two V panels)
                const uint64_t dv = sdesc_mnmajor(stage + (DP + 2 * h) * TL::KPanel, TL::KPanel);
                const uint32_t dst = tb + TL::COL_O + ((uint32_t)(16 * h) << 16);
#pragma unroll
                for (int kk = 0; kk < NK / 16; ++kk)
                    mma_f16(dst, sdesc_add(dpn, kk * 32), sdesc_add(dv, kk * 2048), id_o, kk > 0);
            }
            mma_commit(&sh.o_done);
            ++o_issued;
        }
        ok = mbar_wait(&sh.o_done, (uint32_t)j & 1, kSiteMma);
        if (!__all_sync(0xffffffffu, ok)) continue;  // the loop condition ends every thread together
        tc_fence_after();
        // the stage is free again: block j + 2 streams in while block j + 1 is computed
        if (tid == issuer && loaded < nb) load_block(loaded++);
#pragma unroll
        for (int c = 0; c < 2 && warp_live; ++c) {
            float ob[64];
            tmem_ld64_wait(tb + TL::COL_O + 64 * c + lane_base, ob);
#pragma unroll
            for (int e = 0; e < 64; ++e) acc[64 * c + e] = acc[64 * c + e] * alpha + ob[e];
        }
        tc_fence_before();
    }
    ok = __syncthreads_and(ok);

    l = __shfl_sync(0xffffffffu, l, lane & 15);
    m = __shfl_sync(0xffffffffu, m, lane & 15);
    if (ok && row_ok && holds_o) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int g = i % p.G;
        const int d0 = owner ? 0 : 128;  // this thread's 128 values of O
        if (p.splits == 1) {
            bf16* dst = p.o + (((int64_t)b * p.R + r) * (p.Hkv * p.G) + kvh * p.G + g) * D + d0;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                uint4 raw;
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    h2[e] = __floats2bfloat162_rn(acc[8 * c + 2 * e] * inv, acc[8 * c + 2 * e + 1] * inv);
                *reinterpret_cast<uint4*>(dst + 8 * c) = raw;
            }
        } else {
            const int64_t slot = (((int64_t)b * p.Hkv + kvh) * p.splits + split) * kRows + i;
            float* dst = p.part_o + slot * D + d0;
#pragma unroll
            for (int c = 0; c < 32; ++c)
                *reinterpret_cast<float4*>(dst + 4 * c) =
                    make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv, acc[4 * c + 3] * inv);
            if (owner) p.part_lse[slot] = l > 0.f ? m + log2f(l) : -INFINITY;
        }
    }
    if (tid == issuer) {  // after a failed wait: the copies and products in flight finish before TMEM is freed
        mbar_wait(&sh.qbar, 0, kSiteDrain);
        for (int j = loaded - 2 < 0 ? 0 : loaded - 2; j < loaded; ++j)
            mbar_wait(&sh.full[j & 1], (uint32_t)(j >> 1) & 1, kSiteDrain);
        if (s_issued) mbar_wait(&sh.s_done, (uint32_t)(s_issued - 1) & 1, kSiteDrain);
        if (o_issued) mbar_wait(&sh.o_done, (uint32_t)(o_issued - 1) & 1, kSiteDrain);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tb, TL::TMEM_COLS);
}

}  // namespace attn
}  // namespace gdn

namespace gdn {
namespace attn {

// The splits of one query row weighted by exp2(lse - max lse); zeros for a row that saw no key.
// One CTA of D threads per (batch row x key head, query row).
template <int D>
__global__ void decode_attention_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                                bf16* __restrict__ o, int splits, int R, int G, int Hkv) {
    const int bh = blockIdx.x, i = blockIdx.y, d = threadIdx.x;
    const int64_t first = (int64_t)bh * splits * kRows + i;
    float top = -INFINITY;
    for (int s = 0; s < splits; ++s) top = fmaxf(top, part_lse[first + (int64_t)s * kRows]);
    const float base = top == -INFINITY ? 0.f : top;
    float acc = 0.f, total = 0.f;
    for (int s = 0; s < splits; ++s) {
        const int64_t slot = first + (int64_t)s * kRows;
        const float w = exp2f(part_lse[slot] - base);
        total += w;
        acc += w * part_o[slot * D + d];
    }
    const int b = bh / Hkv, kvh = bh % Hkv, r = i / G, g = i % G;
    o[(((int64_t)b * R + r) * (Hkv * G) + kvh * G + g) * D + d] = __float2bfloat16_rn(acc / (total > 0.f ? total : 1.f));
}

// 4-D map over a [n3, n2, n1, D] bf16 tensor with element strides (s3, s2, s1), box (64, b1, b2, 1).
static bool make_map4(CUtensorMap* map, const void* base, int64_t D, int64_t n1, int64_t n2, int64_t n3, int64_t s1,
                      int64_t s2, int64_t s3, uint32_t b1, uint32_t b2) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n1, (cuuint64_t)n2, (cuuint64_t)n3};
    cuuint64_t strides[3] = {(cuuint64_t)s1 * 2, (cuuint64_t)s2 * 2, (cuuint64_t)s3 * 2};
    cuuint32_t box[4] = {64, b1, b2, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int keys_per_block(int64_t D) { return D == 128 ? Tile<128>::NK : Tile<256>::NK; }

static int sm_count() {
    static int sms[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (sms[dev] == 0 && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        sms[dev] = 0;
    return sms[dev];
}

// Key blocks per CTA and the number of ranges: one range per (batch row, key head) when those
// pairs fill the SMs; otherwise each pair's blocks are split so that the CTAs cover every SM.
struct Ranges {
    int64_t per, splits;
};
static Ranges key_ranges(int64_t B, int64_t Hkv, int64_t L, int64_t D) {
    const int64_t nk = keys_per_block(D);
    const int64_t blocks = (L + nk - 1) / nk;
    const int64_t pairs = B * Hkv, sms = sm_count();
    Ranges rg{blocks, 1};
    if (blocks > 0 && pairs > 0 && pairs < sms) {
        const int64_t want = (sms + pairs - 1) / pairs;
        rg.per = (blocks + want - 1) / want;
        rg.splits = (blocks + rg.per - 1) / rg.per;
    }
    return rg;
}

template <int D>
static int launch(const AttentionArgs& a, cudaStream_t s) {
    static bool ready[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_LAUNCH;
    if (!ready[dev]) {
        if (cudaFuncSetAttribute(decode_attention_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Tile<D>::BYTES) != cudaSuccess)
            return GDN_ERR_LAUNCH;
        ready[dev] = true;
    }
    const int G = (int)(a.H / a.Hkv);
    Params p;
    memset(&p, 0, sizeof(p));
    // The key maps end at L, not at the cache's length: the last block's keys past L arrive as
    // zeros (as the reference's masked loads give them), so stale cache slots holding Inf or NaN
    // never reach S or the P V product.
    if (!make_map4(&p.tm_q, a.q, D, a.H, a.R, a.B, a.qsh, a.qsr, a.qsb, (uint32_t)G, (uint32_t)a.R) ||
        !make_map4(&p.tm_k, a.k, D, a.Hkv, a.L, a.cache_rows, a.ksh, a.kss, a.ksb, 1, Tile<D>::NK) ||
        !make_map4(&p.tm_v, a.v, D, a.Hkv, a.L, a.cache_rows, a.vsh, a.vss, a.vsb, 1, Tile<D>::NK))
        return GDN_ERR_LAUNCH;
    p.mask = static_cast<const bf16*>(a.mask);
    p.smb = a.msb;
    p.smr = a.msr;
    p.o = static_cast<bf16*>(a.o);
    p.R = (int)a.R;
    p.G = G;
    p.Hkv = (int)a.Hkv;
    p.L = (int)a.L;
    const Ranges rg = key_ranges(a.B, a.Hkv, a.L, D);
    p.splits = (int)rg.splits;
    p.blocks_per_split = (int)rg.per;
    p.scale_log2e = a.scale * kLog2e;
    if (p.splits > 1) {
        const int64_t slots = a.B * a.Hkv * p.splits * kRows;
        p.part_o = static_cast<float*>(a.workspace);
        p.part_lse = p.part_o + slots * D;
    }
    dim3 grid((unsigned)p.splits, (unsigned)a.Hkv, (unsigned)a.B);
    decode_attention_kernel<D><<<grid, 128, Tile<D>::BYTES, s>>>(p);
    int st = launch_status();
    if (st != GDN_OK || p.splits == 1) return st;
    dim3 cgrid((unsigned)(a.B * a.Hkv), (unsigned)(a.R * G));
    decode_attention_combine_kernel<D><<<cgrid, D, 0, s>>>(p.part_o, p.part_lse, p.o, p.splits, p.R, G, p.Hkv);
    return launch_status();
}

}  // namespace attn

size_t decode_attention_workspace_bytes(int64_t B, int64_t Hkv, int64_t L, int64_t D) {
    if (B <= 0 || Hkv <= 0 || L <= 0) return 0;
    const int64_t splits = attn::key_ranges(B, Hkv, L, D).splits;
    if (splits <= 1) return 0;
    const int64_t slots = B * Hkv * splits * attn::kRows;
    return (size_t)slots * (size_t)(D + 1) * sizeof(float);
}

int launch_decode_attention(const AttentionArgs& a, cudaStream_t s) {
    if (a.B == 0) return GDN_OK;
    if (a.L == 0) {  // no keys: zeros, as the reference returns
        const size_t bytes = (size_t)a.B * a.R * a.H * a.D * sizeof(bf16);
        return cudaMemsetAsync(a.o, 0, bytes, s) == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
    }
    if (a.workspace_bytes < decode_attention_workspace_bytes(a.B, a.Hkv, a.L, a.D) ||
        (decode_attention_workspace_bytes(a.B, a.Hkv, a.L, a.D) > 0 && a.workspace == nullptr))
        return GDN_ERR_WORKSPACE;
    return a.D == 128 ? attn::launch<128>(a, s) : attn::launch<256>(a, s);
}

}  // namespace gdn
