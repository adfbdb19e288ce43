// Decode attention over a KV cache on tcgen05 (decode_attention, model/model.py:354-361; the
// reference's CUDA kernel is model/triton_kernels.py:117-211): the drafter's mask-row queries over
// the delta layers' key cache (inference/engine.py:436-437, R = K(K-1) rows, G = 1, D = 128) and
// the attention layers' candidate + mask rows (G = 4, D = 256).
//
// o[b, r, h] = softmax_n(scale * q[b, r, h] . k[b, n, h / G] + mask[b, 0, r, n]) v[b, n, h / G]
// over keys n < L. One CTA per (batch row, key head, split of NK keys): the query rows of the key
// head (R * G <= 64, row rq = r * G + g, padded to 64), the split's keys and values are loaded
// whole with TMA (128-byte swizzle, 64-element d-panels), so the softmax of the split is exact
// (no running rescale):
//   S = Q K^T   two M=64 accumulators (keys 0..NK/2-1 at TMEM lane offset 0, the rest at +16),
//               so that each of the 4 warps reads 16 rows x 2 key halves;
//   P = exp2(S * scale * log2 e + mask * log2 e - m), m the row max over the split (0 when every
//       key of the row is masked), stored as bf16 (the operand of the next product), l = sum of
//       the fp32 values;
//   O = P V     one M=64 accumulator per 64-wide d-panel (panels 2j and 2j + 1 share columns at
//               lane offsets 0 and +16).
// With one split the CTA writes o = O / l in bf16 (0 for a row with every key masked); otherwise
// it writes O / l and lse = m + log2 l (or -inf) in fp32 and decode_attention_combine_kernel
// weights the splits by exp2(lse - max lse), as the reference's second kernel does.

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
    static constexpr int NK = D == 128 ? 128 : 64;                   // keys per split
    static constexpr int DP = D / 64;                                // d-panels
    static constexpr uint32_t Q = 0;                                 // DP panels of 64 rows
    static constexpr uint32_t QPanel = kRows * kPanelRow;            // 8 KB
    static constexpr uint32_t K = Q + DP * QPanel;                   // DP panels of NK rows
    static constexpr uint32_t KPanel = NK * kPanelRow;
    static constexpr uint32_t V = K + DP * KPanel;
    static constexpr uint32_t P = V + DP * KPanel;                   // NK / 64 panels of 64 rows
    static constexpr uint32_t END = P + (NK / 64) * QPanel;
    static constexpr uint32_t BYTES = END + 1024;                    // + alignment slack
    static constexpr uint32_t COL_S = 0;                             // NK / 2 columns
    static constexpr uint32_t COL_O = 64;                            // D / 2 columns
    static constexpr uint32_t TMEM_COLS = COL_O + D / 2 <= 128 ? 128 : 256;
    static_assert(NK % 64 == 0 && NK / 2 <= COL_O, "keys per split");
};

struct Params {
    CUtensorMap tm_q;  // 4-D (D, H, R, B), box (64, G, R, 1)
    CUtensorMap tm_k;  // 4-D (D, Hkv, Lc, Bc), box (64, 1, NK, 1)
    CUtensorMap tm_v;
    const bf16* mask;  // [B, 1, R, L] additive, element strides (smb, smr), keys contiguous
    int64_t smb, smr;
    bf16* o;           // [B, R, H, D] contiguous (one split)
    float* part_o;     // [B * Hkv * splits * 64, D] (several splits)
    float* part_lse;   // [B * Hkv * splits * 64]
    int R, G, Hkv, L, splits;
    float scale_log2e;
};

struct Shared {
    uint64_t tma, s_done, o_done;
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
    constexpr int NK = TL::NK, DP = TL::DP, NH = NK / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ Shared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int n0 = split * NK;
    const int rows = p.R * p.G;

    if (tid == 0) {
        mbar_init(&sh.tma, 1);
        mbar_init(&sh.s_done, 1);
        mbar_init(&sh.o_done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, TL::TMEM_COLS);
        tmem_relinquish();
    }
    // query rows past R * G: zeros (TMA writes rows 0 .. R * G - 1 of each panel)
    for (int i = rows * 8 + tid; i < kRows * 8; i += 128) {
#pragma unroll
        for (int dp = 0; dp < DP; ++dp)
            *reinterpret_cast<uint4*>(sm + TL::Q + dp * TL::QPanel + (i >> 3) * kPanelRow + ((i & 7) << 4)) =
                make_uint4(0, 0, 0, 0);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;

    if (tid == 0) {
        constexpr uint32_t kv_bytes = 2u * DP * NK * kPanelRow;
        mbar_arrive_expect_tx(&sh.tma, (uint32_t)(DP * rows) * kPanelRow + kv_bytes);
#pragma unroll
        for (int dp = 0; dp < DP; ++dp) {
            tma_load_4d(sm + TL::Q + dp * TL::QPanel, &p.tm_q, &sh.tma, 64 * dp, kvh * p.G, 0, b);
            tma_load_4d(sm + TL::K + dp * TL::KPanel, &p.tm_k, &sh.tma, 64 * dp, kvh, n0, b);
            tma_load_4d(sm + TL::V + dp * TL::KPanel, &p.tm_v, &sh.tma, 64 * dp, kvh, n0, b);
        }
    }
    bool ok = mbar_wait(&sh.tma, 0, kSiteTmaLoad);
    bool s_issued = false, o_issued = false;  // (thread 0) products to drain if a wait gives up
    if (tid == 0 && ok) {
        // S = Q K^T: keys 0 .. NH - 1 into lane offset 0, NH .. NK - 1 into lane offset 16
        tc_fence_after();
        const uint32_t id_s = make_idesc(kRows, NH, kFmtBF16, false, false);
        const uint64_t dq = sdesc_kmajor(sm + TL::Q, 0), dk = sdesc_kmajor(sm + TL::K, 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t qo = (kk >> 2) * TL::QPanel + (kk & 3) * 32;
            const uint32_t ko = (kk >> 2) * TL::KPanel + (kk & 3) * 32;
            mma_f16(tb + TL::COL_S, sdesc_add(dq, qo), sdesc_add(dk, ko), id_s, kk > 0);
            mma_f16(tb + TL::COL_S + (16u << 16), sdesc_add(dq, qo), sdesc_add(dk, ko + NH * kPanelRow), id_s, kk > 0);
        }
        mma_commit(&sh.s_done);
        s_issued = true;
    }
    // ---- softmax of this thread's row half: row i = 16 warp + lane % 16, keys of half lane / 16
    const int i = 16 * warp + (lane & 15), half = lane >> 4;
    const bool row_ok = i < rows;
    const int r = row_ok ? i / p.G : 0;
    ok = __all_sync(0xffffffffu, ok) && mbar_wait(&sh.s_done, 0, kSiteMma);
    float m = -INFINITY, l = 0.f;
    if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        float s[NH];
        if constexpr (NH == 64) {
            tmem_ld64_wait(tb + TL::COL_S + ((uint32_t)(32 * warp) << 16), s);
        } else {
            tmem_ld32_wait(tb + TL::COL_S + ((uint32_t)(32 * warp) << 16), s);
        }
        const int nb = n0 + half * NH;
        const bf16* mrow = p.mask + (int64_t)b * p.smb + (int64_t)r * p.smr + nb;
#pragma unroll
        for (int c = 0; c < NH / 8; ++c) {
            float mv[8];
            if (row_ok && nb + 8 * c + 8 <= p.L) {
                const uint4 raw = *reinterpret_cast<const uint4*>(mrow + 8 * c);
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(h2[e]);
                    mv[2 * e] = f.x;
                    mv[2 * e + 1] = f.y;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    mv[e] = (row_ok && nb + 8 * c + e < p.L) ? __bfloat162float(mrow[8 * c + e]) : -INFINITY;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float x = s[8 * c + e] * p.scale_log2e + mv[e] * kLog2e;
                s[8 * c + e] = x;
                m = fmaxf(m, x);
            }
        }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        const float shift = m == -INFINITY ? 0.f : m;  // a row with every key masked keeps p = 0
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            s[j] = exp2f(s[j] - shift);
            l += s[j];
        }
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        // P (bf16) as the K-major A operand of O = P V: panel of keys (64 per panel), row i
        uint8_t* ppanel = sm + TL::P + (half * NH / 64) * TL::QPanel;
        const int chunk0 = (half * NH % 64) / 8;
#pragma unroll
        for (int c = 0; c < NH / 8; ++c) put_chunk8(ppanel, i, chunk0 + c, s + 8 * c);
    }
    fence_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    if (tid == 0 && ok) {
        // O = P V: d-panel dp into columns COL_O + 64 (dp / 2), lane offset 16 (dp % 2)
        tc_fence_after();
        const uint32_t id_o = make_idesc(kRows, 64, kFmtBF16, false, true);
        const uint64_t dpn = sdesc_kmajor(sm + TL::P, 0);
#pragma unroll
        for (int dp = 0; dp < DP; ++dp) {
            const uint64_t dv = sdesc_mnmajor(sm + TL::V + dp * TL::KPanel, TL::KPanel);
            const uint32_t dst = tb + TL::COL_O + 64 * (dp >> 1) + ((uint32_t)(16 * (dp & 1)) << 16);
#pragma unroll
            for (int kk = 0; kk < NK / 16; ++kk)
                mma_f16(dst, sdesc_add(dpn, (kk >> 2) * TL::QPanel + (kk & 3) * 32), sdesc_add(dv, kk * 2048), id_o,
                        kk > 0);
        }
        mma_commit(&sh.o_done);
        o_issued = true;
    }
    ok = ok && mbar_wait(&sh.o_done, 0, kSiteMma);
    if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const float lse = l > 0.f ? m + log2f(l) : -INFINITY;
        const int g = row_ok ? i % p.G : 0;
#pragma unroll
        for (int j = 0; j < DP / 2; ++j) {
            float o[64];
            tmem_ld64_wait(tb + TL::COL_O + 64 * j + ((uint32_t)(32 * warp) << 16), o);
            const int d0 = 64 * (2 * j + half);  // this thread's d-panel
            if (!row_ok) continue;
            if (p.splits == 1) {
                bf16* dst = p.o + (((int64_t)b * p.R + r) * (p.Hkv * p.G) + kvh * p.G + g) * D + d0;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint4 raw;
                    __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        h2[e] = __floats2bfloat162_rn(o[8 * c + 2 * e] * inv, o[8 * c + 2 * e + 1] * inv);
                    *reinterpret_cast<uint4*>(dst + 8 * c) = raw;
                }
            } else {
                const int64_t slot = (((int64_t)b * p.Hkv + kvh) * p.splits + split) * kRows + i;
                float* dst = p.part_o + slot * D + d0;
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    *reinterpret_cast<float4*>(dst + 4 * c) =
                        make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
                if (j == 0 && half == 0) p.part_lse[slot] = lse;
            }
        }
    }
    if (tid == 0) {  // after a failed wait: the copies and products in flight finish before TMEM is freed
        mbar_wait(&sh.tma, 0, kSiteDrain);
        if (s_issued) mbar_wait(&sh.s_done, 0, kSiteDrain);
        if (o_issued) mbar_wait(&sh.o_done, 0, kSiteDrain);
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

static int keys_per_split(int64_t D) { return D == 128 ? Tile<128>::NK : Tile<256>::NK; }

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
    if (!make_map4(&p.tm_q, a.q, D, a.H, a.R, a.B, a.qsh, a.qsr, a.qsb, (uint32_t)G, (uint32_t)a.R) ||
        !make_map4(&p.tm_k, a.k, D, a.Hkv, a.cache_len, a.cache_rows, a.ksh, a.kss, a.ksb, 1, Tile<D>::NK) ||
        !make_map4(&p.tm_v, a.v, D, a.Hkv, a.cache_len, a.cache_rows, a.vsh, a.vss, a.vsb, 1, Tile<D>::NK))
        return GDN_ERR_LAUNCH;
    p.mask = static_cast<const bf16*>(a.mask);
    p.smb = a.msb;
    p.smr = a.msr;
    p.o = static_cast<bf16*>(a.o);
    p.R = (int)a.R;
    p.G = G;
    p.Hkv = (int)a.Hkv;
    p.L = (int)a.L;
    p.splits = (int)((a.L + Tile<D>::NK - 1) / Tile<D>::NK);
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
    const int64_t nk = attn::keys_per_split(D);
    const int64_t splits = (L + nk - 1) / nk;
    if (splits <= 1 || B <= 0 || Hkv <= 0) return 0;
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
