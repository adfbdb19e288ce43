// The gated-delta layer's merged input projection with the causal conv fused into the GEMM's
// epilogue (tcgen05). The prefill branch of GatedDeltaNet.forward computes qkv = in_proj_qkv(x)
// and, beside it, z, b and a (model/model.py:458-461; the engine merges the projections,
// inference/engine.py:154-166, :374-375), then qkv = silu(causal_conv1d(qkv)) (:478-479). Here
// one call computes Y = X W^T for the merged weight W = [W_qkv; W_rest] ([N, K], nn.Linear
// layout) and writes
//   out[t, c] = silu(conv_c(Y_bf16[t-3..t, c]))   for c < C (the qkv channels),
//   out[t, c] = Y_bf16[t, c]                       for c >= C,
// with Y rounded to bf16 first, as the two eager steps do, and the conv / SiLU in the rounding of
// the conv kernel (fp32 sum of fp32 products in tap order, rounded to bf16, exact SiLU). With
// cu_seqlens the window restarts at every sequence. Optionally the last `taps` pre-conv rows of
// each sequence go to conv_tail [nseq, C, taps] (the conv state the cache keeps,
// model/model.py:468-469).
//
// Tiles: 128 GEMM rows x 256 channels. A tile's 128 rows are tokens t0 - 3 .. t0 + 124 (the three
// before t0 recomputed for the conv window; TMA fills rows before 0 and past T with zeros), so it
// writes the 125 rows t0 .. t0 + 124. Warp 4 streams 64-wide K slices of X and W through four
// stages with TMA (128-byte swizzle); thread 160 issues tcgen05.mma (M = 128, N = 256, K = 16) into
// a 256-column fp32 accumulator in TMEM and frees each stage with a commit; warps 0-3 read the
// accumulator (one row per thread), round to bf16 into a shared-memory tile and compute the conv
// from it.

#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"
#include "tensor_map.h"

namespace gdn {
namespace inproj {

using namespace sm100;

constexpr int kBM = 128;                 // GEMM rows per tile
constexpr int kHalo = 3;                 // rows before the tile's outputs (taps - 1 of a 4-tap conv)
constexpr int kOutRows = kBM - kHalo;    // 125 output rows per tile
constexpr int kBN = 256;                 // channels per tile
constexpr int kBK = 64;                  // K per stage (one 128-byte swizzle panel)
constexpr int kStages = 4;
constexpr uint32_t kAStage = kBM * 128;  // 16 KB
constexpr uint32_t kBStage = kBN * 128;  // 32 KB
constexpr uint32_t kStageBytes = kAStage + kBStage;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024;
constexpr uint32_t kTileRowBytes = kBN * 2;  // the bf16 tile row in the epilogue (reuses the stages)
constexpr int kThreads = 192;            // warps 0-3 epilogue, 4 producer, 5 MMA issuer
constexpr uint32_t kBarEpilogue = 1;
static_assert(kBM * kTileRowBytes <= kStages * kStageBytes, "the epilogue tile fits in the stages");

struct Params {
    CUtensorMap tm_x;  // 2-D (K, T), box (64, 128)
    CUtensorMap tm_w;  // 2-D (K, N), box (64, 256)
    const bf16* conv_w;  // [C, taps]
    const int32_t* cu_seqlens;  // [nseq + 1] or null (one sequence of T tokens)
    bf16* out;           // [T, N], row stride ldo
    bf16* conv_tail;     // [nseq, C, taps] or null
    int64_t ldo;
    int T, N, C, K, nseq;
};

struct Shared {
    uint64_t full[kStages], empty[kStages], acc_full;
    uint32_t tmem_base;
    int seq_start[kBM];  // first token of the sequence of each tile row (a packed batch)
    int seq_end[kBM];
    int seq_id[kBM];
    int abort;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// 16-byte chunk j (0..31) of tile row r in the epilogue tile: chunks XOR-swizzled by the row, so
// that the 32 lanes writing one column chunk of 32 rows hit distinct banks.
__device__ __forceinline__ uint32_t tile_off(int r, int j) { return r * kTileRowBytes + (((j ^ r) & 31) << 4); }

}  // namespace inproj
}  // namespace gdn

namespace gdn {
namespace inproj {

__global__ void __launch_bounds__(kThreads, 1) in_proj_conv_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ Shared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kOutRows;  // first output token of the tile
    const int row0 = t0 - kHalo;           // token of GEMM row 0
    const int n0 = blockIdx.y * kBN;
    const int kblocks = p.K / kBK;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 1);
        }
        mbar_init(&sh.acc_full, 1);
        sh.abort = 0;
        fence_mbar_init();
        tma_prefetch_map(&p.tm_x);
        tma_prefetch_map(&p.tm_w);
    }
    if (warp == 0) {
        tmem_alloc(&sh.tmem_base, kBN);
        tmem_relinquish();
    }
    if (tid < kBM) {  // the sequence of each tile row's token
        const int t = row0 + tid;
        int s0 = 0, s1 = p.T, id = 0;
        if (p.cu_seqlens && t >= 0 && t < p.T) {
            int lo = 0, hi = p.nseq - 1;  // the last sequence that starts at or before t
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (p.cu_seqlens[mid] <= t) lo = mid;
                else hi = mid - 1;
            }
            id = lo;
            s0 = p.cu_seqlens[lo];
            s1 = p.cu_seqlens[lo + 1];
        }
        sh.seq_start[tid] = s0;
        sh.seq_end[tid] = s1;
        sh.seq_id[tid] = id;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = sh.tmem_base;

    if (warp == 4) {
        // ============================== producer ==============================
        if (lane != 0) return;
        int issued = 0;
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % kStages;
            if (kb >= kStages &&
                !mbar_wait_or_abort(&sh.empty[s], (uint32_t)((kb / kStages) - 1) & 1, kSiteTmaLoad, &sh.abort)) {
                atomicExch(&sh.abort, 1);
                break;
            }
            uint8_t* st = sm + s * kStageBytes;
            mbar_arrive_expect_tx(&sh.full[s], kStageBytes);
            tma_load_2d(st, &p.tm_x, &sh.full[s], kb * kBK, row0);
            tma_load_2d(st + kAStage, &p.tm_w, &sh.full[s], kb * kBK, n0);
            ++issued;
        }
        // the copies in flight land before the CTA's shared memory can go away
        for (int kb = issued - kStages > 0 ? issued - kStages : 0; kb < issued; ++kb)
            mbar_wait(&sh.full[kb % kStages], (uint32_t)(kb / kStages) & 1, kSiteDrain);
        return;
    }
    if (warp == 5) {
        // ============================== MMA issuer ==============================
        if (lane != 0) return;
        const uint32_t idesc = make_idesc(kBM, kBN, kFmtBF16, false, false);
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % kStages;
            if (!mbar_wait_or_abort(&sh.full[s], (uint32_t)(kb / kStages) & 1, kSiteTmaLoad, &sh.abort)) {
                atomicExch(&sh.abort, 1);
                break;
            }
            tc_fence_after();
            const uint8_t* st = sm + s * kStageBytes;
            const uint64_t da = sdesc_kmajor(st, 0), db = sdesc_kmajor(st + kAStage, 0);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
                mma_f16(tb, sdesc_add(da, kk * 32), sdesc_add(db, kk * 32), idesc, (kb | kk) != 0 ? 1u : 0u);
            mma_commit(&sh.empty[s]);  // the stage is free once these products have read it
        }
        mma_commit(&sh.acc_full);  // after every product issued (also after a failed wait)
        return;
    }

    // ================================ epilogue ================================
    const int r = 32 * warp + lane;  // tile row = TMEM lane
    const bool ok = mbar_wait(&sh.acc_full, 0, kSiteMma) && !*reinterpret_cast<volatile int*>(&sh.abort);
    tc_fence_after();
    // every product is done, so the stages are free: the bf16 tile goes there
    uint8_t* tile = sm;
#pragma unroll 1
    for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld32_wait(tb + ((uint32_t)(32 * warp) << 16) + 32 * c, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 raw;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
            *reinterpret_cast<uint4*>(tile + tile_off(r, 4 * c + q)) = raw;
        }
    }
    tc_fence_before();
    named_sync(kBarEpilogue, kBM);
    if (ok) {
        for (int task = tid; task < kOutRows * (kBN / 8); task += kBM) {
            const int rr = kHalo + task / (kBN / 8), j = task % (kBN / 8);
            const int t = row0 + rr;
            const int c = n0 + 8 * j;
            if (t >= p.T || c >= p.N) continue;
            const uint4 cur = *reinterpret_cast<const uint4*>(tile + tile_off(rr, j));
            uint4 res = cur;
            if (c < p.C) {
                float win[4][8];
                const int start = sh.seq_start[rr];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (t - 3 + i >= start) {
                        const uint4 raw = *reinterpret_cast<const uint4*>(tile + tile_off(rr - 3 + i, j));
                        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __bfloat1622float2(h[e]);
                            win[i][2 * e] = f.x;
                            win[i][2 * e + 1] = f.y;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) win[i][e] = 0.f;
                    }
                }
                bf16 wr[32];
                const uint4* wsrc = reinterpret_cast<const uint4*>(p.conv_w + (int64_t)c * 4);
#pragma unroll
                for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(wr)[i] = __ldg(wsrc + i);
                float pre[8], out[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc = __fadd_rn(acc, __fmul_rn(to_f32(wr[4 * q + i]), win[i][q]));
                    pre[q] = round_bf16(acc);
                }
                silu8(pre, out);
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&res);
#pragma unroll
                for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(out[2 * e], out[2 * e + 1]);
                if (p.conv_tail && t >= sh.seq_end[rr] - 4) {  // the pre-conv rows the cache keeps
                    const int pos = 4 - (sh.seq_end[rr] - t);
                    const bf16* cv = reinterpret_cast<const bf16*>(&cur);
                    bf16* dst = p.conv_tail + ((int64_t)sh.seq_id[rr] * p.C + c) * 4 + pos;
#pragma unroll
                    for (int q = 0; q < 8; ++q) dst[4 * q] = cv[q];
                }
            }
            *reinterpret_cast<uint4*>(p.out + (int64_t)t * p.ldo + c) = res;
        }
    }
    tc_fence_before();
    named_sync(kBarEpilogue, kBM);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tb, kBN);
    }
}

// 2-D map over a [rows, K] bf16 matrix with row stride ld (elements), box (64, box_rows).
static bool make_map2(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace inproj

int launch_in_proj_conv(const InProjArgs& a, cudaStream_t s) {
    using namespace inproj;
    if (a.T == 0 || a.N == 0) return GDN_OK;
    static bool ready[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_LAUNCH;
    if (!ready[dev]) {
        if (cudaFuncSetAttribute(in_proj_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
            cudaSuccess)
            return GDN_ERR_LAUNCH;
        ready[dev] = true;
    }
    Params p;
    memset(&p, 0, sizeof(p));
    if (!make_map2(&p.tm_x, a.x, a.T, a.K, a.ldx, kBM) || !make_map2(&p.tm_w, a.w, a.N, a.K, a.ldw, kBN))
        return GDN_ERR_LAUNCH;
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
    if (a.conv_tail &&
        cudaMemsetAsync(a.conv_tail, 0, (size_t)a.nseq * a.C * 4 * sizeof(bf16), s) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    dim3 grid((unsigned)((a.T + kOutRows - 1) / kOutRows), (unsigned)((a.N + kBN - 1) / kBN));
    in_proj_conv_kernel<<<grid, kThreads, kSmemBytes, s>>>(p);
    return launch_status();
}

}  // namespace gdn
