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
#include "gates.cuh"
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
    float* deltas;  // [B, T, HV, 128]: each token's update vector delta_t, or null
    int64_t T;
    int HV, rep;
    int64_t qsb, qst, qsh, ksb, kst, ksh, vsb, vst, vsh;
    float scale;
    GateInputs gates;  // beta and g from the raw projections when gates.b is set
    int64_t ahead;     // (16-column tiles) CTAs resident at once, or 0; see the kernel
};

// 1 / sqrt(|k|^2 + 1e-6) of one token's key row; lane l holds elements 4l .. 4l + 3.
__device__ __forceinline__ float key_rnorm(const float4& kl) {
    const float kk = warp_sum(kl.x * kl.x + kl.y * kl.y + kl.z * kl.z + kl.w * kl.w);
    return rsqrtf(kk + 1e-6f);
}

// S <- e^g S + k delta^T on this thread's RPT state rows row0 .. row0 + RPT - 1 (four columns):
// the normalised key element of row i is lane i/4's element i%4 times rk. The recurrent step
// and the delta commit share it, so that they leave the same bits.
template <int RPT>
__device__ __forceinline__ void state_step(float4 (&S)[RPT], const float4& kl, float rk, float decay,
                                           const float4& delta, int row0) {
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
}

// GATES: beta and g are computed from p.gates (a separate instantiation, so that the plain
// path keeps its code unchanged).
template <typename TIn, typename TBeta, int VS, int NT, bool GATES>
__global__ void __launch_bounds__(NT) recurrent_kernel(const RecurrentParams p) {
    constexpr int COLG = VS / 4;   // threads along one state row
    constexpr int ROWG = NT / COLG;
    constexpr int RPT = kHeadDim / ROWG;  // state rows per thread
    // Every tile sums k^T S and q^T S in one tree: 8-row leaves (in row order), leaves combined
    // pairwise by xor shuffles up to the 32 / COLG leaves of a warp of the 8-row tile (RPT = 8),
    // then those warp sums in order through shared memory. A tile with RPT = 16 adds its two
    // leaves in the thread and continues the same tree, so that both tiles give the same bits.
    constexpr int LEAVES = RPT / 8;
    constexpr int L = 32 / COLG;          // leaves a warp of the 8-row tile holds
    constexpr int NREF = 16 / L;          // warp sums of the 8-row tile
    constexpr int GROUP = L / LEAVES;     // row groups that hold one warp sum after the shuffles
    static_assert(COLG <= 32 && 32 % COLG == 0 && (RPT == 8 || RPT == 16) && GROUP >= 1, "bad tile");
    __shared__ float4 red[2][2][NREF][COLG];

    const int tid = threadIdx.x, lane = tid & 31;
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
    // The small-batch tiles (16 columns) run their grid in about two waves: each CTA of the first asks
    // L2 for the slice of the CTA one wave later in the grid's linear order, so that the second
    // wave's loads find their state there (decode at 32 rows 0.734 -> 0.680 ms a 24-layer step).
    // The 32-column tile runs many waves and keeps its registers (with this code 87 instead of 80,
    // one CTA an SM fewer: 256 rows 4.12 -> 4.75 ms).
    if constexpr (VS == 16) {
        if (p.ahead > 0 && p.state_in) {
            const int64_t gx = gridDim.x, gy = gridDim.y;
            const int64_t tgt = blockIdx.x + gx * (blockIdx.y + gy * (int64_t)blockIdx.z) + p.ahead;
            if (tgt < gx * gy * (int64_t)gridDim.z) {
                const int64_t tx = tgt % gx, ty = (tgt / gx) % gy, tz = tgt / (gx * gy);
                const float* far = p.state_in + (tz * p.HV + ty) * (int64_t)(kHeadDim * kHeadDim) +
                                   (int64_t)row0 * kHeadDim + tx * VS + cg * 4;
#pragma unroll
                for (int r = 0; r < RPT; ++r) asm volatile("prefetch.global.L2 [%0];" ::"l"(far + r * kHeadDim));
            }
        }
    }
    // As a programmatic dependent of the decode layer's conv step, the state loads above overlap
    // that kernel; q, k, v come from it, so they are read only past this point.
    pdl_wait();
    pdl_launch_dependents();

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
        float decay, bt;
        if constexpr (GATES) {
            float gv;
            delta_gate(p.gates, brow * p.T + tok, hv, bt, gv);
            decay = expf(gv);
        } else {
            decay = expf(p.g[gi]);
            bt = to_f32(beta[gi]);
        }

        const float rk = key_rnorm(kl);
        float rq = 0.f, qk = 0.f;
        if (outputs) {
            const float qq = warp_sum(ql.x * ql.x + ql.y * ql.y + ql.z * ql.z + ql.w * ql.w);
            qk = warp_sum(ql.x * kl.x + ql.y * kl.y + ql.z * kl.z + ql.w * kl.w);
            rq = rsqrtf(qq + 1e-6f) * p.scale;
        }

        // Partial sums over this thread's rows, one per 8-row leaf. Row i of k sits in lane i/4,
        // element i%4; RPT is a multiple of 4, so the element index is the same across the warp.
        float4 pk[LEAVES], pq[LEAVES];
#pragma unroll
        for (int e = 0; e < LEAVES; ++e) pk[e] = pq[e] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            const int src = (row0 + r) >> 2;
            const float kr = (r & 3) == 0 ? kl.x : (r & 3) == 1 ? kl.y : (r & 3) == 2 ? kl.z : kl.w;
            const float ki = __shfl_sync(0xffffffffu, kr, src) * rk;
            float4& a = pk[r >> 3];
            a.x += ki * S[r].x; a.y += ki * S[r].y; a.z += ki * S[r].z; a.w += ki * S[r].w;
            if (outputs) {
                const float qr = (r & 3) == 0 ? ql.x : (r & 3) == 1 ? ql.y : (r & 3) == 2 ? ql.z : ql.w;
                const float qi = __shfl_sync(0xffffffffu, qr, src) * rq;
                float4& b = pq[r >> 3];
                b.x += qi * S[r].x; b.y += qi * S[r].y; b.z += qi * S[r].z; b.w += qi * S[r].w;
            }
        }
        float4 sk = pk[0], sq = pq[0];
        if (LEAVES == 2) {
            sk.x += pk[LEAVES - 1].x; sk.y += pk[LEAVES - 1].y; sk.z += pk[LEAVES - 1].z; sk.w += pk[LEAVES - 1].w;
            sq.x += pq[LEAVES - 1].x; sq.y += pq[LEAVES - 1].y; sq.z += pq[LEAVES - 1].z; sq.w += pq[LEAVES - 1].w;
        }
#pragma unroll
        for (int off = COLG; off < COLG * GROUP; off <<= 1) {
            sk.x += __shfl_xor_sync(0xffffffffu, sk.x, off);
            sk.y += __shfl_xor_sync(0xffffffffu, sk.y, off);
            sk.z += __shfl_xor_sync(0xffffffffu, sk.z, off);
            sk.w += __shfl_xor_sync(0xffffffffu, sk.w, off);
            if (outputs) {
                sq.x += __shfl_xor_sync(0xffffffffu, sq.x, off);
                sq.y += __shfl_xor_sync(0xffffffffu, sq.y, off);
                sq.z += __shfl_xor_sync(0xffffffffu, sq.z, off);
                sq.w += __shfl_xor_sync(0xffffffffu, sq.w, off);
            }
        }
        if (rg % GROUP == 0) {
            red[buf][0][rg / GROUP][cg] = sk;
            if (outputs) red[buf][1][rg / GROUP][cg] = sq;
        }
        __syncthreads();
        float4 rs = red[buf][0][0][cg];
#pragma unroll
        for (int w = 1; w < NREF; ++w) {
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
            for (int w = 1; w < NREF; ++w) {
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
        if (p.deltas && rg == 0) *reinterpret_cast<float4*>(p.deltas + gi * kHeadDim + col) = delta;
        state_step(S, kl, rk, decay, delta, row0);
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

// The commit of a verify that kept its update vectors (gdn_recurrent_deltas): state[n] advances
// by clamp(accepted[n], 0, T) tokens with S <- e^{g_t} S + k_t delta_t^T, the recurrent step's
// own arithmetic (state_step) without its reductions, so it leaves the bits the advance would.
// Pure streaming: one CTA per 128 x VS slice, the slice loaded once, every token applied in
// registers, stored once.
//
// LAYERS: one launch commits up to kCommitLayers layers (the engine's commit loop over its layers,
// inference/engine.py:471-472). The grid's z index runs over (row, layer), the layer slowest, so
// the CTAs resident at a time stream one layer's states in address order, as one launch a layer
// would, without the tails and gaps between launches (24 layers: 16 rows 14.5 -> 10.5 us a layer,
// 64 rows 45 -> 41.5, 128 rows 89.5 -> 89.2). With the layer index fastest the CTAs in flight
// spread over every layer's states, and 128 rows took 5 % longer. The one-layer form reads its
// pointers straight from the parameters.
constexpr int kCommitLayers = 64;
struct DeltaCommitParams {
    float* state[kCommitLayers];
    const void* k[kCommitLayers];
    const float* g[kCommitLayers];
    const float* deltas[kCommitLayers];
    const int64_t* accepted;
    int64_t rows, T;
    int HV, rep;
    int64_t ksb, kst, ksh;
};

// At most 64 registers, so that 8 CTAs an SM keep their state loads in flight.
template <typename TIn, int VS, int NT, bool LAYERS>
__global__ void __launch_bounds__(NT, 65536 / (NT * 64)) delta_commit_kernel(const __grid_constant__ DeltaCommitParams p) {
    constexpr int COLG = VS / 4;
    constexpr int ROWG = NT / COLG;
    constexpr int RPT = kHeadDim / ROWG;
    static_assert(COLG <= 32 && 32 % COLG == 0 && RPT % 4 == 0, "bad tile");
    const int tid = threadIdx.x, lane = tid & 31;
    const int cg = tid % COLG, rg = tid / COLG;
    const int row0 = rg * RPT;
    const int hv = blockIdx.y;
    const int64_t n = LAYERS ? blockIdx.z % (uint32_t)p.rows : blockIdx.z;
    const int layer = LAYERS ? (int)(blockIdx.z / (uint32_t)p.rows) : 0;
    const int h = hv / p.rep;
    const int col = blockIdx.x * VS + cg * 4;
    const int64_t a = p.accepted[n];
    const int64_t nsteps = a < 0 ? 0 : (a > p.T ? p.T : a);
    if (nsteps == 0) return;  // nothing accepted: the state stays as it is
    float* tile = p.state[layer] + (n * p.HV + hv) * (int64_t)(kHeadDim * kHeadDim) + (int64_t)row0 * kHeadDim + col;
    float4 S[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) S[r] = ldg_stream(reinterpret_cast<const float4*>(tile + r * kHeadDim));
    const TIn* kbase = static_cast<const TIn*>(p.k[layer]) + n * p.ksb + h * p.ksh;
    const float* g = p.g[layer];
    const float* deltas = p.deltas[layer];
    for (int64_t t = 0; t < nsteps; ++t) {
        const float4 kl = load4(kbase + t * p.kst + 4 * lane);
        const int64_t gi = (n * p.T + t) * p.HV + hv;
        const float decay = expf(g[gi]);
        const float4 delta = *reinterpret_cast<const float4*>(deltas + gi * kHeadDim + col);
        state_step(S, kl, key_rnorm(kl), decay, delta, row0);
    }
#pragma unroll
    for (int r = 0; r < RPT; ++r) stg_stream(reinterpret_cast<float4*>(tile + r * kHeadDim), S[r]);
}

int launch_delta_commit(const DeltaCommitArgs& a, cudaStream_t s) {
    if (a.rows == 0 || a.T == 0 || a.layers == 0) return GDN_OK;
    DeltaCommitParams p;
    memset(&p, 0, sizeof(p));
    p.accepted = a.accepted;
    p.rows = a.rows; p.T = a.T; p.HV = a.HV; p.rep = a.HV / a.H;
    p.ksb = a.ksb; p.kst = a.kst; p.ksh = a.ksh;
    int per = kCommitLayers;
    if (per > 65535 / a.rows) per = (int)(65535 / a.rows);  // the grid's z index covers rows x layers
    for (int64_t l0 = 0; l0 < a.layers; l0 += per) {
        const int n = (int)(a.layers - l0 < per ? a.layers - l0 : per);
        for (int i = 0; i < n; ++i) {
            p.state[i] = a.states[l0 + i];
            p.k[i] = a.ks[l0 + i];
            p.g[i] = a.gs[l0 + i];
            p.deltas[i] = a.deltas[l0 + i];
        }
        const dim3 grid(kHeadDim / 32, a.HV, (unsigned)(a.rows * n));
        if (n > 1) {
            if (a.k_dtype == GDN_BF16) delta_commit_kernel<bf16, 32, 128, true><<<grid, 128, 0, s>>>(p);
            else delta_commit_kernel<float, 32, 128, true><<<grid, 128, 0, s>>>(p);
        } else {
            if (a.k_dtype == GDN_BF16) delta_commit_kernel<bf16, 32, 128, false><<<grid, 128, 0, s>>>(p);
            else delta_commit_kernel<float, 32, 128, false><<<grid, 128, 0, s>>>(p);
        }
        const int st = launch_status();
        if (st != GDN_OK) return st;
    }
    return GDN_OK;
}

template <typename Kernel>
static int launch_maybe_dependent(Kernel kernel, dim3 grid, int threads, bool dependent, const RecurrentParams& p,
                                  cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? launch_status() : GDN_ERR_LAUNCH;
}

// CTAs of `Kernel` resident at once on this device when the grid of `ctas` exceeds them (the
// prefetch distance of the 16-column tiles), else 0. Cached per (kernel, device).
template <auto Kernel>
static int64_t resident_ctas(int threads, int64_t ctas) {
    static int cached[64] = {0};  // one instantiation, so one cache, per kernel
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev] == 0) {
        int per_sm = 0, sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, Kernel, threads, 0) != cudaSuccess || per_sm <= 0)
            return 0;
        cached[dev] = per_sm * sms;
    }
    return ctas > cached[dev] ? cached[dev] : 0;
}

template <typename TIn, typename TBeta, bool GATES = false>
static int dispatch_recurrent(const RecurrentParams& p, int64_t rows, cudaStream_t s, bool dependent) {
    // Small grids split the value columns finer so that more SMs share the work.
    // Calls of several tokens a sequence (or packed sequences) hold 16 state rows a thread, which
    // spreads the per-token work (loads, norms, reductions) over twice the state; one-token
    // decode keeps 8 rows a thread and twice the threads, to keep more state loads in flight.
    // Both compute the same bits.
    const int64_t heads = rows * p.HV;
    const bool multi = p.T > 1 || p.cu_seqlens;
    if (heads >= 2048) {
        dim3 grid(kHeadDim / 32, p.HV, (unsigned)rows);
        if (multi) return launch_maybe_dependent(recurrent_kernel<TIn, TBeta, 32, 64, GATES>, grid, 64, dependent, p, s);
        return launch_maybe_dependent(recurrent_kernel<TIn, TBeta, 32, 128, GATES>, grid, 128, dependent, p, s);
    }
    dim3 grid(kHeadDim / 16, p.HV, (unsigned)rows);
    RecurrentParams q = p;
    const int64_t ctas = (int64_t)grid.x * grid.y * grid.z;
    if (multi) {
        q.ahead = resident_ctas<recurrent_kernel<TIn, TBeta, 16, 32, GATES>>(32, ctas);
        return launch_maybe_dependent(recurrent_kernel<TIn, TBeta, 16, 32, GATES>, grid, 32, dependent, q, s);
    }
    q.ahead = resident_ctas<recurrent_kernel<TIn, TBeta, 16, 64, GATES>>(64, ctas);
    return launch_maybe_dependent(recurrent_kernel<TIn, TBeta, 16, 64, GATES>, grid, 64, dependent, q, s);
}

int launch_recurrent(const RecurrentArgs& a, cudaStream_t s) {
    RecurrentParams p{};
    p.q = a.q; p.k = a.k; p.v = a.v; p.g = a.g; p.beta = a.beta;
    p.state_in = a.state_in; p.state_out = a.state_out; p.snapshots = a.snapshots; p.o = a.o;
    p.steps = a.steps; p.cu_seqlens = a.cu_seqlens; p.deltas = a.deltas;
    p.T = a.T; p.HV = a.HV; p.rep = a.HV / a.H;
    p.qsb = a.qsb; p.qst = a.qst; p.qsh = a.qsh;
    p.ksb = a.ksb; p.kst = a.kst; p.ksh = a.ksh;
    p.vsb = a.vsb; p.vst = a.vst; p.vsh = a.vsh;
    p.scale = a.scale;
    p.gates = a.gates;
    if (a.rows == 0) return GDN_OK;
    if (a.gates.b) {
        return a.qkv_dtype == GDN_BF16 ? dispatch_recurrent<bf16, bf16, true>(p, a.rows, s, a.dependent)
                                       : dispatch_recurrent<float, bf16, true>(p, a.rows, s, a.dependent);
    }
    if (a.qkv_dtype == GDN_BF16) {
        return a.beta_dtype == GDN_BF16 ? dispatch_recurrent<bf16, bf16>(p, a.rows, s, a.dependent)
                                        : dispatch_recurrent<bf16, float>(p, a.rows, s, a.dependent);
    }
    return a.beta_dtype == GDN_BF16 ? dispatch_recurrent<float, bf16>(p, a.rows, s, a.dependent)
                                    : dispatch_recurrent<float, float>(p, a.rows, s, a.dependent);
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
// Decode layer: one new token per row through conv step (+SiLU), q/k L2 norm, the gated
// delta rule step on the state in place and the output-gated RMSNorm, as three launches on
// the stream: (1) the conv step over all channels, each channel once, writing the post-conv
// activations to the caller's workspace and rolling the conv state forward; (2) the
// recurrent kernel above on 32-column state slices, writing o (bf16, as the reference rounds
// it before the norm) into `out`; (3) the gated RMSNorm in place on `out`.
// ---------------------------------------------------------------------------------------
int launch_decode_layer(const DecodeLayerArgs& a, cudaStream_t s) {
    if (a.B == 0) return GDN_OK;
    const int64_t key_dim = (int64_t)a.H * kHeadDim;
    const int64_t C = 2 * key_dim + (int64_t)a.HV * kHeadDim;
    // the conv launches as a programmatic dependent of whatever ran before (it waits for it before
    // touching memory), so that its launch overlaps the previous layer's last kernel
    int st = launch_conv1d_silu_step(a.qkv, a.qkv_sb, a.conv_state, a.conv_w, a.workspace, a.B, C, a.taps, a.K, s,
                                     true);
    if (st != GDN_OK) return st;
    const bf16* y = static_cast<const bf16*>(a.workspace);
    RecurrentArgs r{};
    r.q = y;
    r.k = y + key_dim;
    r.v = y + 2 * key_dim;
    r.qkv_dtype = GDN_BF16;
    r.g = a.g;
    r.beta = a.beta;
    r.beta_dtype = GDN_BF16;
    r.state_in = a.state;
    r.state_out = a.state;
    r.snapshots = nullptr;
    r.o = a.out;
    r.steps = nullptr;
    r.cu_seqlens = nullptr;
    r.rows = a.B;
    r.T = 1;
    r.H = a.H;
    r.HV = a.HV;
    r.qsb = C; r.qst = C; r.qsh = kHeadDim;
    r.ksb = C; r.kst = C; r.ksh = kHeadDim;
    r.vsb = C; r.vst = C; r.vsh = kHeadDim;
    r.scale = a.scale;
    r.dependent = true;  // its state loads overlap the conv step
    st = launch_recurrent(r, s);
    if (st != GDN_OK) return st;
    return launch_gated_rmsnorm(a.out, a.z, a.norm_w, a.out, a.B * a.HV, kHeadDim, a.eps, s, true);
}

}  // namespace gdn
