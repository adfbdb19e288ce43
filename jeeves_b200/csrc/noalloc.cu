// Decode layer for callers that cannot allocate device memory.
//
// gdn_decode_layer needs a [B, C] bf16 workspace for the post-conv activations, which the
// caller normally allocates. Some callers cannot do that: a plugin host or serving process
// that has handed all device memory to its own pool and gives this library no allocator,
// a foreign-language binding (cgo, JNI) with no device buffer of its own to pass, or code
// that must not grow the process's device footprint after start-up. This variant keeps the
// workspace in a fixed file-scope device array instead and calls no allocating routine.
//
// Limits and sharing rules (also stated in include/gdn_b200.h):
//   * the array holds kNoAllocScratchElems bf16 values (4 MiB): batch * C must not exceed
//     it, larger requests return GDN_ERR_SCRATCH before anything is launched;
//   * every GPU that loads the library holds the 4 MiB until the process exits;
//   * every call on a device shares the one array, which keeps the last call's contents;
//     nothing in it needs to start at zero (the conv pass writes all batch * C values before
//     the step reads them), but calls that overlap on the GPU (concurrent streams) race;
//   * the first call on a device looks the array's device address up (cudaGetSymbolAddress
//     with that device current) and caches it; make that first call before any stream
//     capture.

#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace gdn {

constexpr int64_t kNoAllocScratchElems = int64_t(1) << 21;  // bf16 values: 4 MiB
static __device__ __align__(256) bf16 g_noalloc_scratch[kNoAllocScratchElems];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device. In host code the array's name
// is only a stand-in for the symbol, so the address is looked up with the device current.
int scratch_address(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_LAUNCH;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void* addr = nullptr;
        if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || addr == nullptr) return GDN_ERR_LAUNCH;
        g_scratch_addr[dev] = addr;
    }
    *out = g_scratch_addr[dev];
    return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_decode_layer_noalloc(const void* qkv, int64_t qkv_stride_b, void* conv_state, const void* conv_w,
                                        const float* g, const void* beta, float* state, const void* z,
                                        const void* norm_w, void* out, int64_t batch, int64_t key_heads,
                                        int64_t value_heads, int64_t head_dim_k, int64_t head_dim_v, int64_t taps,
                                        int64_t kernel_size, float scale, float eps, void* stream) {
    using namespace gdn;
    if (batch < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads) return GDN_ERR_SHAPE;
    if (taps < 1 || kernel_size < 1 || kernel_size > taps + 1) return GDN_ERR_SHAPE;
    if (taps < 2 || taps > 4 || kernel_size < 2) return GDN_ERR_UNSUPPORTED;
    if (head_dim_k != kHeadDim || head_dim_v != kHeadDim) return GDN_ERR_UNSUPPORTED;
    if (batch > 65535 || value_heads > 65535) return GDN_ERR_SHAPE;
    const int64_t channels = (2 * key_heads + value_heads) * kHeadDim;
    if (batch * channels > kNoAllocScratchElems) return GDN_ERR_SCRATCH;
    if (batch == 0) return GDN_OK;
    if (!qkv || !conv_state || !conv_w || !g || !beta || !state || !z || !norm_w || !out) return GDN_ERR_NULL;
    if (!aligned16(qkv) || (qkv_stride_b * 2) % 16 || !aligned16(conv_state) || !aligned16(state) || !aligned16(z) ||
        !aligned16(conv_w) || !aligned16(out) || !aligned16(norm_w))
        return GDN_ERR_ALIGN;
    void* workspace = nullptr;
    const int st = scratch_address(&workspace);
    if (st != GDN_OK) return st;
    DecodeLayerArgs a;
    a.qkv = qkv; a.qkv_sb = qkv_stride_b; a.conv_state = conv_state; a.conv_w = conv_w;
    a.g = g; a.beta = beta; a.state = state; a.z = z; a.norm_w = norm_w; a.out = out; a.workspace = workspace;
    a.B = batch; a.H = (int)key_heads; a.HV = (int)value_heads; a.taps = (int)taps; a.K = (int)kernel_size;
    a.scale = scale; a.eps = eps;
    return launch_decode_layer(a, static_cast<cudaStream_t>(stream));
}
