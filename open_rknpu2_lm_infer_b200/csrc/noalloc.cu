// Router + top-k without any device allocation.
//
// The regular router path (moe_b200_route_device) keeps its logits and tile
// counters in a workspace made by moe_b200_workspace_create, which calls
// cudaMalloc. Some callers cannot do that: a serving engine that hands all of
// HBM to its own pool or caching allocator at start-up and must not allocate
// behind its back, or a latency-critical hot path where cudaMalloc (which may
// synchronise the device) or an out-of-memory error mid-request is not
// acceptable. moe_b200_route_noalloc serves them: it takes device inputs and
// outputs from the caller and uses the fixed scratch array below instead of
// a workspace. It allocates nothing (no cudaMalloc, cudaFree or allocating
// library call).
//
// The scratch array is file-scope device memory: every GPU that loads this
// library holds it (about 4.3 MiB) until the process exits. All calls on a
// device share it and it keeps the last call's contents, so calls whose
// execution overlaps on that GPU (different streams, or several host threads)
// race on it and must be serialised by the caller.
#include <mutex>

#include "../../include/moe_b200.h"
#include "kernels.cuh"

namespace {

constexpr long kMaxLogits = MOE_B200_NOALLOC_MAX_LOGITS;  // rows * experts
constexpr long kMaxTiles = MOE_B200_NOALLOC_MAX_LOGITS / 16;  // router tile counters
constexpr long kScratchWords = kMaxLogits + kMaxTiles + 64;

// [0, kMaxLogits): logits; then the tile counters; then the status word.
static __device__ __align__(256) uint32_t g_route_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device. The host-side
// name g_route_scratch is only a stand-in, so the address is looked up with
// cudaGetSymbolAddress, once per device, on the first call made with that
// device current.
int scratch_for_device(int dev, uint32_t** out) {
    if (dev < 0 || dev >= kMaxDevices) return MOE_B200_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess || !p) return MOE_B200_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *out = static_cast<uint32_t*>(g_scratch_addr[dev]);
    return MOE_B200_OK;
}

}  // namespace

extern "C" int moe_b200_route_noalloc(const float* d_input, const float* d_router,
                                      const float* d_bias, int32_t rows, int32_t hidden,
                                      int32_t experts, int32_t top, int32_t order,
                                      float min_weight, int32_t* d_ids, float* d_routes,
                                      void* stream) {
    if (rows < 0 || hidden <= 0 || experts <= 0 || experts > 1024 || top <= 0 || top > 32 ||
        top > experts)
        return MOE_B200_ERR_INVALID;
    if (order != MOE_B200_ROUTER_NEON16 && order != MOE_B200_ROUTER_SEQUENTIAL)
        return MOE_B200_ERR_INVALID;
    if (!(min_weight >= 0.0f && min_weight <= 1.0f)) return MOE_B200_ERR_INVALID;
    // the router kernels stream rows in 16-byte vectors (the workspace path's
    // hidden % 32 rule); a small batch stages its weight rows in shared memory
    if (hidden % 32) return MOE_B200_ERR_UNSUPPORTED;
    if ((long)rows * experts > kMaxLogits) return MOE_B200_ERR_NOALLOC_LIMIT;
    if (rows == 0) return MOE_B200_OK;
    if (!moe::router_fits(rows, hidden, order)) return MOE_B200_ERR_UNSUPPORTED;
    if (!d_input || !d_router || !d_ids || !d_routes) return MOE_B200_ERR_INVALID;
    auto misaligned = [](const void* p, uintptr_t a) {
        return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0;
    };
    if (misaligned(d_input, 16) || misaligned(d_router, 16) || misaligned(d_bias, 4) ||
        misaligned(d_ids, 4) || misaligned(d_routes, 4))
        return MOE_B200_ERR_INVALID;
    int dev = -1, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MOE_B200_ERR_NO_DEVICE;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) return MOE_B200_ERR_NO_DEVICE;
    uint32_t* scratch = nullptr;
    int rc = scratch_for_device(dev, &scratch);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* logits = reinterpret_cast<float*>(scratch);
    int* counters = reinterpret_cast<int*>(scratch + kMaxLogits);
    uint32_t* err = scratch + kMaxLogits + kMaxTiles;
    // The router's tile counters and the status word must start at zero; the
    // logits are fully overwritten before they are read.
    // (one counter per router tile; never more tiles than rows, nor than kMaxTiles)
    const long tiles = rows < kMaxTiles ? rows : kMaxTiles;
    if (cudaMemsetAsync(counters, 0, sizeof(int) * (size_t)tiles, s) != cudaSuccess ||
        cudaMemsetAsync(err, 0, sizeof(uint32_t), s) != cudaSuccess)
        return MOE_B200_ERR_CUDA;
    moe::RouterArgs a{};
    a.x = d_input;
    a.w = d_router;
    a.bias = d_bias;
    a.T = rows;
    a.H = hidden;
    a.E = experts;
    a.k = top;
    a.order = order;
    a.min_weight = min_weight;
    a.logits = logits;
    a.counters = counters;
    a.ids = d_ids;
    a.weights = d_routes;
    a.err = err;
    if (moe::launch_router(a, s)) return MOE_B200_ERR_UNSUPPORTED;
    return cudaPeekAtLastError() == cudaSuccess ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}
