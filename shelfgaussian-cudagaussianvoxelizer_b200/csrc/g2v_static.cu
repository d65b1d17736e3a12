// g2v_static.cu -- g2v_forward_prepare_static: the forward's first stage without a caller workspace.
//
// Some callers cannot hand the library scratch memory.  A serving process that reserves all of its
// device memory at start-up and treats any later cudaMalloc as an error, or a plugin whose host
// application owns every device allocation, has no way to provide the workspace that
// g2v_forward_prepare asks for.  For them this entry point keeps its scratch in a fixed array in the
// library's own device memory, so a call needs nothing but its inputs and outputs.
//
// The array is file-scope device memory: every GPU that loads the library holds it (about 1 MiB)
// until the process exits.  Host code cannot use the array's name as a device address, so the first
// call on each device looks the address up with cudaGetSymbolAddress (with that device current) and
// caches it; that lookup can load the library's device code on the device, so make the first call
// before capturing a stream into a CUDA graph.  The cache is kept per device ordinal and assumes one
// primary context per device for the life of the process: after cudaDeviceReset (or any teardown and
// re-creation of the device's context) the cached address is stale and must not be used.  All calls
// share the one array: two calls whose work overlaps on the GPU (different streams, or different host
// threads without ordering) race on it.
//
// Grid limits and error reporting are those of g2v_forward_prepare: the same make_grid checks, and the
// library's device error word is read at the call's one synchronisation and reported as a status.
#include <mutex>

#include "g2v.h"
#include "g2v_internal.cuh"

namespace g2v {

namespace {

constexpr int64_t kStaticMaxGaussians = G2V_STATIC_MAX_GAUSSIANS;
// per-Gaussian tile counts, then the scan's block sums, then the scan total (all 256-byte aligned)
constexpr size_t kCountsBytes = ((size_t)kStaticMaxGaussians * sizeof(int32_t) + 255) & ~size_t(255);
constexpr size_t kScanBytes = (((size_t)(kStaticMaxGaussians + 2047) / 2048) * sizeof(int64_t) + 255) & ~size_t(255);
constexpr size_t kScratchBytes = kCountsBytes + kScanBytes + 256;

static __device__ __align__(256) unsigned char g_prepare_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {nullptr};

// Device address of g_prepare_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    G2V_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("device ordinal %d is beyond the %d devices this entry point supports", dev, kMaxDevices);
        return G2V_ERROR_NOT_SUPPORTED;
    }
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (g_addr[dev] == nullptr) {
        void* p = nullptr;
        G2V_CUDA(cudaGetSymbolAddress(&p, g_prepare_scratch));
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return 0;
}

}  // namespace
}  // namespace g2v

using namespace g2v;

extern "C" int g2v_forward_prepare_static(const float* means3d, const float* covariances, int64_t num_gaussians,
                                          const float voxel_size[3], const float voxel_range[6], float* cov_inv,
                                          int32_t* valid_voxel_lb, int32_t* valid_voxel_ub, int32_t* num_voxels,
                                          int32_t* g2t_offsets, void* stream, int64_t* num_pairs) {
    clear_error();
    if (num_gaussians > kStaticMaxGaussians) {
        set_error("g2v_forward_prepare_static handles at most %lld Gaussians (got %lld); use "
                  "g2v_forward_prepare with a workspace for larger inputs",
                  (long long)kStaticMaxGaussians, (long long)num_gaussians);
        return G2V_ERROR_SIZE_LIMIT;
    }
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if (num_gaussians < 0 || !g2t_offsets || !num_pairs ||
        (num_gaussians > 0 && (!means3d || !covariances || !cov_inv || !valid_voxel_lb || !valid_voxel_ub ||
                               !num_voxels))) {
        set_error("g2v_forward_prepare_static: invalid pointer or Gaussian count");
        return G2V_ERROR_INVALID_VALUE;
    }
    void* base = nullptr;
    rc = scratch_address(&base);
    if (rc) return rc;
    unsigned char* b = static_cast<unsigned char*>(base);
    int32_t* counts = reinterpret_cast<int32_t*>(b);
    void* scan_ws = b + kCountsBytes;
    int64_t* total = reinterpret_cast<int64_t*>(b + kCountsBytes + kScanBytes);
    // Every scratch word this call reads is written earlier in the same call (counts by the box kernel,
    // block sums and total by the scan), so nothing has to be cleared between calls.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((rc = launch_prepare_boxes(means3d, covariances, num_gaussians, G, cov_inv, valid_voxel_lb, valid_voxel_ub,
                                   num_voxels, counts, s)))
        return rc;
    if ((rc = launch_exclusive_scan(counts, num_gaussians, g2t_offsets, total, scan_ws, s))) return rc;
    int64_t m = 0;
    int word = 0;
    G2V_CUDA(cudaMemcpyAsync(&m, total, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    if ((rc = queue_error_read(s, &word))) return rc;
    G2V_CUDA(cudaStreamSynchronize(s));
    if ((rc = report_device_error(word, s))) return rc;
    if (m > INT32_MAX) {
        set_error("%lld (Gaussian, tile) pairs exceed the int32 range of the Gaussian->Tile map", (long long)m);
        return G2V_ERROR_SIZE_LIMIT;
    }
    *num_pairs = m;
    return G2V_SUCCESS;
}
