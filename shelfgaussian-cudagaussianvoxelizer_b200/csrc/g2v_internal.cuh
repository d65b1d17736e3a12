// g2v_internal.cuh -- shared constants, device helpers and host plumbing of libg2v.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>

namespace g2v {

constexpr int kTile = 4;                          // tile edge in voxels (reference include/utils.cuh:50-52)
constexpr int kVoxPerTile = kTile * kTile * kTile;  // 64
constexpr float kEps = 1e-6f;                     // density clamp of the normalisation (utils.cuh:80)
// Bits of the library's device error word (bits 1, 2, 4: bounded waits and CSR capacity guards of the
// tensor-core kernels).
constexpr int kErrCapacity = 8;                   // a capacity-capped call needed more pairs than its cap

// ---------------------------------------------------------------------------------------------
// Grid geometry passed by value to kernels.
struct Grid {
    float r0[3];     // range origin
    float r1[3];     // range end
    float h[3];      // voxel size
    int dims[3];     // X, Y, Z voxels
    int tiles[3];    // Tx, Ty, Tz tiles
    int xoff;        // voxel x of the first row of the volume arrays (0: the arrays cover the whole grid)
    int xlen;        // voxel x rows held by the volume arrays (dims[0] for whole-grid arrays)
    int scene_x;     // scenes stacked along x: voxel x rows per scene (0: one scene); dims/tiles[0] cover all
};

// Row (voxel index) of voxel (x, y, z) in the volume arrays (density, grid_feats and their gradients).
__host__ __device__ __forceinline__ int64_t grid_row(const Grid& G, int x, int y, int z) {
    return ((int64_t)(x - G.xoff) * G.dims[1] + y) * G.dims[2] + z;
}

// Voxel centre along one axis: origin + (i + 1/2) * h (reference cu:825-828).  For a batch of scenes
// stacked along x the index is first made scene-local (an integer step, so the centre is the same float
// as in a single-scene call).
__device__ __forceinline__ float voxel_centre(const Grid& G, int a, int i) {
    if (a == 0 && G.scene_x > 0) i -= (i / G.scene_x) * G.scene_x;
    return G.r0[a] + (static_cast<float>(i) + 0.5f) * G.h[a];
}

// Local voxel index inside a tile, x-major: lv = (lx*4 + ly)*4 + lz (reference DecodeTileVoxel cu:1226).
__device__ __forceinline__ void local_voxel(int lv, int& lx, int& ly, int& lz) {
    lx = lv >> 4;
    ly = (lv >> 2) & 3;
    lz = lv & 3;
}

__device__ __forceinline__ void decode_tile(int tile, const Grid& G, int& tx, int& ty, int& tz) {
    const int tyz = G.tiles[1] * G.tiles[2];
    tx = tile / tyz;
    const int r = tile - tx * tyz;
    ty = r / G.tiles[2];
    tz = r - ty * G.tiles[2];
}

// Tile box of a Gaussian from its voxel box; empty (returns false) when the voxel box is empty.
__device__ __forceinline__ bool tile_box(const int32_t* lb, const int32_t* ub, int64_t g, int lo[3], int hi[3]) {
    bool ok = true;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        const int l = lb[g * 3 + a], u = ub[g * 3 + a];
        ok = ok && (u >= l);
        lo[a] = l / kTile;
        hi[a] = u / kTile;
    }
    return ok;
}

// exp(-1/2 d^T P d) with d = centre - mean and q = P d; returns the exponential, writes q.
__device__ __forceinline__ float eval_gaussian(const float* c, float dx, float dy, float dz, float& qx, float& qy,
                                               float& qz) {
    qx = c[0] * dx + c[1] * dy + c[2] * dz;
    qy = c[3] * dx + c[4] * dy + c[5] * dz;
    qz = c[6] * dx + c[7] * dy + c[8] * dz;
    const float maha = dx * qx + dy * qy + dz * qz;
    return __expf(-0.5f * maha);
}

// ---------------------------------------------------------------------------------------------
// Host side: workspace carving (256-byte aligned sub-buffers of one caller-provided block).
struct Carver {
    char* base;
    size_t off = 0;
    explicit Carver(void* p) : base(static_cast<char*>(p)) {}
    template <typename T>
    T* take(size_t count) {
        off = (off + 255) & ~size_t(255);
        T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
    size_t bytes() const { return (off + 255) & ~size_t(255); }
};

// Error reporting (defined in g2v_api.cu).
void set_error(const char* fmt, ...);
void clear_error();  // empties the thread's g2v_last_error() message (done at every entry point)
int cuda_fail(cudaError_t e, const char* what);
// Grid geometry from voxel_size / voxel_range, with the library's size limits (a g2v_status code).
int make_grid(const float size[3], const float range[6], Grid& G);
// Device error word of the bounded waits and capacity guards: queue its read on `s` (the caller
// synchronises the stream before looking at *host_word), then turn a non-zero word into a status
// (clearing the word on the device).
int queue_error_read(cudaStream_t s, int* host_word);
int report_device_error(int word, cudaStream_t s);

#define G2V_LAUNCH_CHECK(what)                                  \
    do {                                                        \
        cudaError_t _e = cudaGetLastError();                    \
        if (_e != cudaSuccess) return ::g2v::cuda_fail(_e, what); \
    } while (0)

#define G2V_CUDA(call)                                          \
    do {                                                        \
        cudaError_t _e = (call);                                \
        if (_e != cudaSuccess) return ::g2v::cuda_fail(_e, #call); \
    } while (0)

// ---------------------------------------------------------------------------------------------
// Launchers implemented in the .cu files (all return a g2v_status code).
// scales / quats non-NULL: the covariance is formed from them in the kernel (cov unused).
// scene_offsets (num_scenes + 1, int32) non-NULL: Gaussians [scene_offsets[b], scene_offsets[b+1]) belong
// to scene b of a batch stacked along x (G.scene_x rows per scene); their boxes are clamped to the scene
// and returned in stacked coordinates (x + b * scene_x).
int launch_prepare_boxes(const float* means, const float* cov, int64_t n, const Grid& G, float* cov_inv,
                         int32_t* lb, int32_t* ub, int32_t* num_voxels, int32_t* num_tiles, cudaStream_t s,
                         const float* scales = nullptr, const float* quats = nullptr,
                         const int32_t* scene_offsets = nullptr, int num_scenes = 1);

size_t scan_workspace_bytes(int64_t n);
// Exclusive prefix sum of n int32 counts into out[0..n] (out[n] = total).  `total` (device, int64)
// receives the sum.  cap >= 0: the offsets are clamped to cap and a larger total sets kErrCapacity in
// *err (capacity-capped calls that never read the total back on the host).
int launch_exclusive_scan(const int32_t* counts, int64_t n, int32_t* out, int64_t* total, void* ws,
                          cudaStream_t s, int64_t cap = -1, int* err = nullptr);

}  // namespace g2v

// ---------------------------------------------------------------------------------------------
// Optional per-kernel timing (g2v_profile_enable): CUDA events recorded on the launch stream around
// every kernel launch, aggregated by kernel name when read back.  Off by default.
namespace g2v {
extern volatile int g_profiling;
int prof_start(const char* name, cudaStream_t s);
void prof_stop(int slot, cudaStream_t s);
}  // namespace g2v

#define G2V_TIMED(name, stream, ...)                                           \
    do {                                                                       \
        const int _slot = ::g2v::g_profiling ? ::g2v::prof_start(name, stream) : -1; \
        __VA_ARGS__;                                                           \
        if (_slot >= 0) ::g2v::prof_stop(_slot, stream);                       \
    } while (0)
