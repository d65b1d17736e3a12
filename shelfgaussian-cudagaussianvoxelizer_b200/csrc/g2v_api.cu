// g2v_api.cu -- the extern "C" entry points of libg2v.so (declared in include/g2v.h).
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "g2v.h"
#include "g2v_internal.cuh"
#include "g2v_tc.cuh"

namespace g2v {

static thread_local char g_msg[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return G2V_ERROR_CUDA;
}

// implemented in the other translation units
int build_cell_lists(const int32_t* lb, const int32_t* ub, int64_t n, const Grid& G, const int cell[3],
                     const int ncells_dim[3], int cell_x_begin, int cell_x_end, const int32_t* g2t_offsets,
                     int32_t* g2t_tile_ids, int64_t g2t_cap, int32_t* per_gaussian, int32_t* counts, int32_t* cell_offsets,
                     int32_t* unsorted, int32_t* lists, void* scan_ws, int64_t* total, cudaStream_t s,
                     int64_t list_cap, int* err, bool x_order = false);
int count_gaussian_cells(const int32_t* lb, const int32_t* ub, int64_t n, const Grid& G, const int cell[3],
                         int32_t* per_gaussian, int32_t* dummy_counts, cudaStream_t s);
int fill_g2t(const int32_t* lb, const int32_t* ub, int64_t n, const Grid& G, const int32_t* g2t_offsets,
             int32_t* g2t_tile_ids, int64_t g2t_cap, cudaStream_t s);
int launch_splat_simt(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                      const int32_t* ub, const float* features, int C, const int32_t* tile_offsets,
                      const int32_t* tile_lists, int first_tile, int num_tiles, const Grid& G, float* density,
                      float* grid_feats, cudaStream_t s);
int launch_splat_tc(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                    const int32_t* ub, const float* features, int64_t n, int C, const int32_t* unit_offsets,
                    const int32_t* unit_lists, int tile_x_begin, int tile_x_end, const Grid& G, float* density,
                    float* grid_feats, void* split, int* err, cudaStream_t s);
size_t splat_tc_split_bytes(int64_t n, int64_t C);
int launch_spass(const float* grad_density, const float* grad_feats, const float* means, const float* opacity,
                 const float* cov_inv, const int32_t* lb, const int32_t* ub, const float* features, int C,
                 const float* density, const int32_t* g2t_offsets, const int32_t* tile_offsets,
                 const int32_t* tile_lists, int first_tile, int num_tiles, const Grid& G, float* partial10,
                 int64_t pair_cap, cudaStream_t s);
int launch_fpass(const float* grad_feats, const float* means, const float* opacity, const float* cov_inv,
                 const int32_t* lb, const int32_t* ub, int C, const float* density, const int32_t* block_offsets,
                 const int32_t* block_lists, const int32_t* g2b_offsets, int bx_begin, int nbx, int nby, int nbz,
                 const int B[3], int tx_begin, int tx_end, const Grid& G, float* partialF, int64_t block_pair_cap,
                 cudaStream_t s);
int launch_fpass_tc(const float* grad_feats, int C, const float* density, const GParams* gparams,
                    const int32_t* block_offsets, const int32_t* block_lists, const int32_t* g2b_offsets, int bx_begin,
                    int nbx, int nby, int nbz, const int B[3], int tx_begin, int tx_end, const Grid& G, float* partialF,
                    int64_t block_pair_cap, int* err, cudaStream_t s);
size_t spass_tc_split_bytes(int64_t n, int64_t C);
void tc_unit_shape(const Grid& G, int cell[3], int ncells[3]);
int launch_spass_tc(const float* grad_density, const float* grad_feats, const float* features, int64_t n, int C,
                    const float* density, const GParams* gparams, const int32_t* g2t_offsets,
                    const int32_t* unit_offsets, const int32_t* unit_lists, int tile_x_begin, int tile_x_end,
                    const Grid& G, float* partial10, int64_t pair_cap, void* split, int* err, cudaStream_t s,
                    const float* grid_feats = nullptr, float* ev_buf = nullptr);
int launch_wait_timeout(int* err, cudaStream_t s, int* gave_up_host);
// scales / quats / grad_quats non-NULL: grad_cov receives dL/dscales (n,3) and grad_quats dL/dquats (n,4).
int launch_reduce10(const float* partial10, const int32_t* g2t_offsets, const int32_t* g2t_tile_ids, int64_t n,
                    const Grid& G, int tx_begin, int tx_end, float* grad_means, float* grad_cov,
                    float* grad_opacity, cudaStream_t s, const float* scales = nullptr,
                    const float* quats = nullptr, float* grad_quats = nullptr);
int launch_cov_from_scale_rot(const float* scales, const float* quats, int64_t n, float* cov, cudaStream_t s);
int launch_cov_from_scale_rot_backward(const float* scales, const float* quats, const float* grad_cov, int64_t n,
                                       float* grad_scales, float* grad_quats, cudaStream_t s);
int launch_reduce_feats(const float* partialF, const int32_t* g2b_offsets, const int32_t* lb, const int32_t* ub,
                        int64_t n, int C, const int B[3], int bx_begin, int bx_end, float* grad_features,
                        cudaStream_t s, int64_t row_cap);
size_t cosine_loss_workspace_bytes();
int launch_cosine_loss_fwd(const float* label, const uint8_t* mask, const float* p, const float* g, int64_t V, int C,
                           float* loss, int* count, void* ws, cudaStream_t s);
int launch_cosine_loss_bwd(const float* grad_out, const int* count_dev, int count_host, const float* label,
                           const uint8_t* mask, const float* p, const float* g, int64_t V, int C, float* gp,
                           cudaStream_t s);

// Device error word: kernels with bounded waits set bits here when a wait gives up.  It is read (and
// cleared) at the synchronisation points the API already has (g2v_forward_prepare, g2v_backward_plan)
// and by g2v_device_error().
__device__ int g_device_error_word = 0;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_err_mu;
int* g_err_ptr[kMaxDevices] = {nullptr};

int device_error_ptr(int** out) {
    int dev = 0;
    G2V_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("device ordinal %d out of range", dev);
        return G2V_ERROR_NOT_SUPPORTED;
    }
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err_ptr[dev]) {
        void* p = nullptr;
        G2V_CUDA(cudaGetSymbolAddress(&p, g_device_error_word));
        g_err_ptr[dev] = static_cast<int*>(p);
    }
    *out = g_err_ptr[dev];
    return 0;
}

}  // namespace

// Reads the error word with the caller's stream (the caller synchronises), queued before the sync.
int queue_error_read(cudaStream_t s, int* host_word) {
    int* p = nullptr;
    int rc = device_error_ptr(&p);
    if (rc) return rc;
    G2V_CUDA(cudaMemcpyAsync(host_word, p, sizeof(int), cudaMemcpyDeviceToHost, s));
    return 0;
}

int report_device_error(int word, cudaStream_t s) {
    if (word == 0) return 0;
    int* p = nullptr;
    if (device_error_ptr(&p) == 0) cudaMemsetAsync(p, 0, sizeof(int), s);
    if (word & kErrCapacity)
        set_error("a capacity-capped call needed more pairs than its capacity (device error word 0x%x); results "
                  "of the preceding calls are invalid", word);
    else
        set_error("a kernel's bounded wait gave up (device error word 0x%x); results of the preceding calls are "
                  "invalid", word);
    return G2V_ERROR_CUDA;
}

// Kernel variant: the tensor-core path unless G2V_VARIANT=simt.
static bool use_tensor_cores() {
    const char* v = getenv("G2V_VARIANT");
    return !(v && strcmp(v, "simt") == 0);
}

int make_grid(const float size[3], const float range[6], Grid& G) {
    if (!size || !range) {
        set_error("voxel_size / voxel_range must not be NULL");
        return G2V_ERROR_INVALID_VALUE;
    }
    for (int a = 0; a < 3; ++a) {
        // float32 host arithmetic, as src/cuda_gaussian_voxelizer.cu:1512-1514
        const float q = (range[3 + a] - range[a]) / size[a];
        if (!(q >= 1.0f) || !(q < 1073741824.0f)) {
            set_error("invalid voxel grid along axis %d: (%g - %g) / %g", a, (double)range[3 + a], (double)range[a],
                      (double)size[a]);
            return G2V_ERROR_INVALID_VALUE;
        }
        G.r0[a] = range[a];
        G.r1[a] = range[3 + a];
        G.h[a] = size[a];
        G.dims[a] = static_cast<int>(q);
        G.tiles[a] = (G.dims[a] + kTile - 1) / kTile;
    }
    G.xoff = 0;
    G.xlen = G.dims[0];
    G.scene_x = 0;
    const int64_t ntiles = (int64_t)G.tiles[0] * G.tiles[1] * G.tiles[2];
    const int64_t nvox = (int64_t)G.dims[0] * G.dims[1] * G.dims[2];
    if (ntiles > INT32_MAX / 2 || nvox > ((int64_t)1 << 40)) {
        set_error("voxel grid %dx%dx%d is too large", G.dims[0], G.dims[1], G.dims[2]);
        return G2V_ERROR_SIZE_LIMIT;
    }
    return 0;
}

void clear_error() { g_msg[0] = 0; }

namespace {

// A batch of num_scenes scenes of the same grid stacked along x: scene b occupies voxel x rows
// [b X, (b+1) X) of the volume arrays, i.e. the arrays are (B, X, Y, Z[, C]).  Tiles must not straddle
// scenes, so X must be a multiple of the tile edge.
int stack_scenes(Grid& G, int num_scenes) {
    if (num_scenes < 1) {
        set_error("num_scenes must be >= 1, got %d", num_scenes);
        return G2V_ERROR_INVALID_VALUE;
    }
    if (num_scenes == 1) return 0;
    if (G.dims[0] % kTile != 0) {
        set_error("a batch of scenes needs the grid's X (%d) to be a multiple of %d", G.dims[0], kTile);
        return G2V_ERROR_NOT_SUPPORTED;
    }
    const int64_t X = (int64_t)G.dims[0] * num_scenes;
    const int64_t ntiles = (X / kTile) * G.tiles[1] * G.tiles[2];
    if (X > INT32_MAX / 2 || ntiles > INT32_MAX / 2 || X * G.dims[1] * G.dims[2] > ((int64_t)1 << 40)) {
        set_error("a batch of %d scenes of %dx%dx%d voxels is too large", num_scenes, G.dims[0], G.dims[1],
                  G.dims[2]);
        return G2V_ERROR_SIZE_LIMIT;
    }
    G.scene_x = G.dims[0];
    G.dims[0] = (int)X;
    G.tiles[0] = (int)(X / kTile);
    G.xlen = G.dims[0];
    return 0;
}

int check_slab(const Grid& G, int& tx_begin, int& tx_end) {
    if (tx_begin == 0 && tx_end == 0) tx_end = G.tiles[0];
    if (tx_begin < 0 || tx_end > G.tiles[0] || tx_begin > tx_end) {
        set_error("tile x range [%d, %d) is outside [0, %d)", tx_begin, tx_end, G.tiles[0]);
        return G2V_ERROR_INVALID_VALUE;
    }
    return 0;
}

// Slab-local volume arrays: they hold the voxel x rows of the tiles [tx_begin, tx_end) only.
void set_slab_local(Grid& G, int tx_begin, int tx_end) {
    G.xoff = tx_begin * kTile;
    G.xlen = (tx_end * kTile < G.dims[0] ? tx_end * kTile : G.dims[0]) - G.xoff;
}

// Blocks of tiles used by the feature-gradient pass: 4 x 2 x 4 by default (cfg3: a block holds ~370
// Gaussians, so its two slot passes are fuller than the 256 + ~33 of 2 x 2 x 4 blocks, and a Gaussian has
// ~40% fewer block partial rows to write and reduce; the pass time is the same).
void block_shape(const Grid& G, int B[3], int nb[3]) {
    B[0] = 4;
    B[1] = 2;
    B[2] = 4;
    if (const char* e = getenv("G2V_FPASS_BLOCK")) {
        int b[3];
        if (sscanf(e, "%d,%d,%d", &b[0], &b[1], &b[2]) == 3 && b[0] > 0 && b[1] > 0 && b[2] > 0 && b[0] * b[1] * b[2] <= 32)
            for (int a = 0; a < 3; ++a) B[a] = b[a];
    }
    B[2] = G.tiles[2] < B[2] ? G.tiles[2] : B[2];
    for (int a = 0; a < 3; ++a) nb[a] = (G.tiles[a] + B[a] - 1) / B[a];
}

struct PrepareWs {
    int32_t* ntiles;
    void* scan;
    int64_t* total;
};
size_t carve_prepare(void* p, int64_t n, PrepareWs& w) {
    Carver c(p);
    w.ntiles = c.take<int32_t>((size_t)(n > 0 ? n : 1));
    w.scan = c.take<char>(scan_workspace_bytes(n));
    w.total = c.take<int64_t>(1);
    return c.bytes();
}

// The Tile->Gaussian part comes first so that its offsets depend only on (tiles, M).
struct T2GWs {
    int32_t* tile_offsets;
    int32_t* lists;
    int32_t* unsorted;
    int32_t* counts;
    void* scan;
    int64_t* total;
};
void carve_t2g(Carver& c, int64_t ntiles, int64_t m, T2GWs& w) {
    w.tile_offsets = c.take<int32_t>((size_t)ntiles + 1);
    w.lists = c.take<int32_t>((size_t)(m > 0 ? m : 1));
    w.unsorted = c.take<int32_t>((size_t)(m > 0 ? m : 1));
    w.counts = c.take<int32_t>((size_t)(ntiles > 0 ? ntiles : 1));
    w.scan = c.take<char>(scan_workspace_bytes(ntiles));
    w.total = c.take<int64_t>(1);
}

struct BackwardWs {
    T2GWs t2g;
    int32_t* g2b_counts;
    int32_t* g2b_offsets;
    int32_t* block_offsets;
    int32_t* block_lists;
    int32_t* block_unsorted;
    int32_t* block_counts;
    void* block_scan;
    void* g_scan;
    float* partial10;
    float* partialF;
    GParams* gparams;
    void* fsplit;
    float* ev;  // e_v = sum_c gF_vc F_vc of the voxels of units with more than one slot pass
};
size_t carve_backward(void* p, int64_t n, int64_t m, int64_t mb, const Grid& G, int64_t C, BackwardWs& w) {
    Carver c(p);
    const int64_t ntiles = (int64_t)G.tiles[0] * G.tiles[1] * G.tiles[2];
    carve_t2g(c, ntiles, m, w.t2g);
    int B[3], nb[3];
    block_shape(G, B, nb);
    const int64_t nblocks = (int64_t)nb[0] * nb[1] * nb[2];
    const bool feats = C > 0;
    w.g2b_counts = c.take<int32_t>((size_t)(feats ? (n > 0 ? n : 1) : 1));
    w.g2b_offsets = c.take<int32_t>((size_t)(feats ? n + 1 : 1));
    w.block_offsets = c.take<int32_t>((size_t)(feats ? nblocks + 1 : 1));
    w.block_lists = c.take<int32_t>((size_t)(feats && mb > 0 ? mb : 1));
    w.block_unsorted = c.take<int32_t>((size_t)(feats && mb > 0 ? mb : 1));
    w.block_counts = c.take<int32_t>((size_t)(feats ? nblocks : 1));
    w.block_scan = c.take<char>(scan_workspace_bytes(feats ? nblocks : 1));
    w.g_scan = c.take<char>(scan_workspace_bytes(feats ? n : 1));
    w.partial10 = c.take<float>((size_t)(m > 0 ? m : 1) * 10);
    w.partialF = c.take<float>((size_t)(feats && mb > 0 ? mb : 1) * (size_t)(feats ? C : 1));
    w.gparams = c.take<GParams>((size_t)(n > 0 ? n : 1));
    w.fsplit = c.take<char>(feats ? spass_tc_split_bytes(n, C) : 1);
    w.ev = c.take<float>(feats ? (size_t)G.dims[0] * G.dims[1] * G.dims[2] : 1);
    return c.bytes();
}

struct PlanWs {
    int32_t* counts;
    int32_t* offsets;
    int32_t* dummy;
    void* scan;
    int64_t* total;
};
size_t carve_plan(void* p, int64_t n, PlanWs& w) {
    Carver c(p);
    w.counts = c.take<int32_t>((size_t)(n > 0 ? n : 1));
    w.offsets = c.take<int32_t>((size_t)n + 1);
    w.dummy = c.take<int32_t>(1);
    w.scan = c.take<char>(scan_workspace_bytes(n));
    w.total = c.take<int64_t>(1);
    return c.bytes();
}

int need_ws(size_t need, size_t have, const void* ws) {
    if (have < need || (need > 0 && ws == nullptr)) {
        set_error("workspace of %zu bytes is smaller than the %zu bytes required", have, need);
        return G2V_ERROR_WORKSPACE_TOO_SMALL;
    }
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
        set_error("workspace must be 256-byte aligned");
        return G2V_ERROR_INVALID_VALUE;
    }
    return 0;
}

}  // namespace
}  // namespace g2v

using namespace g2v;

extern "C" {

int g2v_abi_version(void) { return G2V_ABI_VERSION; }

const char* g2v_status_string(int status) {
    switch (status) {
        case G2V_SUCCESS: return "G2V_SUCCESS";
        case G2V_ERROR_INVALID_VALUE: return "G2V_ERROR_INVALID_VALUE";
        case G2V_ERROR_WORKSPACE_TOO_SMALL: return "G2V_ERROR_WORKSPACE_TOO_SMALL";
        case G2V_ERROR_SIZE_LIMIT: return "G2V_ERROR_SIZE_LIMIT";
        case G2V_ERROR_CUDA: return "G2V_ERROR_CUDA";
        case G2V_ERROR_NOT_SUPPORTED: return "G2V_ERROR_NOT_SUPPORTED";
        default: return "G2V_UNKNOWN_STATUS";
    }
}

const char* g2v_last_error(void) { return g_msg; }

int g2v_grid_shape(const float voxel_size[3], const float voxel_range[6], int dims[3], int tiles[3]) {
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    for (int a = 0; a < 3; ++a) {
        if (dims) dims[a] = G.dims[a];
        if (tiles) tiles[a] = G.tiles[a];
    }
    return G2V_SUCCESS;
}

int g2v_forward_prepare_workspace_size(int64_t num_gaussians, size_t* bytes) {
    if (!bytes || num_gaussians < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    PrepareWs w;
    *bytes = carve_prepare(nullptr, num_gaussians, w);
    return G2V_SUCCESS;
}

int g2v_forward_prepare(const float* means3d, const float* covariances, int64_t num_gaussians,
                        const float voxel_size[3], const float voxel_range[6], float* cov_inv,
                        int32_t* valid_voxel_lb, int32_t* valid_voxel_ub, int32_t* num_voxels,
                        int32_t* g2t_offsets, void* workspace, size_t workspace_bytes, void* stream,
                        int64_t* num_pairs) {
    g_msg[0] = 0;
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if (num_gaussians < 0 || num_gaussians > INT32_MAX - 1 || !g2t_offsets || !num_pairs ||
        (num_gaussians > 0 && (!means3d || !covariances || !cov_inv || !valid_voxel_lb || !valid_voxel_ub ||
                               !num_voxels))) {
        set_error("g2v_forward_prepare: invalid pointer or Gaussian count");
        return G2V_ERROR_INVALID_VALUE;
    }
    PrepareWs w;
    const size_t need = carve_prepare(nullptr, num_gaussians, w);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    carve_prepare(workspace, num_gaussians, w);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((rc = launch_prepare_boxes(means3d, covariances, num_gaussians, G, cov_inv, valid_voxel_lb, valid_voxel_ub,
                                   num_voxels, w.ntiles, s)))
        return rc;
    if ((rc = launch_exclusive_scan(w.ntiles, num_gaussians, g2t_offsets, w.total, w.scan, s))) return rc;
    int64_t m = 0;
    int word = 0;
    G2V_CUDA(cudaMemcpyAsync(&m, w.total, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
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

int g2v_forward_prepare_capped(const float* means3d, const float* covariances, int64_t num_gaussians,
                               const float voxel_size[3], const float voxel_range[6], int64_t max_pairs,
                               float* cov_inv, int32_t* valid_voxel_lb, int32_t* valid_voxel_ub,
                               int32_t* num_voxels, int32_t* g2t_offsets, void* workspace, size_t workspace_bytes,
                               void* stream) {
    g_msg[0] = 0;
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if (num_gaussians < 0 || num_gaussians > INT32_MAX - 1 || max_pairs < 0 || max_pairs > INT32_MAX ||
        !g2t_offsets ||
        (num_gaussians > 0 && (!means3d || !covariances || !cov_inv || !valid_voxel_lb || !valid_voxel_ub ||
                               !num_voxels))) {
        set_error("g2v_forward_prepare_capped: invalid pointer, count or capacity");
        return G2V_ERROR_INVALID_VALUE;
    }
    PrepareWs w;
    const size_t need = carve_prepare(nullptr, num_gaussians, w);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    carve_prepare(workspace, num_gaussians, w);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* err = nullptr;
    if ((rc = device_error_ptr(&err))) return rc;
    if ((rc = launch_prepare_boxes(means3d, covariances, num_gaussians, G, cov_inv, valid_voxel_lb, valid_voxel_ub,
                                   num_voxels, w.ntiles, s)))
        return rc;
    return launch_exclusive_scan(w.ntiles, num_gaussians, g2t_offsets, w.total, w.scan, s, max_pairs, err);
}

int g2v_forward_splat_workspace_size(int64_t num_gaussians, int64_t num_pairs, const int dims[3],
                                     int64_t channels, size_t* bytes) {
    if (!bytes || !dims || num_gaussians < 0 || num_pairs < 0 || channels < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    const int64_t ntiles = (int64_t)((dims[0] + 3) / 4) * ((dims[1] + 3) / 4) * ((dims[2] + 3) / 4);
    Carver c(nullptr);
    T2GWs w, wu;
    carve_t2g(c, ntiles, num_pairs, w);
    carve_t2g(c, ntiles, num_pairs, wu);  // the tensor-core path's unit lists (z quads of tiles)
    c.take<char>(splat_tc_split_bytes(num_gaussians, channels));
    *bytes = c.bytes();
    return G2V_SUCCESS;
}

static int forward_splat_impl(const float* means3d, const float* opacity, const float* features,
                              int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                              const float voxel_range[6], const float* cov_inv, const int32_t* valid_voxel_lb,
                              const int32_t* valid_voxel_ub, const int32_t* g2t_offsets, int64_t num_pairs,
                              int32_t* g2t_tile_ids, float* density, float* grid_feats, int tile_x_begin,
                              int tile_x_end, void* workspace, size_t workspace_bytes, void* stream, bool local,
                              int num_scenes = 1) {
    g_msg[0] = 0;
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if ((rc = stack_scenes(G, num_scenes))) return rc;
    if ((rc = check_slab(G, tile_x_begin, tile_x_end))) return rc;
    if (local) set_slab_local(G, tile_x_begin, tile_x_end);
    const int C = features ? (int)channels : 0;
    if (num_gaussians < 0 || num_pairs < 0 || channels < 0 || channels > INT32_MAX / 2 || !density ||
        !g2t_offsets || (num_pairs > 0 && !g2t_tile_ids) || (features && channels > 0 && !grid_feats) ||
        (num_gaussians > 0 && (!means3d || !opacity || !cov_inv || !valid_voxel_lb || !valid_voxel_ub))) {
        set_error("g2v_forward_splat: invalid pointer or size");
        return G2V_ERROR_INVALID_VALUE;
    }
    size_t need = 0;
    g2v_forward_splat_workspace_size(num_gaussians, num_pairs, G.dims, channels, &need);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    Carver c(workspace);
    T2GWs w, wu;
    const int64_t ntiles_all = (int64_t)G.tiles[0] * G.tiles[1] * G.tiles[2];
    carve_t2g(c, ntiles_all, num_pairs, w);
    carve_t2g(c, ntiles_all, num_pairs, wu);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* err = nullptr;
    if ((rc = device_error_ptr(&err))) return rc;
    const int one[3] = {1, 1, 1};
    const bool tcore = features != nullptr && C > 0 && use_tensor_cores();
    // the reference's G2T tile ids; the per-tile Gaussian lists only for the FP32-FMA splat (the
    // tensor-core splat lists z quads of tiles; g2v_build_t2g builds the per-tile map on request)
    if (tcore) {
        if ((rc = fill_g2t(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, g2t_offsets, g2t_tile_ids, num_pairs, s)))
            return rc;
    } else if ((rc = build_cell_lists(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, one, G.tiles, tile_x_begin,
                                      tile_x_end, g2t_offsets, g2t_tile_ids, num_pairs, nullptr, w.counts,
                                      w.tile_offsets, w.unsorted, w.lists, w.scan, w.total, s, num_pairs, err))) {
        return rc;
    }
    const int first_tile = tile_x_begin * G.tiles[1] * G.tiles[2];
    const int nt = (tile_x_end - tile_x_begin) * G.tiles[1] * G.tiles[2];
    if (tcore) {
        // unit lists: z quads of tiles, Gaussian ids ascending (at most M entries over fewer cells)
        int cell[3], ncells[3];
        tc_unit_shape(G, cell, ncells);
        if ((rc = build_cell_lists(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, cell, ncells, tile_x_begin,
                                   tile_x_end, g2t_offsets, nullptr, 0, nullptr, wu.counts, wu.tile_offsets,
                                   wu.unsorted, wu.lists, wu.scan, wu.total, s, num_pairs, err)))
            return rc;
        void* split = c.take<char>(splat_tc_split_bytes(num_gaussians, C));
        return launch_splat_tc(means3d, opacity, cov_inv, valid_voxel_lb, valid_voxel_ub, features, num_gaussians, C,
                               wu.tile_offsets, wu.lists, tile_x_begin, tile_x_end, G, density, grid_feats, split,
                               err, s);
    }
    return launch_splat_simt(means3d, opacity, cov_inv, valid_voxel_lb, valid_voxel_ub, features, C, w.tile_offsets,
                             w.lists, first_tile, nt, G, density, grid_feats, s);
}

int g2v_forward_splat(const float* means3d, const float* opacity, const float* features, int64_t num_gaussians,
                      int64_t channels, const float voxel_size[3], const float voxel_range[6],
                      const float* cov_inv, const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub,
                      const int32_t* g2t_offsets, int64_t num_pairs, int32_t* g2t_tile_ids, float* density,
                      float* grid_feats, int tile_x_begin, int tile_x_end, void* workspace,
                      size_t workspace_bytes, void* stream) {
    return forward_splat_impl(means3d, opacity, features, num_gaussians, channels, voxel_size, voxel_range, cov_inv,
                              valid_voxel_lb, valid_voxel_ub, g2t_offsets, num_pairs, g2t_tile_ids, density,
                              grid_feats, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream, false);
}

int g2v_forward_splat_local(const float* means3d, const float* opacity, const float* features,
                            int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                            const float voxel_range[6], const float* cov_inv, const int32_t* valid_voxel_lb,
                            const int32_t* valid_voxel_ub, const int32_t* g2t_offsets, int64_t num_pairs,
                            int32_t* g2t_tile_ids, float* density, float* grid_feats, int tile_x_begin,
                            int tile_x_end, void* workspace, size_t workspace_bytes, void* stream) {
    return forward_splat_impl(means3d, opacity, features, num_gaussians, channels, voxel_size, voxel_range, cov_inv,
                              valid_voxel_lb, valid_voxel_ub, g2t_offsets, num_pairs, g2t_tile_ids, density,
                              grid_feats, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream, true);
}

int g2v_build_t2g_workspace_size(int64_t num_gaussians, int64_t num_pairs, const int dims[3], size_t* bytes) {
    if (!bytes || !dims || num_gaussians < 0 || num_pairs < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    const int64_t ntiles = (int64_t)((dims[0] + 3) / 4) * ((dims[1] + 3) / 4) * ((dims[2] + 3) / 4);
    Carver c(nullptr);
    T2GWs w;
    carve_t2g(c, ntiles, num_pairs, w);
    *bytes = c.bytes();
    return G2V_SUCCESS;
}

int g2v_forward_splat_unit_lists(const void* splat_workspace, int64_t num_gaussians, int64_t num_pairs,
                                 const int dims[3], int64_t channels, int32_t* unit_offsets, int32_t* unit_lists,
                                 int64_t* num_units, void* stream) {
    g_msg[0] = 0;
    (void)num_gaussians;
    if (!dims || !num_units || num_pairs < 0) {
        set_error("g2v_forward_splat_unit_lists: invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    if (channels <= 0 || !use_tensor_cores()) {
        set_error("g2v_forward_splat_unit_lists: the splat built no unit lists (no features, or the FP32-FMA variant)");
        return G2V_ERROR_INVALID_VALUE;
    }
    Grid G{};
    for (int a = 0; a < 3; ++a) {
        G.dims[a] = dims[a];
        G.tiles[a] = (dims[a] + 3) / 4;
    }
    int cell[3], ncells[3];
    tc_unit_shape(G, cell, ncells);
    const int64_t nu = (int64_t)ncells[0] * ncells[1] * ncells[2];
    *num_units = nu;
    if (!unit_offsets) return G2V_SUCCESS;  // size query
    if (!splat_workspace || (num_pairs > 0 && !unit_lists)) {
        set_error("g2v_forward_splat_unit_lists: invalid pointer");
        return G2V_ERROR_INVALID_VALUE;
    }
    // the splat workspace holds the tile lists, then the unit lists (g2v_forward_splat)
    const int64_t ntiles = (int64_t)G.tiles[0] * G.tiles[1] * G.tiles[2];
    Carver c(const_cast<void*>(splat_workspace));
    T2GWs w, wu;
    carve_t2g(c, ntiles, num_pairs, w);
    carve_t2g(c, ntiles, num_pairs, wu);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    G2V_CUDA(cudaMemcpyAsync(unit_offsets, wu.tile_offsets, sizeof(int32_t) * (size_t)(nu + 1), cudaMemcpyDeviceToDevice,
                             s));
    if (num_pairs > 0)
        G2V_CUDA(cudaMemcpyAsync(unit_lists, wu.lists, sizeof(int32_t) * (size_t)num_pairs, cudaMemcpyDeviceToDevice,
                                 s));
    return G2V_SUCCESS;
}

int g2v_build_t2g(const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, int64_t num_gaussians,
                  const float voxel_size[3], const float voxel_range[6], int64_t num_pairs, int32_t* tile_offsets,
                  int32_t* t2g_gaussians, void* workspace, size_t workspace_bytes, void* stream) {
    g_msg[0] = 0;
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if (num_gaussians < 0 || num_pairs < 0 || !tile_offsets || (num_pairs > 0 && !t2g_gaussians) ||
        (num_gaussians > 0 && (!valid_voxel_lb || !valid_voxel_ub))) {
        set_error("g2v_build_t2g: invalid pointer or size");
        return G2V_ERROR_INVALID_VALUE;
    }
    size_t need = 0;
    g2v_build_t2g_workspace_size(num_gaussians, num_pairs, G.dims, &need);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    Carver c(workspace);
    T2GWs w;
    const int64_t ntiles = (int64_t)G.tiles[0] * G.tiles[1] * G.tiles[2];
    carve_t2g(c, ntiles, num_pairs, w);
    int* err = nullptr;
    if ((rc = device_error_ptr(&err))) return rc;
    const int one[3] = {1, 1, 1};
    return build_cell_lists(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, one, G.tiles, 0, G.tiles[0], nullptr,
                            nullptr, 0, nullptr, w.counts, tile_offsets, w.unsorted, t2g_gaussians, w.scan, w.total,
                            static_cast<cudaStream_t>(stream), num_pairs, err);
}

int g2v_debug_wait_timeout(void* stream, int* gave_up) {
    g_msg[0] = 0;
    if (!gave_up) {
        set_error("gave_up must not be NULL");
        return G2V_ERROR_INVALID_VALUE;
    }
    int* err = nullptr;
    int rc = device_error_ptr(&err);
    if (rc) return rc;
    return launch_wait_timeout(err, static_cast<cudaStream_t>(stream), gave_up);
}

int g2v_device_error(void* stream, int* word) {
    if (!word) {
        set_error("word must not be NULL");
        return G2V_ERROR_INVALID_VALUE;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc = queue_error_read(s, word);
    if (rc) return rc;
    G2V_CUDA(cudaStreamSynchronize(s));
    if (*word) {
        int* p = nullptr;
        if (device_error_ptr(&p) == 0) G2V_CUDA(cudaMemsetAsync(p, 0, sizeof(int), s));
    }
    return G2V_SUCCESS;
}

int g2v_backward_plan_workspace_size(int64_t num_gaussians, size_t* bytes) {
    if (!bytes || num_gaussians < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    PlanWs w;
    *bytes = carve_plan(nullptr, num_gaussians, w);
    return G2V_SUCCESS;
}

int g2v_backward_plan(const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, int64_t num_gaussians,
                      const int dims[3], int64_t channels, void* workspace, size_t workspace_bytes, void* stream,
                      int64_t* num_block_pairs) {
    g_msg[0] = 0;
    if (!dims || !num_block_pairs || num_gaussians < 0 || channels < 0 ||
        (num_gaussians > 0 && (!valid_voxel_lb || !valid_voxel_ub))) {
        set_error("g2v_backward_plan: invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    if (channels == 0 || num_gaussians == 0) {
        *num_block_pairs = 0;
        return G2V_SUCCESS;
    }
    Grid G{};
    for (int a = 0; a < 3; ++a) {
        G.dims[a] = dims[a];
        G.tiles[a] = (dims[a] + 3) / 4;
    }
    PlanWs w;
    int rc;
    const size_t need = carve_plan(nullptr, num_gaussians, w);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    carve_plan(workspace, num_gaussians, w);
    int B[3], nb[3];
    block_shape(G, B, nb);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((rc = count_gaussian_cells(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, B, w.counts, w.dummy, s)))
        return rc;
    if ((rc = launch_exclusive_scan(w.counts, num_gaussians, w.offsets, w.total, w.scan, s))) return rc;
    int64_t mb = 0;
    int word = 0;
    G2V_CUDA(cudaMemcpyAsync(&mb, w.total, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    if ((rc = queue_error_read(s, &word))) return rc;
    G2V_CUDA(cudaStreamSynchronize(s));
    if ((rc = report_device_error(word, s))) return rc;
    if (mb > INT32_MAX) {
        set_error("%lld (Gaussian, block) pairs exceed the int32 range", (long long)mb);
        return G2V_ERROR_SIZE_LIMIT;
    }
    *num_block_pairs = mb;
    return G2V_SUCCESS;
}

int g2v_forward_prepare_plan_workspace_size(int64_t num_gaussians, size_t* bytes) {
    if (!bytes || num_gaussians < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    Carver c(nullptr);
    PrepareWs wp;
    PlanWs wb;
    c.take<char>(carve_prepare(nullptr, num_gaussians, wp));
    c.take<char>(carve_plan(nullptr, num_gaussians, wb));
    *bytes = c.bytes();
    return G2V_SUCCESS;
}

}  // extern "C"

// covariances, or (scales, rotations) when scales is non-NULL
static int prepare_plan_impl(const float* means3d, const float* covariances, const float* scales,
                             const float* rotations, int64_t num_gaussians, const float voxel_size[3],
                             const float voxel_range[6], float* cov_inv, int32_t* valid_voxel_lb,
                             int32_t* valid_voxel_ub, int32_t* num_voxels, int32_t* g2t_offsets, int64_t channels,
                             void* workspace, size_t workspace_bytes, void* stream, int64_t* num_pairs,
                             int64_t* num_block_pairs, const int32_t* scene_offsets = nullptr,
                             int num_scenes = 1) {
    g_msg[0] = 0;
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if ((rc = stack_scenes(G, num_scenes))) return rc;
    if (num_scenes > 1 && !scene_offsets) {
        set_error("g2v_forward_prepare_plan_batched: scene_offsets is required for %d scenes", num_scenes);
        return G2V_ERROR_INVALID_VALUE;
    }
    const bool have_cov = scales ? rotations != nullptr : covariances != nullptr;
    if (num_gaussians < 0 || num_gaussians > INT32_MAX - 1 || channels < 0 || !g2t_offsets || !num_pairs ||
        !num_block_pairs ||
        (num_gaussians > 0 && (!means3d || !have_cov || !cov_inv || !valid_voxel_lb || !valid_voxel_ub ||
                               !num_voxels))) {
        set_error("g2v_forward_prepare_plan: invalid pointer or count");
        return G2V_ERROR_INVALID_VALUE;
    }
    size_t need = 0;
    g2v_forward_prepare_plan_workspace_size(num_gaussians, &need);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    Carver c(workspace);
    PrepareWs wp;
    PlanWs wb;
    carve_prepare(c.take<char>(carve_prepare(nullptr, num_gaussians, wp)), num_gaussians, wp);
    carve_plan(c.take<char>(carve_plan(nullptr, num_gaussians, wb)), num_gaussians, wb);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((rc = launch_prepare_boxes(means3d, covariances, num_gaussians, G, cov_inv, valid_voxel_lb, valid_voxel_ub,
                                   num_voxels, wp.ntiles, s, scales, rotations, num_scenes > 1 ? scene_offsets : nullptr,
                                   num_scenes)))
        return rc;
    if ((rc = launch_exclusive_scan(wp.ntiles, num_gaussians, g2t_offsets, wp.total, wp.scan, s))) return rc;
    const bool blocks = channels > 0 && num_gaussians > 0;
    if (blocks) {
        int B[3], nb[3];
        block_shape(G, B, nb);
        if ((rc = count_gaussian_cells(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, B, wb.counts, wb.dummy, s)))
            return rc;
        if ((rc = launch_exclusive_scan(wb.counts, num_gaussians, wb.offsets, wb.total, wb.scan, s))) return rc;
    }
    int64_t m = 0, mb = 0;
    int word = 0;
    int32_t ends[2] = {0, (int32_t)num_gaussians};
    G2V_CUDA(cudaMemcpyAsync(&m, wp.total, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    if (blocks) G2V_CUDA(cudaMemcpyAsync(&mb, wb.total, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    if (num_scenes > 1) {
        G2V_CUDA(cudaMemcpyAsync(&ends[0], scene_offsets, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
        G2V_CUDA(cudaMemcpyAsync(&ends[1], scene_offsets + num_scenes, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    }
    if ((rc = queue_error_read(s, &word))) return rc;
    G2V_CUDA(cudaStreamSynchronize(s));
    if ((rc = report_device_error(word, s))) return rc;
    if (ends[0] != 0 || ends[1] != (int32_t)num_gaussians) {
        set_error("scene_offsets must run from 0 to num_gaussians (%lld), got %d .. %d", (long long)num_gaussians,
                  ends[0], ends[1]);
        return G2V_ERROR_INVALID_VALUE;
    }
    if (m > INT32_MAX || mb > INT32_MAX) {
        set_error("%lld tile pairs / %lld block pairs exceed the int32 range of the CSR maps", (long long)m,
                  (long long)mb);
        return G2V_ERROR_SIZE_LIMIT;
    }
    *num_pairs = m;
    *num_block_pairs = mb;
    return G2V_SUCCESS;
}

extern "C" {

int g2v_forward_prepare_plan(const float* means3d, const float* covariances, int64_t num_gaussians,
                             const float voxel_size[3], const float voxel_range[6], float* cov_inv,
                             int32_t* valid_voxel_lb, int32_t* valid_voxel_ub, int32_t* num_voxels,
                             int32_t* g2t_offsets, int64_t channels, void* workspace, size_t workspace_bytes,
                             void* stream, int64_t* num_pairs, int64_t* num_block_pairs) {
    return prepare_plan_impl(means3d, covariances, nullptr, nullptr, num_gaussians, voxel_size, voxel_range, cov_inv,
                             valid_voxel_lb, valid_voxel_ub, num_voxels, g2t_offsets, channels, workspace,
                             workspace_bytes, stream, num_pairs, num_block_pairs);
}

int g2v_forward_prepare_plan_sr(const float* means3d, const float* scales, const float* rotations,
                                int64_t num_gaussians, const float voxel_size[3], const float voxel_range[6],
                                float* cov_inv, int32_t* valid_voxel_lb, int32_t* valid_voxel_ub,
                                int32_t* num_voxels, int32_t* g2t_offsets, int64_t channels, void* workspace,
                                size_t workspace_bytes, void* stream, int64_t* num_pairs, int64_t* num_block_pairs) {
    if (num_gaussians > 0 && (!scales || !rotations)) {
        g_msg[0] = 0;
        set_error("g2v_forward_prepare_plan_sr: scales and rotations are required");
        return G2V_ERROR_INVALID_VALUE;
    }
    static const float kDummy = 0.f;  // non-NULL marker for the empty case
    return prepare_plan_impl(means3d, nullptr, scales ? scales : &kDummy, rotations ? rotations : &kDummy,
                             num_gaussians, voxel_size, voxel_range, cov_inv, valid_voxel_lb, valid_voxel_ub,
                             num_voxels, g2t_offsets, channels, workspace, workspace_bytes, stream, num_pairs,
                             num_block_pairs);
}

int g2v_forward_prepare_plan_batched(const float* means3d, const float* covariances, const float* scales,
                                     const float* rotations, const int32_t* scene_offsets, int num_scenes,
                                     int64_t num_gaussians, const float voxel_size[3], const float voxel_range[6],
                                     float* cov_inv, int32_t* valid_voxel_lb, int32_t* valid_voxel_ub,
                                     int32_t* num_voxels, int32_t* g2t_offsets, int64_t channels, void* workspace,
                                     size_t workspace_bytes, void* stream, int64_t* num_pairs,
                                     int64_t* num_block_pairs) {
    if (num_gaussians > 0 && (scales ? !rotations : !covariances)) {
        g_msg[0] = 0;
        set_error("g2v_forward_prepare_plan_batched: covariances, or scales and rotations, are required");
        return G2V_ERROR_INVALID_VALUE;
    }
    static const float kDummy = 0.f;  // non-NULL marker for the empty case
    const float* sc = scales ? scales : nullptr;
    const float* cv = scales ? nullptr : (covariances ? covariances : &kDummy);
    return prepare_plan_impl(means3d, cv, sc, scales ? rotations : nullptr, num_gaussians, voxel_size, voxel_range,
                             cov_inv, valid_voxel_lb, valid_voxel_ub, num_voxels, g2t_offsets, channels, workspace,
                             workspace_bytes, stream, num_pairs, num_block_pairs, scene_offsets, num_scenes);
}

int g2v_covariance_from_scale_rot(const float* scales, const float* rotations, int64_t num_gaussians,
                                  float* covariances, void* stream) {
    g_msg[0] = 0;
    if (num_gaussians < 0 || (num_gaussians > 0 && (!scales || !rotations || !covariances))) {
        set_error("g2v_covariance_from_scale_rot: invalid pointer or count");
        return G2V_ERROR_INVALID_VALUE;
    }
    return launch_cov_from_scale_rot(scales, rotations, num_gaussians, covariances,
                                     static_cast<cudaStream_t>(stream));
}

int g2v_covariance_from_scale_rot_backward(const float* scales, const float* rotations,
                                           const float* grad_covariances, int64_t num_gaussians, float* grad_scales,
                                           float* grad_rotations, void* stream) {
    g_msg[0] = 0;
    if (num_gaussians < 0 ||
        (num_gaussians > 0 && (!scales || !rotations || !grad_covariances || !grad_scales || !grad_rotations))) {
        set_error("g2v_covariance_from_scale_rot_backward: invalid pointer or count");
        return G2V_ERROR_INVALID_VALUE;
    }
    return launch_cov_from_scale_rot_backward(scales, rotations, grad_covariances, num_gaussians, grad_scales,
                                              grad_rotations, static_cast<cudaStream_t>(stream));
}

int g2v_backward_workspace_size(int64_t num_gaussians, int64_t num_pairs, int64_t num_block_pairs,
                                const int dims[3], int64_t channels, size_t* bytes) {
    if (!bytes || !dims || num_gaussians < 0 || num_pairs < 0 || num_block_pairs < 0 || channels < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    Grid G{};
    for (int a = 0; a < 3; ++a) {
        G.dims[a] = dims[a];
        G.tiles[a] = (dims[a] + 3) / 4;
    }
    BackwardWs w;
    *bytes = carve_backward(nullptr, num_gaussians, num_pairs, num_block_pairs, G, channels, w);
    return G2V_SUCCESS;
}

static int backward_impl(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                         const float* opacity, const float* cov_inv, const float* features, int64_t num_gaussians,
                         int64_t channels, const float voxel_size[3], const float voxel_range[6], const int dims[3],
                         const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                         const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                         const float* density, const float* grid_feats, float* grad_means3d,
                         float* grad_covariances, float* grad_opacity, float* grad_features, int tile_x_begin,
                         int tile_x_end, void* workspace, size_t workspace_bytes, void* stream, bool local,
                         const float* scales = nullptr, const float* rotations = nullptr,
                         float* grad_rotations = nullptr, int num_scenes = 1,
                         const int32_t* unit_offsets_in = nullptr, const int32_t* unit_lists_in = nullptr) {
    g_msg[0] = 0;
    Grid G;
    int rc = make_grid(voxel_size, voxel_range, G);
    if (rc) return rc;
    if ((rc = stack_scenes(G, num_scenes))) return rc;
    if (!dims || dims[0] != G.dims[0] || dims[1] != G.dims[1] || dims[2] != G.dims[2]) {
        set_error("g2v_backward: dims do not match the voxel grid %dx%dx%d", G.dims[0], G.dims[1], G.dims[2]);
        return G2V_ERROR_INVALID_VALUE;
    }
    if ((rc = check_slab(G, tile_x_begin, tile_x_end))) return rc;
    if (local) set_slab_local(G, tile_x_begin, tile_x_end);
    const int C = features ? (int)channels : 0;
    if (num_gaussians < 0 || num_pairs < 0 || channels < 0 || channels > INT32_MAX / 2 || num_block_pairs < 0 ||
        !grad_density || !density || !g2t_offsets || (num_pairs > 0 && !g2t_tile_ids) ||
        (C > 0 && !grad_grid_feats) || (C > 0 && num_gaussians > 0 && !grad_features) ||
        (num_gaussians > 0 && (!means3d || !opacity || !cov_inv || !valid_voxel_lb || !valid_voxel_ub ||
                               !grad_means3d || !grad_covariances || !grad_opacity)) ||
        (num_gaussians > 0 && scales && (!rotations || !grad_rotations))) {
        set_error("g2v_backward: invalid pointer or size");
        return G2V_ERROR_INVALID_VALUE;
    }
    BackwardWs w;
    const size_t need = carve_backward(nullptr, num_gaussians, num_pairs, num_block_pairs, G, C, w);
    if ((rc = need_ws(need, workspace_bytes, workspace))) return rc;
    carve_backward(workspace, num_gaussians, num_pairs, num_block_pairs, G, C, w);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tcore = C > 0 && num_gaussians > 0 && use_tensor_cores();
    // Tile->Gaussian lists for the FP32-FMA tile pass, or the lists of the tensor-core pass's units
    // (z quads of tiles); both fit the tile-sized buffers (fewer cells, at most M entries)
    int cell[3] = {1, 1, 1}, ncells[3] = {G.tiles[0], G.tiles[1], G.tiles[2]};
    if (tcore) tc_unit_shape(G, cell, ncells);
    int* err = nullptr;
    if ((rc = device_error_ptr(&err))) return rc;
    // the tile pass's unit lists: given by the caller (the forward splat built the same ones) or built here
    const bool given_units = tcore && unit_offsets_in != nullptr && unit_lists_in != nullptr;
    const int32_t* unit_offsets = given_units ? unit_offsets_in : w.t2g.tile_offsets;
    const int32_t* unit_lists = given_units ? unit_lists_in : w.t2g.lists;
    if (!given_units &&
        (rc = build_cell_lists(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, cell, ncells, tile_x_begin,
                               tile_x_end, g2t_offsets, nullptr, 0, nullptr, w.t2g.counts, w.t2g.tile_offsets,
                               w.t2g.unsorted, w.t2g.lists, w.t2g.scan, w.t2g.total, s, num_pairs, err)))
        return rc;
    const int first_tile = tile_x_begin * G.tiles[1] * G.tiles[2];
    const int nt = (tile_x_end - tile_x_begin) * G.tiles[1] * G.tiles[2];
    if (tcore) {
        if ((rc = launch_pack_params(means3d, opacity, cov_inv, valid_voxel_lb, valid_voxel_ub, num_gaussians,
                                     w.gparams, s)))
            return rc;
        if ((rc = launch_spass_tc(grad_density, grad_grid_feats, features, num_gaussians, C, density, w.gparams,
                                  g2t_offsets, unit_offsets, unit_lists, tile_x_begin, tile_x_end, G,
                                  w.partial10, num_pairs, w.fsplit, err, s, grid_feats, w.ev)))
            return rc;
    } else if ((rc = launch_spass(grad_density, grad_grid_feats, means3d, opacity, cov_inv, valid_voxel_lb,
                                  valid_voxel_ub, features, C, density, g2t_offsets, w.t2g.tile_offsets, w.t2g.lists,
                                  first_tile, nt, G, w.partial10, num_pairs, s))) {
        return rc;
    }
    if ((rc = launch_reduce10(w.partial10, g2t_offsets, g2t_tile_ids, num_gaussians, G, tile_x_begin, tile_x_end,
                              grad_means3d, grad_covariances, grad_opacity, s, scales, rotations, grad_rotations)))
        return rc;
    if (C > 0 && num_gaussians > 0) {
        int B[3], nb[3];
        block_shape(G, B, nb);
        const int bx_begin = tile_x_begin / B[0];
        const int bx_end = (tile_x_end + B[0] - 1) / B[0];
        int64_t* total = w.t2g.total;
        // per-Gaussian block counts, then the offsets of the partial rows
        if ((rc = build_cell_lists(valid_voxel_lb, valid_voxel_ub, num_gaussians, G, B, nb, bx_begin, bx_end,
                                   nullptr, nullptr, 0, w.g2b_counts, w.block_counts, w.block_offsets,
                                   w.block_unsorted, w.block_lists, w.block_scan, total, s, num_block_pairs, err,
                                   /*x_order: the tensor-core pass skips the steps outside a slot range's boxes*/ tcore)))
            return rc;
        if ((rc = launch_exclusive_scan(w.g2b_counts, num_gaussians, w.g2b_offsets, total, w.g_scan, s,
                                        num_block_pairs, err)))
            return rc;
        if (tcore) {
            if ((rc = launch_fpass_tc(grad_grid_feats, C, density, w.gparams, w.block_offsets, w.block_lists,
                                      w.g2b_offsets, bx_begin, bx_end - bx_begin, nb[1], nb[2], B, tile_x_begin,
                                      tile_x_end, G, w.partialF, num_block_pairs, err, s)))
                return rc;
        } else if ((rc = launch_fpass(grad_grid_feats, means3d, opacity, cov_inv, valid_voxel_lb, valid_voxel_ub, C,
                                      density, w.block_offsets, w.block_lists, w.g2b_offsets, bx_begin,
                                      bx_end - bx_begin, nb[1], nb[2], B, tile_x_begin, tile_x_end, G, w.partialF,
                                      num_block_pairs, s))) {
            return rc;
        }
        if ((rc = launch_reduce_feats(w.partialF, w.g2b_offsets, valid_voxel_lb, valid_voxel_ub, num_gaussians, C, B,
                                      bx_begin, bx_end, grad_features, s, num_block_pairs)))
            return rc;
    }
    return G2V_SUCCESS;
}

int g2v_backward(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                 const float* opacity, const float* cov_inv, const float* features, int64_t num_gaussians,
                 int64_t channels, const float voxel_size[3], const float voxel_range[6], const int dims[3],
                 const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                 const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs, const float* density,
                 const float* grid_feats, float* grad_means3d, float* grad_covariances, float* grad_opacity,
                 float* grad_features, int tile_x_begin, int tile_x_end, void* workspace, size_t workspace_bytes,
                 void* stream) {
    return backward_impl(grad_density, grad_grid_feats, means3d, opacity, cov_inv, features, num_gaussians, channels,
                         voxel_size, voxel_range, dims, valid_voxel_lb, valid_voxel_ub, g2t_offsets, g2t_tile_ids,
                         num_pairs, num_block_pairs, density, grid_feats, grad_means3d, grad_covariances,
                         grad_opacity, grad_features, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream,
                         false);
}

int g2v_backward_units(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                       const float* opacity, const float* cov_inv, const float* features, int64_t num_gaussians,
                       int64_t channels, const float voxel_size[3], const float voxel_range[6], const int dims[3],
                       const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                       const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                       const float* density, const float* grid_feats, float* grad_means3d, float* grad_covariances,
                       float* grad_opacity, float* grad_features, const int32_t* unit_offsets,
                       const int32_t* unit_lists, void* workspace, size_t workspace_bytes, void* stream) {
    if (!unit_offsets || !unit_lists) {
        g_msg[0] = 0;
        set_error("g2v_backward_units: unit_offsets and unit_lists are required");
        return G2V_ERROR_INVALID_VALUE;
    }
    return backward_impl(grad_density, grad_grid_feats, means3d, opacity, cov_inv, features, num_gaussians, channels,
                         voxel_size, voxel_range, dims, valid_voxel_lb, valid_voxel_ub, g2t_offsets, g2t_tile_ids,
                         num_pairs, num_block_pairs, density, grid_feats, grad_means3d, grad_covariances,
                         grad_opacity, grad_features, 0, 0, workspace, workspace_bytes, stream, false, nullptr,
                         nullptr, nullptr, 1, unit_offsets, unit_lists);
}

int g2v_backward_local(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                       const float* opacity, const float* cov_inv, const float* features, int64_t num_gaussians,
                       int64_t channels, const float voxel_size[3], const float voxel_range[6], const int dims[3],
                       const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                       const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                       const float* density, const float* grid_feats, float* grad_means3d, float* grad_covariances,
                       float* grad_opacity, float* grad_features, int tile_x_begin, int tile_x_end, void* workspace,
                       size_t workspace_bytes, void* stream) {
    return backward_impl(grad_density, grad_grid_feats, means3d, opacity, cov_inv, features, num_gaussians, channels,
                         voxel_size, voxel_range, dims, valid_voxel_lb, valid_voxel_ub, g2t_offsets, g2t_tile_ids,
                         num_pairs, num_block_pairs, density, grid_feats, grad_means3d, grad_covariances,
                         grad_opacity, grad_features, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream,
                         true);
}

int g2v_cosine_loss_workspace_size(int64_t num_voxels, size_t* bytes) {
    if (!bytes || num_voxels < 0) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    *bytes = cosine_loss_workspace_bytes();
    return G2V_SUCCESS;
}

int g2v_cosine_loss_forward(const float* voxel_label, const uint8_t* occ_mask, const float* grid_feats,
                            const float* gt_feats, int64_t num_voxels, int64_t channels, float* loss, int32_t* count,
                            void* workspace, size_t workspace_bytes, void* stream) {
    g_msg[0] = 0;
    if (num_voxels < 0 || channels < 0 || channels > INT32_MAX || num_voxels > INT32_MAX || !loss || !count ||
        (num_voxels > 0 && (!voxel_label || !occ_mask)) ||
        (num_voxels > 0 && channels > 0 && (!grid_feats || !gt_feats))) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    int rc = need_ws(cosine_loss_workspace_bytes(), workspace_bytes, workspace);
    if (rc) return rc;
    return launch_cosine_loss_fwd(voxel_label, occ_mask, grid_feats, gt_feats, num_voxels, (int)channels, loss,
                                  reinterpret_cast<int*>(count), workspace, static_cast<cudaStream_t>(stream));
}

int g2v_cosine_loss_backward(const float* grad_loss, const int32_t* count, int32_t count_host,
                             const float* voxel_label, const uint8_t* occ_mask, const float* grid_feats,
                             const float* gt_feats, int64_t num_voxels, int64_t channels, float* grad_grid_feats,
                             void* stream) {
    g_msg[0] = 0;
    if (num_voxels < 0 || channels < 0 || channels > INT32_MAX || num_voxels > INT32_MAX || !grad_loss ||
        (num_voxels > 0 && channels > 0 && (!voxel_label || !occ_mask || !grid_feats || !gt_feats || !grad_grid_feats))) {
        set_error("invalid argument");
        return G2V_ERROR_INVALID_VALUE;
    }
    return launch_cosine_loss_bwd(grad_loss, reinterpret_cast<const int*>(count), count_host, voxel_label, occ_mask,
                                  grid_feats, gt_feats, num_voxels, (int)channels, grad_grid_feats,
                                  static_cast<cudaStream_t>(stream));
}

int g2v_forward_splat_batched(int num_scenes, const float* means3d, const float* opacity, const float* features,
                              int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                              const float voxel_range[6], const float* cov_inv, const int32_t* valid_voxel_lb,
                              const int32_t* valid_voxel_ub, const int32_t* g2t_offsets, int64_t num_pairs,
                              int32_t* g2t_tile_ids, float* density, float* grid_feats, int tile_x_begin,
                              int tile_x_end, void* workspace, size_t workspace_bytes, void* stream) {
    return forward_splat_impl(means3d, opacity, features, num_gaussians, channels, voxel_size, voxel_range, cov_inv,
                              valid_voxel_lb, valid_voxel_ub, g2t_offsets, num_pairs, g2t_tile_ids, density,
                              grid_feats, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream, false,
                              num_scenes);
}

int g2v_backward_batched(int num_scenes, const float* grad_density, const float* grad_grid_feats,
                         const float* means3d, const float* opacity, const float* scales, const float* rotations,
                         const float* cov_inv, const float* features, int64_t num_gaussians, int64_t channels,
                         const float voxel_size[3], const float voxel_range[6], const int dims[3],
                         const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                         const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                         const float* density, const float* grid_feats, float* grad_means3d,
                         float* grad_covariances_or_scales, float* grad_rotations, float* grad_opacity,
                         float* grad_features, int tile_x_begin, int tile_x_end, void* workspace,
                         size_t workspace_bytes, void* stream) {
    if (num_gaussians > 0 && scales && !rotations) {
        g_msg[0] = 0;
        set_error("g2v_backward_batched: rotations are required with scales");
        return G2V_ERROR_INVALID_VALUE;
    }
    return backward_impl(grad_density, grad_grid_feats, means3d, opacity, cov_inv, features, num_gaussians, channels,
                         voxel_size, voxel_range, dims, valid_voxel_lb, valid_voxel_ub, g2t_offsets, g2t_tile_ids,
                         num_pairs, num_block_pairs, density, grid_feats, grad_means3d, grad_covariances_or_scales,
                         grad_opacity, grad_features, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream,
                         false, scales, scales ? rotations : nullptr, scales ? grad_rotations : nullptr,
                         num_scenes);
}

int g2v_backward_sr(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                    const float* opacity, const float* scales, const float* rotations, const float* cov_inv,
                    const float* features, int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                    const float voxel_range[6], const int dims[3], const int32_t* valid_voxel_lb,
                    const int32_t* valid_voxel_ub, const int32_t* g2t_offsets, const int32_t* g2t_tile_ids,
                    int64_t num_pairs, int64_t num_block_pairs, const float* density, const float* grid_feats,
                    float* grad_means3d, float* grad_scales, float* grad_rotations, float* grad_opacity,
                    float* grad_features, int tile_x_begin, int tile_x_end, void* workspace, size_t workspace_bytes,
                    void* stream) {
    if (num_gaussians > 0 && (!scales || !rotations)) {
        g_msg[0] = 0;
        set_error("g2v_backward_sr: scales and rotations are required");
        return G2V_ERROR_INVALID_VALUE;
    }
    static const float kDummy = 0.f;  // non-NULL marker for the empty case
    return backward_impl(grad_density, grad_grid_feats, means3d, opacity, cov_inv, features, num_gaussians, channels,
                         voxel_size, voxel_range, dims, valid_voxel_lb, valid_voxel_ub, g2t_offsets, g2t_tile_ids,
                         num_pairs, num_block_pairs, density, grid_feats, grad_means3d, grad_scales, grad_opacity,
                         grad_features, tile_x_begin, tile_x_end, workspace, workspace_bytes, stream, false,
                         scales ? scales : &kDummy, rotations ? rotations : &kDummy, grad_rotations);
}

}  // extern "C"
