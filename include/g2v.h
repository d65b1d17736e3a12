/*
 * g2v.h -- C ABI of libg2v.so, the B200 (sm_100a) Gaussian-to-voxel (G2V) splatting library.
 *
 * The library replaces the reference's CUDA path behind `CudaGaussianVoxelizer._C`
 * (src/bindings.cpp:8-64 of lunarlab-gatech/ShelfGaussian-CudaGaussianVoxelizer).  Every argument is a
 * plain pointer or size; device pointers are CUDA device memory on the current device, `stream` is a
 * cudaStream_t (NULL = legacy default stream).  The library never allocates device memory: every call
 * that needs scratch takes a caller-provided `workspace` whose size comes from the matching
 * *_workspace_size query.  No call exits the process; errors come back as a g2v_status and
 * g2v_last_error() holds a message for the calling thread.
 *
 * Layouts (row-major, float32 unless noted):
 *   means3d (N,3), opacity (N), covariances (N,9) (flattened 3x3), features (N,C)
 *   cov_inv (N,9), valid_voxel_lb / valid_voxel_ub (N,3) int32, num_voxels (N) int32
 *   g2t_offsets (N+1) int32, g2t_tile_ids (M) int32        -- the Gaussian->Tile CSR
 *   density (X,Y,Z), grid_feats (X,Y,Z,C)
 * Tiles are 4x4x4 voxels; the tile id of tile (tx,ty,tz) is (tx*Ty+ty)*Tz+tz.
 */
#ifndef G2V_H
#define G2V_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define G2V_API __attribute__((visibility("default")))
#else
#define G2V_API
#endif

#define G2V_ABI_VERSION 1
#define G2V_TILE 4

typedef enum g2v_status {
    G2V_SUCCESS = 0,
    G2V_ERROR_INVALID_VALUE = 1,        /* bad pointer, shape or voxel grid */
    G2V_ERROR_WORKSPACE_TOO_SMALL = 2,  /* workspace_bytes below the queried size */
    G2V_ERROR_SIZE_LIMIT = 3,           /* a count exceeds the int32 range of the CSR maps */
    G2V_ERROR_CUDA = 4,                 /* a CUDA runtime call or kernel launch failed */
    G2V_ERROR_NOT_SUPPORTED = 5         /* e.g. no sm_100 device */
} g2v_status;

/* Version of this ABI (G2V_ABI_VERSION). */
G2V_API int g2v_abi_version(void);

/* Short name of a status code. */
G2V_API const char* g2v_status_string(int status);

/* Message of the last failing call made by this thread ("" if none). */
G2V_API const char* g2v_last_error(void);

/*
 * Voxel grid and tile grid from the voxel size (3) and range [x0,y0,z0,x1,y1,z1] (6), computed with
 * float32 host arithmetic: dims[a] = (int)((range[a+3]-range[a]) / size[a]), tiles[a] = ceil(dims[a]/4).
 * Replaces src/cuda_gaussian_voxelizer.cu:1512-1519 (which reads the values with 9 .item() syncs).
 * Fails with G2V_ERROR_INVALID_VALUE when a dimension is < 1.
 */
G2V_API int g2v_grid_shape(const float voxel_size[3], const float voxel_range[6], int dims[3], int tiles[3]);

/* Workspace of g2v_forward_prepare for N Gaussians. */
G2V_API int g2v_forward_prepare_workspace_size(int64_t num_gaussians, size_t* bytes);

/*
 * Forward, stage 1: per-Gaussian 3-sigma voxel box, tile count and inverse covariance, then the
 * exclusive prefix sum of the tile counts (g2t_offsets, N+1 entries).  Writes cov_inv, valid_voxel_lb,
 * valid_voxel_ub, num_voxels and g2t_offsets, then reads M = g2t_offsets[N] back to *num_pairs
 * (host) -- the one stream synchronisation of the forward.
 * Replaces src/cuda_gaussian_voxelizer.cu:1484-1631 (ComputeGaussianVoxelPairTile cu:348-536, the CUB
 * scan cu:1608-1615 and the total_tiles_touched readback cu:1628-1631).
 */
G2V_API int g2v_forward_prepare(const float* means3d, const float* covariances, int64_t num_gaussians,
                        const float voxel_size[3], const float voxel_range[6], float* cov_inv,
                        int32_t* valid_voxel_lb, int32_t* valid_voxel_ub, int32_t* num_voxels,
                        int32_t* g2t_offsets, void* workspace, size_t workspace_bytes, void* stream,
                        int64_t* num_pairs);

/*
 * Forward, stage 1, without any host synchronisation (no counterpart in the reference): the same outputs
 * as g2v_forward_prepare except that M is not read back.  The caller chooses the capacity max_pairs in
 * advance (e.g. from an earlier g2v_forward_prepare on the same scene, with headroom) and passes it as
 * num_pairs to g2v_forward_splat and g2v_backward (and its own block-pair capacity as num_block_pairs);
 * every offset is clamped to its capacity, and a call that needed more sets the capacity bit (8) of the
 * device error word -- its results are then invalid, and the next synchronising call or
 * g2v_device_error reports it.  The sequence capped prepare -> splat -> backward contains no host
 * synchronisation and no size-dependent allocation, so it can be captured in a CUDA graph and replayed
 * (the density-only fast path of training loops with a fixed number of Gaussians).
 */
G2V_API int g2v_forward_prepare_capped(const float* means3d, const float* covariances, int64_t num_gaussians,
                                       const float voxel_size[3], const float voxel_range[6], int64_t max_pairs,
                                       float* cov_inv, int32_t* valid_voxel_lb, int32_t* valid_voxel_ub,
                                       int32_t* num_voxels, int32_t* g2t_offsets, void* workspace,
                                       size_t workspace_bytes, void* stream);

/*
 * Forward, stage 1, for callers that cannot allocate device memory (no counterpart in the reference).
 * Same inputs, outputs and single stream synchronisation as g2v_forward_prepare, but no workspace: some
 * callers cannot provide one -- e.g. a serving process that reserves all device memory at start-up and
 * must not call cudaMalloc afterwards, or a plugin whose host application owns every device allocation.
 * The scratch is a fixed array of about 1 MiB in the library's own device memory, so inputs are limited
 * to G2V_STATIC_MAX_GAUSSIANS Gaussians (larger inputs fail with G2V_ERROR_SIZE_LIMIT); the grid limits
 * and the device-error reporting are those of g2v_forward_prepare.  The first call on a device looks up
 * that array's address (call it once before any stream capture) and caches it per device ordinal, which
 * assumes one primary context per device for the life of the process (not after cudaDeviceReset); all
 * calls share the array, so calls that overlap on the GPU race.
 */
#define G2V_STATIC_MAX_GAUSSIANS 262144
G2V_API int g2v_forward_prepare_static(const float* means3d, const float* covariances, int64_t num_gaussians,
                                       const float voxel_size[3], const float voxel_range[6], float* cov_inv,
                                       int32_t* valid_voxel_lb, int32_t* valid_voxel_ub, int32_t* num_voxels,
                                       int32_t* g2t_offsets, void* stream, int64_t* num_pairs);

/* Workspace of g2v_forward_splat. */
G2V_API int g2v_forward_splat_workspace_size(int64_t num_gaussians, int64_t num_pairs, const int dims[3],
                                     int64_t channels, size_t* bytes);

/*
 * Forward, stage 2: fills the Gaussian->Tile tile ids (g2t_tile_ids, M entries, x-major over each
 * Gaussian's tile box), builds the Tile->Gaussian CSR (Gaussian ids ascending inside a tile) and
 * splats every tile: density D_v = sum_g w_gv and grid_feats F_v = sum_g w_gv f_g / max(D_v, 1e-6),
 * w_gv = opacity_g * exp(-1/2 d^T cov_inv_g d) over the voxels of the Gaussian's box.  Every voxel of
 * the tiles with tile x in [tile_x_begin, tile_x_end) is written (zeros where no Gaussian reaches);
 * pass 0 and tiles[0] for the whole grid.  features == NULL selects the density-only path
 * (grid_feats unused, channels ignored).  With features != NULL and channels == 0 the density is
 * left at zero, as the reference does (its density sum sits inside the channel loop, cu:857-926).
 * Replaces src/cuda_gaussian_voxelizer.cu:1633-1913 (FillG2TKernel, CUB SortPairs / RunLengthEncode /
 * scan, zero_, ComputeGaussian2VoxelTileWithFeats or ComputeGaussian2VoxelTile, clamp_min + div_).
 */
G2V_API int g2v_forward_splat(const float* means3d, const float* opacity, const float* features, int64_t num_gaussians,
                      int64_t channels, const float voxel_size[3], const float voxel_range[6],
                      const float* cov_inv, const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub,
                      const int32_t* g2t_offsets, int64_t num_pairs, int32_t* g2t_tile_ids, float* density,
                      float* grid_feats, int tile_x_begin, int tile_x_end, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * g2v_forward_splat for one x-slab of a scene sharded across devices: the same arguments, but density
 * and grid_feats hold only the slab's voxel x rows, [4 * tile_x_begin, min(4 * tile_x_end, X)), as
 * (rows, Y, Z) and (rows, Y, Z, C) arrays.  Each rank of a single-scene split calls it for its slab;
 * the slabs' outputs are disjoint.  No reference counterpart (the reference is single-device).
 */
G2V_API int g2v_forward_splat_local(const float* means3d, const float* opacity, const float* features,
                                    int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                                    const float voxel_range[6], const float* cov_inv, const int32_t* valid_voxel_lb,
                                    const int32_t* valid_voxel_ub, const int32_t* g2t_offsets, int64_t num_pairs,
                                    int32_t* g2t_tile_ids, float* density, float* grid_feats, int tile_x_begin,
                                    int tile_x_end, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward planning: counts the (Gaussian, tile block) pairs that the feature-gradient pass needs and
 * reads the count back to *num_block_pairs (one stream synchronisation).  Needed only to size the
 * backward workspace; the Python layer obtains it once per forward.
 * No direct reference counterpart (the reference backward allocates inside cu:1964-1967).
 */
G2V_API int g2v_backward_plan(const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, int64_t num_gaussians,
                      const int dims[3], int64_t channels, void* workspace, size_t workspace_bytes,
                      void* stream, int64_t* num_block_pairs);

/* Workspace of g2v_backward_plan (N-sized). */
G2V_API int g2v_backward_plan_workspace_size(int64_t num_gaussians, size_t* bytes);

/*
 * g2v_forward_prepare and g2v_backward_plan in one call with a single stream synchronisation: the same
 * outputs as g2v_forward_prepare plus *num_block_pairs (0 when channels == 0).  For training loops that
 * run the backward after every forward; saves the backward's planning round trip.
 * Replaces cu:1484-1631 like g2v_forward_prepare (the planning part has no reference counterpart).
 */
G2V_API int g2v_forward_prepare_plan(const float* means3d, const float* covariances, int64_t num_gaussians,
                                     const float voxel_size[3], const float voxel_range[6], float* cov_inv,
                                     int32_t* valid_voxel_lb, int32_t* valid_voxel_ub, int32_t* num_voxels,
                                     int32_t* g2t_offsets, int64_t channels, void* workspace,
                                     size_t workspace_bytes, void* stream, int64_t* num_pairs,
                                     int64_t* num_block_pairs);

/* Workspace of g2v_forward_prepare_plan (N-sized); also that of g2v_forward_prepare_plan_sr. */
G2V_API int g2v_forward_prepare_plan_workspace_size(int64_t num_gaussians, size_t* bytes);

/*
 * Batches of scenes in one call (no reference counterpart: GaussTR-style callers loop over the batch,
 * one forward with its synchronisation per scene).  B scenes share voxel_size / voxel_range; scene b owns
 * the Gaussians [scene_offsets[b], scene_offsets[b+1]) of the concatenated per-Gaussian arrays (ragged
 * sizes; scene_offsets is a device int32 array of B+1 entries from 0 to num_gaussians) and voxel x rows
 * [b X, (b+1) X) of the volume arrays, which are therefore (B, X, Y, Z) and (B, X, Y, Z, C).  Boxes
 * are clamped to each Gaussian's own scene; valid_voxel_lb / ub and g2t_tile_ids are in the coordinates
 * of this stacked grid (x + b X, tile id of the (B*X, Y, Z) grid), and every *_workspace_size / dims
 * argument takes the stacked dims (B*X, Y, Z).  X must be a multiple of 4 when B > 1
 * (G2V_ERROR_NOT_SUPPORTED otherwise).  Per scene the results are those of a single-scene call.
 *
 * g2v_forward_prepare_plan_batched: g2v_forward_prepare_plan for the batch -- covariances, or (when
 * scales is non-NULL) scales + rotations as in g2v_forward_prepare_plan_sr; one synchronisation for the
 * whole batch.
 */
G2V_API int g2v_forward_prepare_plan_batched(const float* means3d, const float* covariances, const float* scales,
                                             const float* rotations, const int32_t* scene_offsets, int num_scenes,
                                             int64_t num_gaussians, const float voxel_size[3],
                                             const float voxel_range[6], float* cov_inv, int32_t* valid_voxel_lb,
                                             int32_t* valid_voxel_ub, int32_t* num_voxels, int32_t* g2t_offsets,
                                             int64_t channels, void* workspace, size_t workspace_bytes,
                                             void* stream, int64_t* num_pairs, int64_t* num_block_pairs);

/*
 * Covariances from per-Gaussian scales (N,3) and rotation quaternions (N,4, (r, x, y, z), any norm):
 * covariances (N,9) = R(q/|q|) diag(s)^2 R(q/|q|)^T, row-major.  Replaces the GaussTR front end that
 * feeds the voxelizer, get_covariance(scales, quat_to_rotmat(rotations)) (test/gaussian_voxelizer.py:
 * 14-37, called at :176-177).  Stream-ordered, no synchronisation.  A zero quaternion gives NaN, as
 * the reference's division does.
 */
G2V_API int g2v_covariance_from_scale_rot(const float* scales, const float* rotations, int64_t num_gaussians,
                                          float* covariances, void* stream);

/*
 * Gradient of g2v_covariance_from_scale_rot: from grad_covariances (N,9, entries independent, the layout
 * g2v_backward writes) to grad_scales (N,3) and grad_rotations (N,4) -- what autograd through the
 * reference front end gives.
 */
G2V_API int g2v_covariance_from_scale_rot_backward(const float* scales, const float* rotations,
                                                   const float* grad_covariances, int64_t num_gaussians,
                                                   float* grad_scales, float* grad_rotations, void* stream);

/*
 * g2v_forward_prepare_plan with the covariances formed inside the preparation kernel from scales (N,3)
 * and rotations (N,4) (the same bits as g2v_covariance_from_scale_rot): no covariance array is read or
 * written.  Same outputs, workspace and single synchronisation.
 */
G2V_API int g2v_forward_prepare_plan_sr(const float* means3d, const float* scales, const float* rotations,
                                        int64_t num_gaussians, const float voxel_size[3],
                                        const float voxel_range[6], float* cov_inv, int32_t* valid_voxel_lb,
                                        int32_t* valid_voxel_ub, int32_t* num_voxels, int32_t* g2t_offsets,
                                        int64_t channels, void* workspace, size_t workspace_bytes, void* stream,
                                        int64_t* num_pairs, int64_t* num_block_pairs);

/* Workspace of g2v_backward. */
G2V_API int g2v_backward_workspace_size(int64_t num_gaussians, int64_t num_pairs, int64_t num_block_pairs,
                                const int dims[3], int64_t channels, size_t* bytes);

/*
 * Backward of L(density, grid_feats) given dL/ddensity (X,Y,Z) and dL/dgrid_feats (X,Y,Z,C):
 * writes grad_means3d (N,3), grad_covariances (N,9, symmetric, off-diagonal not halved),
 * grad_opacity (N) and, when features != NULL, grad_features (N,C).  Every output element is written.
 * Only the voxels of tiles with tile x in [tile_x_begin, tile_x_end) contribute (0 / tiles[0] for the
 * whole grid): on an x-slab the outputs are that slab's partial gradients.
 * e_v = sum_c dL/dF_vc F_vc (the reference's at::bmm) is formed from the per-pair dot products the
 * tile pass computes anyway; only for the voxels of cells (z columns of four tiles) with more than 256 Gaussians
 * is it read from grid_feats (the forward's output), which saves running their slot passes twice.
 * grid_feats may be NULL: then those cells run both passes.
 * Replaces src/cuda_gaussian_voxelizer.cu:1920-2057 (the at::bmm at cu:1996 and
 * ComputeGaussian2VoxelGradientTileWithFeats / ComputeGaussian2VoxelGradientTile).
 */
G2V_API int g2v_backward(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                 const float* opacity, const float* cov_inv, const float* features, int64_t num_gaussians,
                 int64_t channels, const float voxel_size[3], const float voxel_range[6], const int dims[3],
                 const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                 const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs, const float* density,
                 const float* grid_feats, float* grad_means3d, float* grad_covariances, float* grad_opacity,
                 float* grad_features, int tile_x_begin, int tile_x_end, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * g2v_backward over the whole grid with the tile pass's unit lists supplied by the caller instead of
 * rebuilt: unit_offsets (num_units + 1) and unit_lists (num_pairs), the z-columns-of-four-tiles CSR that
 * g2v_forward_splat built for the same Gaussians (copied out with g2v_forward_splat_unit_lists).  Used
 * only by the tensor-core path (the FP32-FMA variant builds its own lists).  Same outputs and workspace as
 * g2v_backward; a host-side saving of the reference's backward, which rebuilds nothing because it walks
 * the G2T map per Gaussian (cu:1376-1482).
 */
G2V_API int g2v_backward_units(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                               const float* opacity, const float* cov_inv, const float* features,
                               int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                               const float voxel_range[6], const int dims[3], const int32_t* valid_voxel_lb,
                               const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                               const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                               const float* density, const float* grid_feats, float* grad_means3d,
                               float* grad_covariances, float* grad_opacity, float* grad_features,
                               const int32_t* unit_offsets, const int32_t* unit_lists, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * Copies the unit lists (Gaussian ids of each z column of four tiles, ascending; the cell->Gaussian CSR the
 * tensor-core splat and tile pass work on) out of a g2v_forward_splat workspace after the call:
 * unit_offsets (num_units + 1, int32) and unit_lists (num_pairs, int32; entries beyond
 * unit_offsets[num_units] unspecified).  With unit_offsets == NULL only *num_units is returned.  Fails
 * when the splat built no unit lists (channels == 0 or the FP32-FMA variant).  No reference counterpart
 * (the reference keeps its lists internal, cu:1675-1772).
 */
G2V_API int g2v_forward_splat_unit_lists(const void* splat_workspace, int64_t num_gaussians, int64_t num_pairs,
                                         const int dims[3], int64_t channels, int32_t* unit_offsets,
                                         int32_t* unit_lists, int64_t* num_units, void* stream);

/*
 * g2v_backward for Gaussians parameterised by scales (N,3) and rotations (N,4): the same inputs plus
 * scales/rotations, and grad_scales (N,3) / grad_rotations (N,4) in place of grad_covariances (the chain
 * rule runs in the per-Gaussian gradient reduction, so dL/dSigma is never written).  Workspace: the
 * g2v_backward_workspace_size of the same sizes.  Replaces autograd through get_covariance /
 * quat_to_rotmat (test/gaussian_voxelizer.py:14-37) after the reference backward (cu:1920-2057).
 */
G2V_API int g2v_backward_sr(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                            const float* opacity, const float* scales, const float* rotations, const float* cov_inv,
                            const float* features, int64_t num_gaussians, int64_t channels,
                            const float voxel_size[3], const float voxel_range[6], const int dims[3],
                            const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub,
                            const int32_t* g2t_offsets, const int32_t* g2t_tile_ids, int64_t num_pairs,
                            int64_t num_block_pairs, const float* density, const float* grid_feats,
                            float* grad_means3d, float* grad_scales, float* grad_rotations, float* grad_opacity,
                            float* grad_features, int tile_x_begin, int tile_x_end, void* workspace,
                            size_t workspace_bytes, void* stream);

/* g2v_forward_splat for a batch of num_scenes stacked scenes (see g2v_forward_prepare_plan_batched). */
G2V_API int g2v_forward_splat_batched(int num_scenes, const float* means3d, const float* opacity,
                                      const float* features, int64_t num_gaussians, int64_t channels,
                                      const float voxel_size[3], const float voxel_range[6], const float* cov_inv,
                                      const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub,
                                      const int32_t* g2t_offsets, int64_t num_pairs, int32_t* g2t_tile_ids,
                                      float* density, float* grid_feats, int tile_x_begin, int tile_x_end,
                                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * g2v_backward for a batch of num_scenes stacked scenes; dims = (B*X, Y, Z).  With scales == NULL the
 * covariance gradient goes to grad_covariances_or_scales (N,9) and grad_rotations is unused; with scales
 * and rotations (the batch was prepared from them) grad_covariances_or_scales receives grad_scales (N,3)
 * and grad_rotations (N,4), as in g2v_backward_sr.
 */
G2V_API int g2v_backward_batched(int num_scenes, const float* grad_density, const float* grad_grid_feats,
                                 const float* means3d, const float* opacity, const float* scales,
                                 const float* rotations, const float* cov_inv, const float* features,
                                 int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                                 const float voxel_range[6], const int dims[3], const int32_t* valid_voxel_lb,
                                 const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                                 const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                                 const float* density, const float* grid_feats, float* grad_means3d,
                                 float* grad_covariances_or_scales, float* grad_rotations, float* grad_opacity,
                                 float* grad_features, int tile_x_begin, int tile_x_end, void* workspace,
                                 size_t workspace_bytes, void* stream);

/*
 * g2v_backward for one x-slab with slab-local volume arrays (grad_density, grad_grid_feats, density,
 * grid_feats hold the slab's voxel x rows only, as in g2v_forward_splat_local).  The outputs are the
 * slab's partial per-Gaussian gradients; summed over the slabs of a split (one all-reduce) they equal
 * the whole-grid gradients.  No reference counterpart.
 */
G2V_API int g2v_backward_local(const float* grad_density, const float* grad_grid_feats, const float* means3d,
                               const float* opacity, const float* cov_inv, const float* features,
                               int64_t num_gaussians, int64_t channels, const float voxel_size[3],
                               const float voxel_range[6], const int dims[3], const int32_t* valid_voxel_lb,
                               const int32_t* valid_voxel_ub, const int32_t* g2t_offsets,
                               const int32_t* g2t_tile_ids, int64_t num_pairs, int64_t num_block_pairs,
                               const float* density, const float* grid_feats, float* grad_means3d,
                               float* grad_covariances, float* grad_opacity, float* grad_features, int tile_x_begin,
                               int tile_x_end, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Feature cosine loss over the voxel grid (the consumer of grid_feats in training).  All arrays are
 * device, contiguous, row-major over V = X*Y*Z voxels: voxel_label [V] f32, occ_mask [V] bool/u8,
 * grid_feats and gt_feats [V, channels] f32.  A voxel is valid when occ_mask != 0 and label > 0;
 * loss_v = 1 - p.g / (sqrt(max(|p|^2, 1e-6)) sqrt(max(|g|^2, 1e-6)) + 1e-6).
 *
 * g2v_cosine_loss_forward writes *loss (device f32: the mean of loss_v over valid voxels, 0 when there
 * are none) and *count (device int32: the number of valid voxels).  Stream-ordered, no synchronisation,
 * deterministic (fixed summation order).  Replaces CudaFeatsCosinelossForward, src/cuda_feats_loss.cu:146-225
 * (VoxelCosineLossKernel :45-101 + ReduceLossAndCountKernel :104-143), which returns the count to the
 * host.  The workspace is a fixed 16 KiB (g2v_cosine_loss_workspace_size).
 */
G2V_API int g2v_cosine_loss_workspace_size(int64_t num_voxels, size_t* bytes);
G2V_API int g2v_cosine_loss_forward(const float* voxel_label, const uint8_t* occ_mask, const float* grid_feats,
                                    const float* gt_feats, int64_t num_voxels, int64_t channels, float* loss,
                                    int32_t* count, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Gradient of the cosine loss with respect to grid_feats: grad_grid_feats [V, channels] f32 (every
 * voxel written; invalid voxels get 0).  grad_loss is the upstream gradient (device f32 scalar); the
 * valid-voxel count comes from `count` (device int32, e.g. the forward's output) or, when count is
 * NULL, from count_host.  Stream-ordered, no synchronisation.  Replaces CudaFeatsCosinelossBackward,
 * src/cuda_feats_loss.cu:311-366 (CosineLossBackwardKernel :228-289), which reads grad_output and the
 * count on the host.
 */
G2V_API int g2v_cosine_loss_backward(const float* grad_loss, const int32_t* count, int32_t count_host,
                                     const float* voxel_label, const uint8_t* occ_mask, const float* grid_feats,
                                     const float* gt_feats, int64_t num_voxels, int64_t channels,
                                     float* grad_grid_feats, void* stream);

/*
 * The reference's Tile->Gaussian CSR over the whole grid, built from the forward's boxes: the stable
 * sort of the (tile id, Gaussian id) pairs by tile, run-length encoding and scan of
 * src/cuda_gaussian_voxelizer.cu:1675-1772 (CUB there; the reference keeps the map internal).
 * tile_offsets (num_tiles+1, int32, all tiles), t2g_gaussians (num_pairs, int32, Gaussian ids ascending
 * within each tile).  The tensor-core splat does not need this map (it lists z columns of four tiles), so the
 * forward no longer builds it; this call exposes it.  workspace: g2v_build_t2g_workspace_size.
 */
G2V_API int g2v_build_t2g_workspace_size(int64_t num_gaussians, int64_t num_pairs, const int dims[3],
                                         size_t* bytes);
G2V_API int g2v_build_t2g(const int32_t* valid_voxel_lb, const int32_t* valid_voxel_ub, int64_t num_gaussians,
                          const float voxel_size[3], const float voxel_range[6], int64_t num_pairs,
                          int32_t* tile_offsets, int32_t* t2g_gaussians, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * Device error word (no reference counterpart): the tensor-core kernels never spin without a bound;
 * a wait that gives up sets a bit in a per-device word instead of hanging.  g2v_forward_prepare and
 * g2v_backward_plan read the word at the synchronisation they already do and fail with
 * G2V_ERROR_CUDA if it is set.  This call reads it explicitly (synchronising `stream`), returns it in
 * *word and clears it.
 */
G2V_API int g2v_device_error(void* stream, int* word);

/*
 * Self-test of the failure path (no reference counterpart): launches one CTA that waits on an mbarrier
 * nothing arrives at, with the library's bounded wait (about 2 s), and synchronises `stream`.  On return
 * *gave_up is 1 when the wait gave up as designed, and the device error word holds its timeout bit
 * (read and clear it with g2v_device_error).  The context stays usable.
 */
G2V_API int g2v_debug_wait_timeout(void* stream, int* gave_up);

/*
 * Profiling hook (no reference counterpart): when enabled, every kernel launch of the library is
 * bracketed by CUDA events on its launch stream.  g2v_profile_enable(1) clears the records and starts
 * recording, g2v_profile_enable(0) stops.  g2v_profile_read(i, ...) waits for the recorded events,
 * aggregates them by kernel name and returns entry i (name, total milliseconds, launches);
 * it returns G2V_ERROR_INVALID_VALUE past the last entry.
 */
G2V_API int g2v_profile_enable(int enabled);
G2V_API int g2v_profile_read(int index, char* name, size_t name_len, double* total_ms, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* G2V_H */
