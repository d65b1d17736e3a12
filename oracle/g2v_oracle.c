/*
 * g2v_oracle.c -- CPU restatement of the reference Gaussian-to-voxel (G2V) path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU legs of
 * bench.py load this library, and only as the checker / the timed CPU baseline.  The
 * product path (libg2v.so) never links or calls it.
 *
 * What it restates (paths are inside the reference project):
 *   grid shape       src/cuda_gaussian_voxelizer.cu:1512-1519  float32 host division, int truncation,
 *                    tile counts ceil(dim/4)
 *   per-Gaussian box src/cuda_gaussian_voxelizer.cu:367-532   sigma = sqrt(diag cov), [mu-3s, mu+3s],
 *                    clamp to the range, floor((v-v0)/h), clamp to the grid, empty box -> lb=0, ub=-1,
 *                    tile box = voxel box / 4
 *   inverse          src/cuda_gaussian_voxelizer.cu:201-220   3x3 adjugate with |det|<1e-6 -> det=1e-6
 *   G2T CSR          src/cuda_gaussian_voxelizer.cu:228-286 + 1608-1615  x-major enumeration of the tile
 *                    box, tile id (tx*Ty+ty)*Tz+tz, offsets = exclusive prefix sum of tile counts
 *   T2G CSR          src/cuda_gaussian_voxelizer.cu:1675-1772  stable sort of the G2T pairs by tile id
 *                    (Gaussian ids ascending inside a tile)
 *   values           test/test_reference.py:57-79  float64 brute force: w = o exp(-1/2 d^T inv(S) d) over the
 *                    voxels of the box, D = sum w, F = sum w f / max(D, 1e-6)
 *   gradients        the analytic derivative of that brute force (what torch autograd computes in
 *                    test/test_reference.py:103-124), float64.
 *
 * The box arithmetic mirrors the reference's float32 operations.  The reference is built with
 * --use_fast_math, so on the GPU sqrtf and '/' are approximate; this file uses IEEE sqrtf and division.
 * The two can disagree when (v-v0)/h lies within a few ulp of an integer.  The GPU parity tests
 * therefore pin the boxes bit-exactly against the reference build itself and only count such
 * boundary flips against this restatement.  `mu - 3*sigma` is evaluated as one fused multiply-add,
 * which is how nvcc contracts that expression.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TILE 4
#define EPS_D 1e-6

/* float -> int32 as PTX cvt.rzi.s32.f32 defines it: truncate, saturate, NaN -> 0. */
static int32_t sat_f2i(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x <= -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}

/* int32 products wrap like the GPU's 32-bit multiply. */
static int32_t mul3_wrap(int32_t a, int32_t b, int32_t c) {
    uint32_t r = (uint32_t)a * (uint32_t)b;
    r = r * (uint32_t)c;
    return (int32_t)r;
}

/* Grid shape, reference cu:1512-1519.  Returns 0 on success, -1 when a dimension is < 1 or too big. */
int g2v_oracle_grid_shape(const float size[3], const float range[6], int dims[3], int tiles[3]) {
    for (int a = 0; a < 3; ++a) {
        float q = (range[3 + a] - range[a]) / size[a];
        if (!(q >= 1.0f) || !(q < 2147483648.0f)) return -1;
        dims[a] = (int)q;
        tiles[a] = (dims[a] + TILE - 1) / TILE;
    }
    return 0;
}

/* 3x3 inverse with the reference's determinant clamp (cu:201-220); IEEE float32 arithmetic. */
static void inverse3_clamped(const float A[9], float R[9]) {
    float c00 = A[4] * A[8] - A[5] * A[7];
    float c01 = A[3] * A[8] - A[5] * A[6];
    float c02 = A[3] * A[7] - A[4] * A[6];
    float det = A[0] * c00 - A[1] * c01 + A[2] * c02;
    if (fabsf(det) < 1e-6f) det = 1e-6f;
    float inv = 1.0f / det;
    R[0] = c00 * inv;
    R[1] = -(A[1] * A[8] - A[2] * A[7]) * inv;
    R[2] = (A[1] * A[5] - A[2] * A[4]) * inv;
    R[3] = -c01 * inv;
    R[4] = (A[0] * A[8] - A[2] * A[6]) * inv;
    R[5] = -(A[0] * A[5] - A[2] * A[3]) * inv;
    R[6] = c02 * inv;
    R[7] = -(A[0] * A[7] - A[1] * A[6]) * inv;
    R[8] = (A[0] * A[4] - A[1] * A[3]) * inv;
}

/*
 * Per-Gaussian boxes, reference cu:367-536.  Outputs (all row-major):
 *   lb, ub (N,3) int32; num_voxels (N) int32; tile_lo, tile_hi (N,3) int32; num_tiles (N) int32;
 *   cov_inv (N,9) float32 (zero for an empty box, like cu:496).
 */
void g2v_oracle_boxes(int64_t n, const float* means, const float* cov, const float size[3],
                      const float range[6], const int dims[3], const int tiles[3], int32_t* lb, int32_t* ub,
                      int32_t* num_voxels, int32_t* tile_lo, int32_t* tile_hi, int32_t* num_tiles,
                      float* cov_inv) {
    for (int64_t g = 0; g < n; ++g) {
        int32_t lo[3], hi[3];
        for (int a = 0; a < 3; ++a) {
            float mu = means[g * 3 + a];
            float s = sqrtf(cov[g * 9 + 4 * a]);
            float lower = fmaf(-3.0f, s, mu);
            float upper = fmaf(3.0f, s, mu);
            lower = fmaxf(lower, range[a]);
            upper = fminf(upper, range[3 + a]);
            int32_t l = sat_f2i(floorf((lower - range[a]) / size[a]));
            int32_t h = sat_f2i(floorf((upper - range[a]) / size[a]));
            lo[a] = l > 0 ? l : 0;
            hi[a] = h < dims[a] - 1 ? h : dims[a] - 1;
        }
        int empty = lo[0] > hi[0] || lo[1] > hi[1] || lo[2] > hi[2];
        if (empty) {
            for (int a = 0; a < 3; ++a) {
                lb[g * 3 + a] = 0; ub[g * 3 + a] = -1;
                tile_lo[g * 3 + a] = 0; tile_hi[g * 3 + a] = -1;
            }
            num_voxels[g] = 0;
            num_tiles[g] = 0;
            for (int k = 0; k < 9; ++k) cov_inv[g * 9 + k] = 0.0f;
            continue;
        }
        int32_t tlo[3], thi[3];
        for (int a = 0; a < 3; ++a) {
            lb[g * 3 + a] = lo[a];
            ub[g * 3 + a] = hi[a];
            tlo[a] = lo[a] / TILE;
            thi[a] = hi[a] / TILE;
            if (tlo[a] < 0) tlo[a] = 0;
            if (thi[a] > tiles[a] - 1) thi[a] = tiles[a] - 1;
            tile_lo[g * 3 + a] = tlo[a];
            tile_hi[g * 3 + a] = thi[a];
        }
        num_voxels[g] = mul3_wrap(hi[0] - lo[0] + 1, hi[1] - lo[1] + 1, hi[2] - lo[2] + 1);
        num_tiles[g] = mul3_wrap(thi[0] - tlo[0] + 1, thi[1] - tlo[1] + 1, thi[2] - tlo[2] + 1);
        inverse3_clamped(cov + g * 9, cov_inv + g * 9);
    }
}

/* G2T offsets (exclusive prefix of num_tiles, N+1 entries); returns M. */
int64_t g2v_oracle_g2t_offsets(int64_t n, const int32_t* num_tiles, int64_t* offsets) {
    int64_t acc = 0;
    offsets[0] = 0;
    for (int64_t g = 0; g < n; ++g) {
        acc += num_tiles[g] > 0 ? num_tiles[g] : 0;
        offsets[g + 1] = acc;
    }
    return acc;
}

/* G2T tile ids, x-major over each Gaussian's tile box (cu:263-284). */
void g2v_oracle_g2t_fill(int64_t n, const int32_t* tile_lo, const int32_t* tile_hi, const int64_t* offsets,
                         const int tiles[3], int32_t* g2t_tile_ids) {
    for (int64_t g = 0; g < n; ++g) {
        int dx = tile_hi[g * 3 + 0] - tile_lo[g * 3 + 0] + 1;
        int dy = tile_hi[g * 3 + 1] - tile_lo[g * 3 + 1] + 1;
        int dz = tile_hi[g * 3 + 2] - tile_lo[g * 3 + 2] + 1;
        if (dx <= 0 || dy <= 0 || dz <= 0) continue;
        int64_t base = offsets[g];
        int64_t count = (int64_t)dx * dy * dz;
        for (int64_t i = 0; i < count; ++i) {
            int lx = (int)(i / (dy * dz));
            int r = (int)(i % (dy * dz));
            int ly = r / dz, lz = r % dz;
            int tx = tile_lo[g * 3 + 0] + lx, ty = tile_lo[g * 3 + 1] + ly, tz = tile_lo[g * 3 + 2] + lz;
            g2t_tile_ids[base + i] = (tx * tiles[1] + ty) * tiles[2] + tz;
        }
    }
}

/*
 * T2G CSR over ALL tiles: tile_offsets (num_tiles+1) and the Gaussian ids of each tile in ascending
 * order -- the result of the reference's stable radix sort + run-length encoding, expressed over the
 * full tile range instead of the active tiles only.
 */
void g2v_oracle_t2g(int64_t n, int64_t num_tiles_total, const int64_t* g2t_offsets, const int32_t* g2t_tile_ids,
                    int64_t* tile_offsets, int32_t* t2g_gaussians) {
    memset(tile_offsets, 0, sizeof(int64_t) * (size_t)(num_tiles_total + 1));
    int64_t m = g2t_offsets[n];
    for (int64_t i = 0; i < m; ++i) tile_offsets[g2t_tile_ids[i] + 1] += 1;
    for (int64_t t = 0; t < num_tiles_total; ++t) tile_offsets[t + 1] += tile_offsets[t];
    int64_t* cursor = (int64_t*)malloc(sizeof(int64_t) * (size_t)(num_tiles_total > 0 ? num_tiles_total : 1));
    memcpy(cursor, tile_offsets, sizeof(int64_t) * (size_t)num_tiles_total);
    for (int64_t g = 0; g < n; ++g)
        for (int64_t i = g2t_offsets[g]; i < g2t_offsets[g + 1]; ++i)
            t2g_gaussians[cursor[g2t_tile_ids[i]]++] = (int32_t)g;
    free(cursor);
}

/* float64 inverse of the float32 covariance (the brute force calls torch.linalg.inv in float64). */
static void inverse3_d(const float* A32, double P[9]) {
    double A[9];
    for (int k = 0; k < 9; ++k) A[k] = (double)A32[k];
    double c00 = A[4] * A[8] - A[5] * A[7];
    double c01 = A[3] * A[8] - A[5] * A[6];
    double c02 = A[3] * A[7] - A[4] * A[6];
    double det = A[0] * c00 - A[1] * c01 + A[2] * c02;
    double inv = 1.0 / det;
    P[0] = c00 * inv;
    P[1] = -(A[1] * A[8] - A[2] * A[7]) * inv;
    P[2] = (A[1] * A[5] - A[2] * A[4]) * inv;
    P[3] = -c01 * inv;
    P[4] = (A[0] * A[8] - A[2] * A[6]) * inv;
    P[5] = -(A[0] * A[5] - A[2] * A[3]) * inv;
    P[6] = c02 * inv;
    P[7] = -(A[0] * A[7] - A[1] * A[6]) * inv;
    P[8] = (A[0] * A[4] - A[1] * A[3]) * inv;
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

/*
 * Brute-force forward (test/test_reference.py:57-79) over the voxel slab x in [x0, x1).
 * vlo/vsize are the float64 range origin and voxel size (Python floats in the reference test).
 * density (X*Y*Z) and grid_feats (X*Y*Z*C) are written only inside the slab; grid_feats is already
 * normalised by max(D, 1e-6).  features may be NULL when c == 0.
 */
void g2v_oracle_forward(int64_t n, int c, const float* means, const float* opacity, const float* cov,
                        const float* features, const int32_t* lb, const int32_t* ub, const double vlo[3],
                        const double vsize[3], const int dims[3], int x0, int x1, double* density,
                        double* grid_feats, int nthreads) {
    const int X = dims[0], Y = dims[1], Z = dims[2];
    (void)X;
    double* P = (double*)malloc(sizeof(double) * 9 * (size_t)(n > 0 ? n : 1));
    for (int64_t g = 0; g < n; ++g) inverse3_d(cov + g * 9, P + g * 9);
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
    for (int x = x0; x < x1; ++x) {
        double* dslab = density + (int64_t)x * Y * Z;
        double* fslab = grid_feats ? grid_feats + (int64_t)x * Y * Z * c : NULL;
        for (int64_t i = 0; i < (int64_t)Y * Z; ++i) dslab[i] = 0.0;
        if (fslab) for (int64_t i = 0; i < (int64_t)Y * Z * c; ++i) fslab[i] = 0.0;
        for (int64_t g = 0; g < n; ++g) {
            if (x < lb[g * 3] || x > ub[g * 3]) continue;
            const double* p = P + g * 9;
            double cx = vlo[0] + (x + 0.5) * vsize[0] - (double)means[g * 3 + 0];
            double o = (double)opacity[g];
            for (int y = lb[g * 3 + 1]; y <= ub[g * 3 + 1]; ++y) {
                double cy = vlo[1] + (y + 0.5) * vsize[1] - (double)means[g * 3 + 1];
                for (int z = lb[g * 3 + 2]; z <= ub[g * 3 + 2]; ++z) {
                    double cz = vlo[2] + (z + 0.5) * vsize[2] - (double)means[g * 3 + 2];
                    double d[3] = {cx, cy, cz};
                    double maha = 0.0;
                    for (int i = 0; i < 3; ++i)
                        for (int j = 0; j < 3; ++j) maha += d[i] * p[i * 3 + j] * d[j];
                    double w = o * exp(-0.5 * maha);
                    int64_t v = (int64_t)y * Z + z;
                    dslab[v] += w;
                    if (fslab && c > 0) {
                        const float* f = features + g * (int64_t)c;
                        double* out = fslab + v * c;
                        for (int k = 0; k < c; ++k) out[k] += w * (double)f[k];
                    }
                }
            }
        }
        if (fslab && c > 0) {
            for (int64_t v = 0; v < (int64_t)Y * Z; ++v) {
                double den = dslab[v] > EPS_D ? dslab[v] : EPS_D;
                for (int k = 0; k < c; ++k) fslab[v * c + k] /= den;
            }
        }
    }
    free(P);
}

/*
 * Analytic float64 gradient of L = sum gD*D + sum gF*F for the brute force above, restricted to the
 * voxels of the slab x in [x0, x1) (so that a slab sample can be timed; the full range gives the whole
 * gradient).  density and grid_feats are the forward outputs (float64) over the same slab.
 * For each Gaussian g and voxel v of its box:
 *   a_gv   = gD_v + (sum_c gF_vc f_gc - [D_v >= eps] sum_c gF_vc F_vc) / max(D_v, eps)
 *   dmu    += a_gv * w_gv * 1/2 (P + P^T) d
 *   dSigma += a_gv * w_gv * 1/2 (P^T d)(P d)^T
 *   dop    += a_gv * exp(-1/2 d^T P d)
 *   df_g   += gF_v * w_gv / max(D_v, eps)
 * which is what autograd returns for test/test_reference.py:57-79 (clamp_min passes the gradient where
 * D >= eps).  Outputs are zero for Gaussians with an empty box.
 */
void g2v_oracle_backward(int64_t n, int c, const float* means, const float* opacity, const float* cov,
                         const float* features, const int32_t* lb, const int32_t* ub, const double vlo[3],
                         const double vsize[3], const int dims[3], int x0, int x1, const float* grad_density,
                         const float* grad_feats, const double* density, const double* grid_feats,
                         double* grad_means, double* grad_cov, double* grad_opacity, double* grad_features,
                         int nthreads) {
    const int Y = dims[1], Z = dims[2];
    const int64_t V = (int64_t)dims[0] * Y * Z;
    double* e = NULL;
    set_threads(nthreads);
    if (c > 0) {
        e = (double*)calloc((size_t)V, sizeof(double));
#pragma omp parallel for schedule(static)
        for (int64_t v = (int64_t)x0 * Y * Z; v < (int64_t)x1 * Y * Z; ++v) {
            double s = 0.0;
            for (int k = 0; k < c; ++k) s += (double)grad_feats[v * c + k] * grid_feats[v * c + k];
            e[v] = s;
        }
    }
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t g = 0; g < n; ++g) {
        double gm[3] = {0, 0, 0}, gc[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0}, go = 0.0;
        double* gf = (c > 0) ? grad_features + g * (int64_t)c : NULL;
        if (gf) for (int k = 0; k < c; ++k) gf[k] = 0.0;
        int xa = lb[g * 3] > x0 ? lb[g * 3] : x0;
        int xb = ub[g * 3] < x1 - 1 ? ub[g * 3] : x1 - 1;
        if (xa <= xb) {
            double p[9];
            inverse3_d(cov + g * 9, p);
            double o = (double)opacity[g];
            const float* f = (c > 0) ? features + g * (int64_t)c : NULL;
            for (int x = xa; x <= xb; ++x)
                for (int y = lb[g * 3 + 1]; y <= ub[g * 3 + 1]; ++y)
                    for (int z = lb[g * 3 + 2]; z <= ub[g * 3 + 2]; ++z) {
                        double d[3] = {vlo[0] + (x + 0.5) * vsize[0] - (double)means[g * 3 + 0],
                                       vlo[1] + (y + 0.5) * vsize[1] - (double)means[g * 3 + 1],
                                       vlo[2] + (z + 0.5) * vsize[2] - (double)means[g * 3 + 2]};
                        double pd[3], ptd[3], maha = 0.0;
                        for (int i = 0; i < 3; ++i) {
                            pd[i] = p[i * 3 + 0] * d[0] + p[i * 3 + 1] * d[1] + p[i * 3 + 2] * d[2];
                            ptd[i] = p[0 * 3 + i] * d[0] + p[1 * 3 + i] * d[1] + p[2 * 3 + i] * d[2];
                            maha += d[i] * pd[i];
                        }
                        double ex = exp(-0.5 * maha);
                        double w = o * ex;
                        int64_t v = ((int64_t)x * Y + y) * Z + z;
                        double D = density[v];
                        double den = D > EPS_D ? D : EPS_D;
                        double a = (double)grad_density[v];
                        if (c > 0) {
                            const float* gv = grad_feats + v * c;
                            double s = 0.0;
                            for (int k = 0; k < c; ++k) s += (double)gv[k] * (double)f[k];
                            a += (s - (D >= EPS_D ? e[v] : 0.0)) / den;
                            double sc = w / den;
                            for (int k = 0; k < c; ++k) gf[k] += (double)gv[k] * sc;
                        }
                        double aw = a * w;
                        for (int i = 0; i < 3; ++i) gm[i] += aw * 0.5 * (pd[i] + ptd[i]);
                        for (int i = 0; i < 3; ++i)
                            for (int j = 0; j < 3; ++j) gc[i * 3 + j] += 0.5 * aw * ptd[i] * pd[j];
                        go += a * ex;
                    }
        }
        for (int i = 0; i < 3; ++i) grad_means[g * 3 + i] = gm[i];
        for (int k = 0; k < 9; ++k) grad_cov[g * 9 + k] = gc[k];
        grad_opacity[g] = go;
    }
    free(e);
}
