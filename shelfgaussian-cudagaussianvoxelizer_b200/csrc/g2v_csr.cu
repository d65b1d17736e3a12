// g2v_csr.cu -- Gaussian->cell and cell->Gaussian maps.
//
// A "cell" is a box of cx*cy*cz tiles.  With a 1x1x1 cell this builds the reference's maps:
//   * the Gaussian->Tile CSR tile ids (FillG2TKernel, src/cuda_gaussian_voxelizer.cu:228-286): the tile
//     box of each Gaussian enumerated x-major, tile id (tx*Ty+ty)*Tz+tz, at g2t_offsets[g];
//   * the Tile->Gaussian CSR (cu:1675-1772: stable radix sort by tile id + run-length encoding + scan):
//     here a count per tile, an exclusive scan, an atomic scatter and a per-tile sort of the Gaussian
//     ids, which gives the same lists (Gaussian ids ascending in every tile) over all tiles instead of
//     the active ones only.
// Larger cells (blocks of tiles) give the block->Gaussian lists of the backward's feature-gradient
// pass.  Only cells whose x index lies in [cell_x_begin, cell_x_end) are counted and listed.
#include <climits>

#include "g2v_internal.cuh"

namespace g2v {

namespace {

struct CellBox {
    int lo[3], hi[3], ext[3];
    int count;
};

__device__ __forceinline__ bool cell_box(const int32_t* lb, const int32_t* ub, int64_t g, const int cell[3],
                                         CellBox& b) {
    int tlo[3], thi[3];
    if (!tile_box(lb, ub, g, tlo, thi)) return false;
    int cnt = 1;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        b.lo[a] = tlo[a] / cell[a];
        b.hi[a] = thi[a] / cell[a];
        b.ext[a] = b.hi[a] - b.lo[a] + 1;
        cnt *= b.ext[a];
    }
    b.count = cnt;
    return true;
}

// Warp per Gaussian.  Writes the reference's G2T tile ids (when g2t_tile_ids != nullptr) and counts
// every listed cell.  per_gaussian (optional) receives the number of cells of the Gaussian's cell box.
__global__ void __launch_bounds__(256) cells_count_kernel(const int32_t* __restrict__ lb,
                                                          const int32_t* __restrict__ ub, int64_t n, Grid G,
                                                          int cx, int cy, int cz, int ncy, int ncz,
                                                          int cell_x_begin, int cell_x_end,
                                                          const int32_t* __restrict__ g2t_offsets,
                                                          int32_t* __restrict__ g2t_tile_ids, int64_t g2t_cap,
                                                          int32_t* __restrict__ cell_counts,
                                                          int32_t* __restrict__ per_gaussian) {
    const int64_t g = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (g >= n) return;
    const int cell[3] = {cx, cy, cz};
    CellBox b;
    const bool ok = cell_box(lb, ub, g, cell, b);
    if (per_gaussian && lane == 0) per_gaussian[g] = ok ? b.count : 0;
    if (!ok) return;
    const int dyz = b.ext[1] * b.ext[2];
    const int64_t base = g2t_tile_ids ? (int64_t)g2t_offsets[g] : 0;
    for (int i = lane; i < b.count; i += 32) {
        const int lx = i / dyz;
        const int r = i - lx * dyz;
        const int ly = r / b.ext[2];
        const int lz = r - ly * b.ext[2];
        const int x = b.lo[0] + lx, y = b.lo[1] + ly, z = b.lo[2] + lz;
        // the offsets come from the caller: never write past the M entries it allocated
        if (g2t_tile_ids && base + i < g2t_cap) g2t_tile_ids[base + i] = (x * G.tiles[1] + y) * G.tiles[2] + z;
        if (x >= cell_x_begin && x < cell_x_end) {
            const int c = ((x - cell_x_begin) * ncy + y) * ncz + z;
            atomicAdd(&cell_counts[c], 1);
        }
    }
}

// Warp per Gaussian: appends g to the list of every listed cell of its cell box (unordered).
__global__ void __launch_bounds__(256) cells_scatter_kernel(const int32_t* __restrict__ lb,
                                                            const int32_t* __restrict__ ub, int64_t n, int cx,
                                                            int cy, int cz, int ncy, int ncz, int cell_x_begin,
                                                            int cell_x_end, const int32_t* __restrict__ cell_offsets,
                                                            int32_t* __restrict__ cursor,
                                                            int32_t* __restrict__ lists) {
    const int64_t g = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (g >= n) return;
    const int cell[3] = {cx, cy, cz};
    CellBox b;
    if (!cell_box(lb, ub, g, cell, b)) return;
    const int xa = max(b.lo[0], cell_x_begin), xb = min(b.hi[0], cell_x_end - 1);
    if (xa > xb) return;
    const int nx = xb - xa + 1;
    const int dyz = b.ext[1] * b.ext[2];
    const int cnt = nx * dyz;
    for (int i = lane; i < cnt; i += 32) {
        const int lx = i / dyz;
        const int r = i - lx * dyz;
        const int ly = r / b.ext[2];
        const int lz = r - ly * b.ext[2];
        const int c = ((xa + lx - cell_x_begin) * ncy + b.lo[1] + ly) * ncz + b.lo[2] + lz;
        const int pos = atomicAdd(&cursor[c], 1);
        // offsets clamped to a capacity (capped calls): a full cell drops the entries beyond it
        if (cell_offsets[c] + pos < cell_offsets[c + 1]) lists[cell_offsets[c] + pos] = (int32_t)g;
    }
}

__device__ __forceinline__ int64_t block_exclusive_i64(int64_t v, int64_t* total, int64_t* warp_sums) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int64_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int64_t w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        if (lane < nw) warp_sums[lane] = w;
    }
    __syncthreads();
    const int64_t before = warp == 0 ? 0 : warp_sums[warp - 1];
    *total = warp_sums[nw - 1];
    __syncthreads();
    return before + inc - v;
}

constexpr int kSortThreads = 256;
constexpr int kBitonicMax = 1024;
constexpr int kBitmapBits = 1 << 16;                 // ids per bitmap pass
constexpr int kBitmapWords = kBitmapBits / 32;       // 2048 words, 8 per thread

// Ordered bitmap compaction of the k distinct ids in[0..k) into out[0..k), in passes of 65536 ids over
// [0, n_ids); `bits` is kBitmapWords words of shared memory.
__device__ void sort_ids_bitmap(const int32_t* __restrict__ in, int32_t* __restrict__ out, int k, int64_t n_ids,
                                unsigned* bits, int64_t* warp_sums);

// One block per cell: writes the cell's Gaussian ids in ascending order from `in` to `out`.
// Small lists use a bitonic sort in shared memory; long lists an ordered bitmap compaction over the
// id range in passes of 65536 ids (the ids of one cell are distinct).
__global__ void __launch_bounds__(kSortThreads) cells_sort_kernel(const int32_t* __restrict__ offsets,
                                                                  const int32_t* __restrict__ in,
                                                                  int32_t* __restrict__ out, int64_t n_ids) {
    __shared__ int32_t sh[kBitmapWords > kBitonicMax ? kBitmapWords : kBitonicMax];
    __shared__ int64_t warp_sums[kSortThreads / 32];
    const int cell = blockIdx.x;
    const int s = offsets[cell], e = offsets[cell + 1];
    const int k = e - s;
    if (k <= 0) return;
    if (k == 1) {
        if (threadIdx.x == 0) out[s] = in[s];
        return;
    }
    if (k <= kBitonicMax) {
        int p = 2;
        while (p < k) p <<= 1;
        for (int i = threadIdx.x; i < p; i += kSortThreads) sh[i] = i < k ? in[s + i] : INT_MAX;
        __syncthreads();
        for (int kk = 2; kk <= p; kk <<= 1) {
            for (int j = kk >> 1; j > 0; j >>= 1) {
                for (int i = threadIdx.x; i < p; i += kSortThreads) {
                    const int ixj = i ^ j;
                    if (ixj > i) {
                        const int a = sh[i], b = sh[ixj];
                        const bool up = (i & kk) == 0;
                        if ((a > b) == up) {
                            sh[i] = b;
                            sh[ixj] = a;
                        }
                    }
                }
                __syncthreads();
            }
        }
        for (int i = threadIdx.x; i < k; i += kSortThreads) out[s + i] = sh[i];
        return;
    }
    sort_ids_bitmap(in + s, out + s, k, n_ids, reinterpret_cast<unsigned*>(sh), warp_sums);
}

__device__ void sort_ids_bitmap(const int32_t* __restrict__ in, int32_t* __restrict__ out, int k, int64_t n_ids,
                                unsigned* bits, int64_t* warp_sums) {
    int64_t written = 0;
    for (int64_t c0 = 0; c0 < n_ids; c0 += kBitmapBits) {
        for (int w = threadIdx.x; w < kBitmapWords; w += kSortThreads) bits[w] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < k; i += kSortThreads) {
            const int64_t id = in[i];
            if (id >= c0 && id < c0 + kBitmapBits) {
                const int r = (int)(id - c0);
                atomicOr(&bits[r >> 5], 1u << (r & 31));
            }
        }
        __syncthreads();
        constexpr int per = kBitmapWords / kSortThreads;  // 8 consecutive words per thread
        unsigned mine[per];
        int cnt = 0;
#pragma unroll
        for (int q = 0; q < per; ++q) {
            mine[q] = bits[threadIdx.x * per + q];
            cnt += __popc(mine[q]);
        }
        int64_t tot;
        int64_t pos = written + block_exclusive_i64(cnt, &tot, warp_sums);
#pragma unroll
        for (int q = 0; q < per; ++q) {
            unsigned m = mine[q];
            while (m) {
                const int bpos = __ffs(m) - 1;
                m &= m - 1;
                out[pos++] = (int32_t)(c0 + (int64_t)(threadIdx.x * per + q) * 32 + bpos);
            }
        }
        written += tot;
        __syncthreads();
    }
}

constexpr int kSortXMax = 4096;  // 32 KB of 64-bit keys
static_assert(kSortXMax * 2 >= kBitmapWords, "the x-order sort's keys also hold the bitmap");

// One block per cell: writes the cell's Gaussian ids ordered by (voxel box lower x, id), so that the
// Gaussians of a slot range of the feature-gradient pass lie close together along x and its steps
// outside their boxes can be skipped.  Lists longer than kSortXMax keep the ascending id order.
__global__ void __launch_bounds__(kSortThreads) cells_sort_x_kernel(const int32_t* __restrict__ offsets,
                                                                    const int32_t* __restrict__ in,
                                                                    const int32_t* __restrict__ lb,
                                                                    int32_t* __restrict__ out, int64_t n_ids) {
    __shared__ unsigned long long sh[kSortXMax];
    __shared__ int64_t warp_sums[kSortThreads / 32];
    const int cell = blockIdx.x;
    const int s = offsets[cell], e = offsets[cell + 1];
    const int k = e - s;
    if (k <= 0) return;
    if (k == 1) {
        if (threadIdx.x == 0) out[s] = in[s];
        return;
    }
    if (k > kSortXMax) {
        sort_ids_bitmap(in + s, out + s, k, n_ids, reinterpret_cast<unsigned*>(sh), warp_sums);
        return;
    }
    int p = 2;
    while (p < k) p <<= 1;
    for (int i = threadIdx.x; i < p; i += kSortThreads) {
        unsigned long long key = ~0ull;
        if (i < k) {
            const int g = in[s + i];
            key = ((unsigned long long)(uint32_t)lb[(int64_t)g * 3] << 32) | (uint32_t)g;
        }
        sh[i] = key;
    }
    __syncthreads();
    for (int kk = 2; kk <= p; kk <<= 1) {
        for (int j = kk >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < p; i += kSortThreads) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = sh[i], b = sh[ixj];
                    const bool up = (i & kk) == 0;
                    if ((a > b) == up) {
                        sh[i] = b;
                        sh[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < k; i += kSortThreads) out[s + i] = (int32_t)(uint32_t)sh[i];
}

}  // namespace

// Builds the cell->Gaussian CSR for the cells with x in [cell_x_begin, cell_x_end) of a cell grid of
// (ncx, ncy, ncz) cells of (cx, cy, cz) tiles.  Also writes the reference's G2T tile ids when
// g2t_tile_ids != nullptr (1x1x1 cells) and the per-Gaussian cell count when per_gaussian != nullptr.
// Buffers: counts (ncells, zeroed here), cell_offsets (ncells+1), unsorted and lists (>= pairs),
// scan_ws (scan_workspace_bytes(ncells)), total (1 int64).  x_order: each list ordered by (voxel box
// lower x, id) instead of by id (lists of at most 4096 Gaussians).
int build_cell_lists(const int32_t* lb, const int32_t* ub, int64_t n, const Grid& G, const int cell[3],
                     const int ncells_dim[3], int cell_x_begin, int cell_x_end, const int32_t* g2t_offsets,
                     int32_t* g2t_tile_ids, int64_t g2t_cap, int32_t* per_gaussian, int32_t* counts, int32_t* cell_offsets,
                     int32_t* unsorted, int32_t* lists, void* scan_ws, int64_t* total, cudaStream_t s,
                     int64_t list_cap, int* err, bool x_order) {
    const int nx = cell_x_end - cell_x_begin;
    const int64_t ncells = (int64_t)nx * ncells_dim[1] * ncells_dim[2];
    if (ncells > 0) G2V_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * (size_t)ncells, s));
    if (n > 0) {
        const int64_t threads = n * 32;
        const unsigned blocks = (unsigned)((threads + 255) / 256);
        G2V_TIMED("cells_count_kernel", s, cells_count_kernel<<<blocks, 256, 0, s>>>(lb, ub, n, G, cell[0], cell[1], cell[2], ncells_dim[1],
                                                  ncells_dim[2], cell_x_begin, cell_x_end, g2t_offsets,
                                                  g2t_tile_ids, g2t_cap, counts, per_gaussian));
        G2V_LAUNCH_CHECK("cells_count_kernel");
    }
    int rc = launch_exclusive_scan(counts, ncells, cell_offsets, total, scan_ws, s, list_cap, err);
    if (rc) return rc;
    if (n > 0 && ncells > 0) {
        G2V_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * (size_t)ncells, s));
        const int64_t threads = n * 32;
        const unsigned blocks = (unsigned)((threads + 255) / 256);
        G2V_TIMED("cells_scatter_kernel", s, cells_scatter_kernel<<<blocks, 256, 0, s>>>(lb, ub, n, cell[0], cell[1], cell[2], ncells_dim[1],
                                                    ncells_dim[2], cell_x_begin, cell_x_end, cell_offsets,
                                                    counts, unsorted));
        G2V_LAUNCH_CHECK("cells_scatter_kernel");
        if (x_order) {
            G2V_TIMED("cells_sort_x_kernel", s,
                      cells_sort_x_kernel<<<(unsigned)ncells, kSortThreads, 0, s>>>(cell_offsets, unsorted, lb, lists, n));
            G2V_LAUNCH_CHECK("cells_sort_x_kernel");
        } else {
            G2V_TIMED("cells_sort_kernel", s, cells_sort_kernel<<<(unsigned)ncells, kSortThreads, 0, s>>>(cell_offsets, unsorted, lists, n));
            G2V_LAUNCH_CHECK("cells_sort_kernel");
        }
    }
    return 0;
}

// The reference's G2T tile ids only (FillG2TKernel, cu:228-286), without the Tile->Gaussian lists:
// the tensor-core splat works on its own unit lists.  Nothing is counted (empty listing range).
int fill_g2t(const int32_t* lb, const int32_t* ub, int64_t n, const Grid& G, const int32_t* g2t_offsets,
             int32_t* g2t_tile_ids, int64_t g2t_cap, cudaStream_t s) {
    if (n == 0) return 0;
    const int64_t threads = n * 32;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    G2V_TIMED("cells_count_kernel", s, cells_count_kernel<<<blocks, 256, 0, s>>>(lb, ub, n, G, 1, 1, 1, 1, 1, 0, 0,
                                                                              g2t_offsets, g2t_tile_ids, g2t_cap,
                                                                              nullptr, nullptr));
    G2V_LAUNCH_CHECK("cells_count_kernel");
    return 0;
}

// Per-Gaussian cell counts only (for sizing the backward's block partial rows).
int count_gaussian_cells(const int32_t* lb, const int32_t* ub, int64_t n, const Grid& G, const int cell[3],
                         int32_t* per_gaussian, int32_t* dummy_counts, cudaStream_t s) {
    if (n == 0) return 0;
    const int64_t threads = n * 32;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    // an empty x range: nothing is counted, only per_gaussian is written
    G2V_TIMED("cells_count_kernel", s, cells_count_kernel<<<blocks, 256, 0, s>>>(lb, ub, n, G, cell[0], cell[1], cell[2], 1, 1, 0, 0, nullptr,
                                              nullptr, 0, dummy_counts, per_gaussian));
    G2V_LAUNCH_CHECK("cells_count_kernel");
    return 0;
}

}  // namespace g2v
