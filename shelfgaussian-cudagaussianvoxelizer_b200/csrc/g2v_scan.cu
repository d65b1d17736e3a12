// g2v_scan.cu -- exclusive prefix sum of int32 counts: one block for up to 64k counts, else three
// kernels (reduce, scan of block sums, scan + write).
//
// Used for the Gaussian->Tile offsets (N+1 entries, replacing the CUB InclusiveSum + memset of
// src/cuda_gaussian_voxelizer.cu:1608-1615), the per-tile offsets of the Tile->Gaussian map and the
// per-Gaussian block offsets of the backward.  Sums are carried in int64 so that a total beyond the
// int32 range of the maps can be detected by the caller.
#include "g2v_internal.cuh"

namespace g2v {

namespace {
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;  // 2048 counts per block

__device__ __forceinline__ int64_t warp_inclusive(int64_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Exclusive scan of one value per thread over the block; returns the block total through *total.
template <int THREADS>
__device__ __forceinline__ int64_t block_exclusive(int64_t v, int64_t* total) {
    __shared__ int64_t warp_sums[THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t inc = warp_inclusive(v);
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int64_t w = lane < THREADS / 32 ? warp_sums[lane] : 0;
        w = warp_inclusive(w);
        if (lane < THREADS / 32) warp_sums[lane] = w;
    }
    __syncthreads();
    const int64_t before = warp == 0 ? 0 : warp_sums[warp - 1];
    *total = warp_sums[THREADS / 32 - 1];
    __syncthreads();
    return before + inc - v;
}

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const int32_t* __restrict__ in, int64_t n,
                                                                   int64_t* __restrict__ block_sums) {
    const int64_t base = blockIdx.x * (int64_t)kScanTile;
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k * kScanThreads + threadIdx.x;
        if (i < n) s += in[i];
    }
    int64_t tot;
    block_exclusive<kScanThreads>(s, &tot);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = tot;
}

// One block of 1024 threads scans the block sums in place (exclusive) and stores the grand total.
__global__ void __launch_bounds__(1024) scan_block_sums_kernel(int64_t* __restrict__ sums, int64_t nb,
                                                               int64_t* __restrict__ total) {
    int64_t carry = 0;
    for (int64_t base = 0; base < nb; base += 1024) {
        const int64_t i = base + threadIdx.x;
        const int64_t v = i < nb ? sums[i] : 0;
        int64_t chunk;
        const int64_t ex = block_exclusive<1024>(v, &chunk);
        if (i < nb) sums[i] = carry + ex;
        carry += chunk;
    }
    if (threadIdx.x == 0) *total = carry;
}

// cap >= 0: every offset is clamped to cap (the capacity of the arrays the offsets index) and a total
// above it sets kErrCapacity in *err, so that a capacity chosen by the caller in advance can never be
// overrun (the results are then flagged invalid instead).
__global__ void __launch_bounds__(kScanThreads) scan_write_kernel(const int32_t* __restrict__ in, int64_t n,
                                                                  const int64_t* __restrict__ block_offsets,
                                                                  const int64_t* __restrict__ total,
                                                                  int32_t* __restrict__ out, int64_t cap,
                                                                  int* __restrict__ err) {
    // blocked arrangement: thread t owns items [base + t*kScanItems, +kScanItems)
    __shared__ int32_t stage[kScanTile];
    const int64_t base = blockIdx.x * (int64_t)kScanTile;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k * kScanThreads + threadIdx.x;
        stage[k * kScanThreads + threadIdx.x] = i < n ? in[i] : 0;
    }
    __syncthreads();
    int32_t v[kScanItems];
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = stage[threadIdx.x * kScanItems + k];
        s += v[k];
    }
    int64_t tot;
    int64_t run = block_offsets[blockIdx.x] + block_exclusive<kScanThreads>(s, &tot);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        stage[threadIdx.x * kScanItems + k] = static_cast<int32_t>(cap >= 0 && run > cap ? cap : run);
        run += v[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k * kScanThreads + threadIdx.x;
        if (i < n) out[i] = stage[k * kScanThreads + threadIdx.x];
    }
    if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
        const int64_t t = *total;
        out[n] = static_cast<int32_t>(cap >= 0 && t > cap ? cap : t);
        if (cap >= 0 && t > cap && err) atomicOr(err, kErrCapacity);
    }
}

// Up to kSmallScan counts (the per-Gaussian and per-cell counts of a scene of up to 64k Gaussians or
// cells): one block of 1024 threads scans them in chunks of 8192 with a running carry, one launch
// instead of three.  Same results as the three-kernel path (integer sums), including the clamp to cap.
constexpr int kSmallThreads = 1024;
constexpr int kSmallChunk = kSmallThreads * kScanItems;  // 8192 counts, 32 KB of shared memory
constexpr int64_t kSmallScan = 8 * kSmallChunk;

__global__ void __launch_bounds__(kSmallThreads) scan_small_kernel(const int32_t* __restrict__ in, int64_t n,
                                                                   int32_t* __restrict__ out,
                                                                   int64_t* __restrict__ total, int64_t cap,
                                                                   int* __restrict__ err) {
    __shared__ int32_t stage[kSmallChunk];
    int64_t carry = 0;
    for (int64_t base = 0; base < n; base += kSmallChunk) {
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            const int64_t i = base + k * kSmallThreads + threadIdx.x;
            stage[k * kSmallThreads + threadIdx.x] = i < n ? in[i] : 0;
        }
        __syncthreads();
        int32_t v[kScanItems];
        int64_t s = 0;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            v[k] = stage[threadIdx.x * kScanItems + k];
            s += v[k];
        }
        int64_t tot;
        int64_t run = carry + block_exclusive<kSmallThreads>(s, &tot);  // ends with a barrier: stage is free
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            stage[threadIdx.x * kScanItems + k] = static_cast<int32_t>(cap >= 0 && run > cap ? cap : run);
            run += v[k];
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            const int64_t i = base + k * kSmallThreads + threadIdx.x;
            if (i < n) out[i] = stage[k * kSmallThreads + threadIdx.x];
        }
        carry += tot;
        __syncthreads();  // the next chunk overwrites stage
    }
    if (threadIdx.x == 0) {
        out[n] = static_cast<int32_t>(cap >= 0 && carry > cap ? cap : carry);
        *total = carry;
        if (cap >= 0 && carry > cap && err) atomicOr(err, kErrCapacity);
    }
}

__global__ void scan_empty_kernel(int32_t* out, int64_t* total) {
    out[0] = 0;
    *total = 0;
}
}  // namespace

size_t scan_workspace_bytes(int64_t n) {
    const int64_t nb = (n + kScanTile - 1) / kScanTile;
    return ((size_t)(nb > 0 ? nb : 1) * sizeof(int64_t) + 255) & ~size_t(255);
}

int launch_exclusive_scan(const int32_t* counts, int64_t n, int32_t* out, int64_t* total, void* ws,
                          cudaStream_t s, int64_t cap, int* err) {
    if (n == 0) {
        G2V_TIMED("scan_empty_kernel", s, scan_empty_kernel<<<1, 1, 0, s>>>(out, total));
        G2V_LAUNCH_CHECK("scan_empty_kernel");
        return 0;
    }
    if (n <= kSmallScan) {
        G2V_TIMED("scan_small_kernel", s,
                  scan_small_kernel<<<1, kSmallThreads, 0, s>>>(counts, n, out, total, cap, err));
        G2V_LAUNCH_CHECK("scan_small_kernel");
        return 0;
    }
    const int64_t nb = (n + kScanTile - 1) / kScanTile;
    int64_t* sums = static_cast<int64_t*>(ws);
    G2V_TIMED("scan_reduce_kernel", s, scan_reduce_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(counts, n, sums));
    G2V_LAUNCH_CHECK("scan_reduce_kernel");
    G2V_TIMED("scan_block_sums_kernel", s, scan_block_sums_kernel<<<1, 1024, 0, s>>>(sums, nb, total));
    G2V_LAUNCH_CHECK("scan_block_sums_kernel");
    G2V_TIMED("scan_write_kernel", s, scan_write_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(counts, n, sums, total, out, cap, err));
    G2V_LAUNCH_CHECK("scan_write_kernel");
    return 0;
}

}  // namespace g2v
