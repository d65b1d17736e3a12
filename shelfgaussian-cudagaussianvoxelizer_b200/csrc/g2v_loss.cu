// g2v_loss.cu -- voxel-wise feature cosine loss (the consumer of grid_feats), forward and backward.
//
// Reference: src/cuda_feats_loss.cu of the voxelizer project (VoxelCosineLossKernel :45-101,
// ReduceLossAndCountKernel :104-143, CudaFeatsCosinelossForward :146-225, CosineLossBackwardKernel
// :228-289, CudaFeatsCosinelossBackward :311-366).  For voxel v, valid when occ_mask[v] && label[v] > 0,
// with p = grid_feats[v], g = gt_feats[v]:
//     a = sqrt(max(|p|^2, eps)), b = sqrt(max(|g|^2, eps)), D = a b + eps,  loss_v = 1 - p.g / D
//     loss = sum_valid loss_v / count            (0 when count == 0)
//     dloss/dp = grad_out * (1/count) * (-g / D + [|p|^2 > eps] (p.g) b / (a D^2) p),  0 for invalid voxels
// with eps = 1e-6 (include/utils.cuh:80).
//
// Both passes are HBM-bound.  Algorithmic bytes: the forward reads label + mask of every voxel (5 B) and
// p, g of the valid ones (8 C B); the backward reads the same and writes the gradient of every voxel
// (4 C B).  A group of G lanes (a power of two <= 32, sized to the row) owns one voxel: 16-byte loads
// over the channels when C % 4 == 0, sums by an xor butterfly inside the group.  The backward keeps the
// row in registers between the sums and the gradient (no second read) up to 8 elements per lane, and
// invalid voxels read nothing and write zeros.  The forward's total is taken in a fixed order (lane ->
// warp -> CTA partial -> one CTA), so it is deterministic; the count and the upstream gradient stay on
// the device (no host synchronisation in either direction).
#include <algorithm>

#include "g2v_internal.cuh"

namespace g2v {

namespace {
constexpr int kLossThreads = 256;  // 8 warps
constexpr int kLossWarps = kLossThreads / 32;
constexpr int kMaxLossParts = 2048;  // CTA partials of the forward (grid <= 8 CTAs per SM, capped)

template <bool kVec>
struct Row;
template <>
struct Row<true> {
    using E = float4;
    static __device__ __forceinline__ E zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
    static __device__ __forceinline__ void acc(const E& x, const E& y, float& d, float& a, float& b) {
        d = fmaf(x.x, y.x, d); d = fmaf(x.y, y.y, d); d = fmaf(x.z, y.z, d); d = fmaf(x.w, y.w, d);
        a = fmaf(x.x, x.x, a); a = fmaf(x.y, x.y, a); a = fmaf(x.z, x.z, a); a = fmaf(x.w, x.w, a);
        b = fmaf(y.x, y.x, b); b = fmaf(y.y, y.y, b); b = fmaf(y.z, y.z, b); b = fmaf(y.w, y.w, b);
    }
    static __device__ __forceinline__ E grad(float c1, const E& y, float c2, const E& x) {
        return make_float4(c1 * y.x + c2 * x.x, c1 * y.y + c2 * x.y, c1 * y.z + c2 * x.z, c1 * y.w + c2 * x.w);
    }
};
template <>
struct Row<false> {
    using E = float;
    static __device__ __forceinline__ E zero() { return 0.f; }
    static __device__ __forceinline__ void acc(E x, E y, float& d, float& a, float& b) {
        d = fmaf(x, y, d);
        a = fmaf(x, x, a);
        b = fmaf(y, y, b);
    }
    static __device__ __forceinline__ E grad(float c1, E y, float c2, E x) { return c1 * y + c2 * x; }
};

// Sum over the G-lane group (every lane of the warp executes it; G is warp-uniform).
__device__ __forceinline__ void group_sum3(float& d, float& a, float& b, int G) {
    for (int o = G >> 1; o > 0; o >>= 1) {
        d += __shfl_xor_sync(0xffffffffu, d, o);
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
}

__device__ __forceinline__ bool voxel_valid(const float* label, const uint8_t* mask, int64_t v, int64_t V) {
    return v < V && mask[v] != 0 && label[v] > 0.f;
}

// Forward: per-CTA partial (sum of loss_v, count) of the voxels the CTA visits.
// gl2 = log2(G); n = row length in elements of Row<kVec>::E.
template <bool kVec>
__global__ void __launch_bounds__(kLossThreads) cosine_loss_fwd_kernel(
    const float* __restrict__ label, const uint8_t* __restrict__ mask, const float* __restrict__ p,
    const float* __restrict__ g, int64_t V, int n, int gl2, float* __restrict__ part_loss,
    int* __restrict__ part_count) {
    using R = Row<kVec>;
    using E = typename R::E;
    __shared__ float sl[kLossWarps];
    __shared__ int sc[kLossWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = 1 << gl2, l = lane & (G - 1), per_warp = 32 >> gl2;
    const E* P = reinterpret_cast<const E*>(p);
    const E* Q = reinterpret_cast<const E*>(g);
    float lsum = 0.f;
    int cnt = 0;
    const int64_t stride = (int64_t)gridDim.x * kLossWarps * per_warp;
    for (int64_t base = ((int64_t)blockIdx.x * kLossWarps + warp) * per_warp; base < V; base += stride) {
        const int64_t v = base + (lane >> gl2);
        const bool valid = voxel_valid(label, mask, v, V);
        float d = 0.f, a = 0.f, b = 0.f;
        if (valid) {
            const E* pr = P + v * n;
            const E* gr = Q + v * n;
#pragma unroll 4
            for (int c = l; c < n; c += G) R::acc(__ldg(pr + c), __ldg(gr + c), d, a, b);
        }
        group_sum3(d, a, b, G);
        if (valid && l == 0) {
            const float pn = sqrtf(fmaxf(a, kEps)), gn = sqrtf(fmaxf(b, kEps));
            lsum += 1.f - d / (pn * gn + kEps);
            ++cnt;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
        cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    }
    if (lane == 0) {
        sl[warp] = lsum;
        sc[warp] = cnt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        int c = 0;
#pragma unroll
        for (int w = 0; w < kLossWarps; ++w) {
            s += sl[w];
            c += sc[w];
        }
        part_loss[blockIdx.x] = s;
        part_count[blockIdx.x] = c;
    }
}

// One CTA: the partials in a fixed order -> mean loss and count.
__global__ void __launch_bounds__(kLossThreads) cosine_loss_final_kernel(const float* __restrict__ part_loss,
                                                                         const int* __restrict__ part_count,
                                                                         int nparts, float* __restrict__ loss,
                                                                         int* __restrict__ count) {
    __shared__ float sl[kLossThreads];
    __shared__ int sc[kLossThreads];
    float s = 0.f;
    int c = 0;
    for (int i = threadIdx.x; i < nparts; i += kLossThreads) {
        s += part_loss[i];
        c += part_count[i];
    }
    sl[threadIdx.x] = s;
    sc[threadIdx.x] = c;
    __syncthreads();
    for (int h = kLossThreads / 2; h > 0; h >>= 1) {
        if (threadIdx.x < h) {
            sl[threadIdx.x] += sl[threadIdx.x + h];
            sc[threadIdx.x] += sc[threadIdx.x + h];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *loss = sc[0] > 0 ? sl[0] / (float)sc[0] : 0.f;
        *count = sc[0];
    }
}

// Backward.  kK > 0: the row stays in registers (kK elements per lane, n <= kK * G); kK == 0: any n,
// the row is read a second time for the gradient.
template <bool kVec, int kK>
__global__ void __launch_bounds__(kLossThreads) cosine_loss_bwd_kernel(
    const float* __restrict__ grad_out, const int* __restrict__ count_dev, int count_host,
    const float* __restrict__ label, const uint8_t* __restrict__ mask, const float* __restrict__ p,
    const float* __restrict__ g, int64_t V, int n, int gl2, float* __restrict__ gp) {
    using R = Row<kVec>;
    using E = typename R::E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = 1 << gl2, l = lane & (G - 1), per_warp = 32 >> gl2;
    const int cnt = count_dev ? *count_dev : count_host;
    const float inv_count = cnt > 0 ? 1.0f / (float)cnt : 0.0f;
    const float scale = *grad_out * inv_count;
    const E* P = reinterpret_cast<const E*>(p);
    const E* Q = reinterpret_cast<const E*>(g);
    E* O = reinterpret_cast<E*>(gp);
    const int64_t stride = (int64_t)gridDim.x * kLossWarps * per_warp;
    for (int64_t base = ((int64_t)blockIdx.x * kLossWarps + warp) * per_warp; base < V; base += stride) {
        const int64_t v = base + (lane >> gl2);
        const bool valid = voxel_valid(label, mask, v, V);
        const E* pr = P + v * n;
        const E* gr = Q + v * n;
        E xs[kK > 0 ? kK : 1], ys[kK > 0 ? kK : 1];
        float d = 0.f, a = 0.f, b = 0.f;
        if (kK > 0) {
#pragma unroll
            for (int k = 0; k < (kK > 0 ? kK : 1); ++k) {
                const int c = l + k * G;
                const bool in = valid && c < n;
                xs[k] = in ? __ldg(pr + c) : R::zero();
                ys[k] = in ? __ldg(gr + c) : R::zero();
                R::acc(xs[k], ys[k], d, a, b);
            }
        } else if (valid) {
#pragma unroll 4
            for (int c = l; c < n; c += G) R::acc(__ldg(pr + c), __ldg(gr + c), d, a, b);
        }
        group_sum3(d, a, b, G);
        if (v >= V) continue;
        E* out = O + v * n;
        if (!valid) {
            for (int c = l; c < n; c += G) out[c] = R::zero();
            continue;
        }
        const float ra = sqrtf(fmaxf(a, kEps)), rb = sqrtf(fmaxf(b, kEps));
        const float D = ra * rb + kEps;
        const float c1 = (-1.0f / D) * scale;                               // multiplies g
        const float c2 = (a > kEps ? (d * rb) / (ra * D * D) : 0.0f) * scale;  // multiplies p
        if (kK > 0) {
#pragma unroll
            for (int k = 0; k < (kK > 0 ? kK : 1); ++k) {
                const int c = l + k * G;
                if (c < n) out[c] = R::grad(c1, ys[k], c2, xs[k]);
            }
        } else {
            for (int c = l; c < n; c += G) out[c] = R::grad(c1, __ldg(gr + c), c2, __ldg(pr + c));
        }
    }
}

int sm_count() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return sms;
}

struct RowShape {
    bool vec;
    int n;    // row length in elements (float4 when vec)
    int gl2;  // log2 of the lanes per voxel
    int grid;
};

RowShape row_shape(int64_t V, int C, const void* a, const void* b, const void* c) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    RowShape r;
    r.vec = C % 4 == 0 && al(a) && al(b) && al(c);
    r.n = r.vec ? C / 4 : C;
    r.gl2 = 0;
    while (r.gl2 < 5 && (1 << r.gl2) < r.n) ++r.gl2;
    const int64_t per_cta = (int64_t)kLossWarps * (32 >> r.gl2);
    const int64_t need = (V + per_cta - 1) / per_cta;
    r.grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, std::min(sm_count() * 8, kMaxLossParts)));
    return r;
}

template <bool kVec>
void launch_bwd_k(int kk, int grid, const float* grad_out, const int* count_dev, int count_host, const float* label,
                  const uint8_t* mask, const float* p, const float* g, int64_t V, int n, int gl2, float* gp,
                  cudaStream_t s) {
#define G2V_LOSS_BWD(K)                                                                                          \
    G2V_TIMED("cosine_loss_bwd_kernel", s,                                                                      \
              (cosine_loss_bwd_kernel<kVec, K><<<grid, kLossThreads, 0, s>>>(grad_out, count_dev, count_host,   \
                                                                             label, mask, p, g, V, n, gl2, gp)))
    switch (kk) {
        case 1: G2V_LOSS_BWD(1); break;
        case 2: G2V_LOSS_BWD(2); break;
        case 4: G2V_LOSS_BWD(4); break;
        case 8: G2V_LOSS_BWD(8); break;
        default: G2V_LOSS_BWD(0); break;
    }
#undef G2V_LOSS_BWD
}
}  // namespace

size_t cosine_loss_workspace_bytes() { return (size_t)kMaxLossParts * (sizeof(float) + sizeof(int)); }

int launch_cosine_loss_fwd(const float* label, const uint8_t* mask, const float* p, const float* g, int64_t V, int C,
                           float* loss, int* count, void* ws, cudaStream_t s) {
    const RowShape r = row_shape(V, C, p, g, nullptr);
    float* part_loss = static_cast<float*>(ws);
    int* part_count = reinterpret_cast<int*>(part_loss + kMaxLossParts);
    if (r.vec)
        G2V_TIMED("cosine_loss_fwd_kernel", s,
                  (cosine_loss_fwd_kernel<true><<<r.grid, kLossThreads, 0, s>>>(label, mask, p, g, V, r.n, r.gl2,
                                                                                 part_loss, part_count)));
    else
        G2V_TIMED("cosine_loss_fwd_kernel", s,
                  (cosine_loss_fwd_kernel<false><<<r.grid, kLossThreads, 0, s>>>(label, mask, p, g, V, r.n, r.gl2,
                                                                                  part_loss, part_count)));
    G2V_LAUNCH_CHECK("cosine_loss_fwd_kernel");
    G2V_TIMED("cosine_loss_final_kernel", s,
              (cosine_loss_final_kernel<<<1, kLossThreads, 0, s>>>(part_loss, part_count, r.grid, loss, count)));
    G2V_LAUNCH_CHECK("cosine_loss_final_kernel");
    return 0;
}

int launch_cosine_loss_bwd(const float* grad_out, const int* count_dev, int count_host, const float* label,
                           const uint8_t* mask, const float* p, const float* g, int64_t V, int C, float* gp,
                           cudaStream_t s) {
    if (V <= 0 || C <= 0) return 0;
    const RowShape r = row_shape(V, C, p, g, gp);
    const int G = 1 << r.gl2;
    const int need = (r.n + G - 1) / G;  // elements per lane
    const int kk = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 0;
    if (r.vec)
        launch_bwd_k<true>(kk, r.grid, grad_out, count_dev, count_host, label, mask, p, g, V, r.n, r.gl2, gp, s);
    else
        launch_bwd_k<false>(kk, r.grid, grad_out, count_dev, count_host, label, mask, p, g, V, r.n, r.gl2, gp, s);
    G2V_LAUNCH_CHECK("cosine_loss_bwd_kernel");
    return 0;
}

}  // namespace g2v
