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

// Valid flag of voxel v; both loads are issued unconditionally (no dependent branch between them).
__device__ __forceinline__ bool voxel_valid(const float* label, const uint8_t* mask, int64_t v, int64_t V) {
    if (v >= V) return false;
    const uint8_t m = __ldg(mask + v);
    const float l = __ldg(label + v);
    return m != 0 && l > 0.f;
}

// Per-warp list of a window's voxels (offsets 0..31): the valid ones in order, then the other in-range
// ones.  Returns the number of valid voxels; *ninv receives the number of the others.
__device__ __forceinline__ int window_list(int* list, bool valid, bool inrange, int lane, int* ninv) {
    const unsigned bal = __ballot_sync(0xffffffffu, valid);
    const unsigned inr = __ballot_sync(0xffffffffu, inrange);
    const unsigned below = (1u << lane) - 1u;
    const int nv = __popc(bal);
    __syncwarp();  // the previous window's list has been read
    if (valid) list[__popc(bal & below)] = lane;
    else if (inrange) list[nv + __popc(inr & ~bal & below)] = lane;
    __syncwarp();
    *ninv = __popc(inr & ~bal);
    return nv;
}

// Row slot of a lane: the voxel window of a warp is 32 consecutive voxels; the valid ones are dealt to
// the warp's S = 32 / G lane groups in order, S per round.  kK > 0: a lane holds kK
// elements of the row (element l + k G), all loads of a round issued before the sums; kK == 0: any
// row length, a strided loop.
template <bool kVec, int kK>
struct RowIO {
    using R = Row<kVec>;
    using E = typename R::E;
    static constexpr int kRegs = kK > 0 ? kK : 1;
    E x[kRegs], y[kRegs];

    __device__ __forceinline__ void sums(const E* pr, const E* gr, bool act, int l, int G, int n, float& d, float& a,
                                         float& b) {
        d = a = b = 0.f;
        if (kK > 0) {
#pragma unroll
            for (int k = 0; k < kRegs; ++k) {
                const int c = l + k * G;
                const bool in = act && c < n;
                x[k] = in ? __ldg(pr + c) : R::zero();
                y[k] = in ? __ldg(gr + c) : R::zero();
            }
#pragma unroll
            for (int k = 0; k < kRegs; ++k) R::acc(x[k], y[k], d, a, b);
        } else if (act) {
#pragma unroll 4
            for (int c = l; c < n; c += G) R::acc(__ldg(pr + c), __ldg(gr + c), d, a, b);
        }
    }

    __device__ __forceinline__ void write_grad(E* out, const E* pr, const E* gr, int l, int G, int n, float c1,
                                               float c2) {
        if (kK > 0) {
#pragma unroll
            for (int k = 0; k < kRegs; ++k) {
                const int c = l + k * G;
                if (c < n) out[c] = R::grad(c1, y[k], c2, x[k]);
            }
        } else {
            for (int c = l; c < n; c += G) out[c] = R::grad(c1, __ldg(gr + c), c2, __ldg(pr + c));
        }
    }

    static __device__ __forceinline__ void write_zero(E* out, int l, int G, int n) {
        if (kK > 0) {
#pragma unroll
            for (int k = 0; k < kRegs; ++k) {
                const int c = l + k * G;
                if (c < n) out[c] = R::zero();
            }
        } else {
            for (int c = l; c < n; c += G) out[c] = R::zero();
        }
    }
};

// Forward: per-CTA partial (sum of loss_v, count) of the voxel windows the CTA's warps visit.
template <bool kVec, int kK>
__global__ void __launch_bounds__(kLossThreads) cosine_loss_fwd_kernel(
    const float* __restrict__ label, const uint8_t* __restrict__ mask, const float* __restrict__ p,
    const float* __restrict__ g, int64_t V, int n, int gl2, float* __restrict__ part_loss,
    int* __restrict__ part_count) {
    using E = typename Row<kVec>::E;
    __shared__ float sl[kLossWarps];
    __shared__ int sc[kLossWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = 1 << gl2, l = lane & (G - 1), sub = lane >> gl2, S = 32 >> gl2;
    const E* P = reinterpret_cast<const E*>(p);
    const E* Q = reinterpret_cast<const E*>(g);
    const int64_t step = (int64_t)gridDim.x * kLossWarps * 32;
    __shared__ int lists[kLossWarps][32];
    int* list = lists[warp];
    float lsum = 0.f;
    int cnt = 0;
    int64_t win = ((int64_t)blockIdx.x * kLossWarps + warp) * 32;
    bool flag = voxel_valid(label, mask, win + lane, V);
    RowIO<kVec, kK> io;
    for (; win < V; win += step) {
        int ninv;
        const int nv = window_list(list, flag, win + lane < V, lane, &ninv);
        flag = voxel_valid(label, mask, win + step + lane, V);  // next window, in flight meanwhile
        cnt += nv;
        for (int j = 0; j < nv; j += S) {
            const int slot = j + sub;
            const bool act = slot < nv;
            const int64_t v = win + (act ? list[slot] : 0);
            float d, a, b;
            io.sums(P + v * n, Q + v * n, act, l, G, n, d, a, b);
            group_sum3(d, a, b, G);
            if (act && l == 0) {
                const float pn = sqrtf(fmaxf(a, kEps)), gn = sqrtf(fmaxf(b, kEps));
                lsum += 1.f - d / (pn * gn + kEps);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
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

// Backward: valid voxels of a window get the gradient (rows read once, kept in registers when kK > 0),
// the other in-range voxels get zero rows (no reads).
template <bool kVec, int kK>
__global__ void __launch_bounds__(kLossThreads) cosine_loss_bwd_kernel(
    const float* __restrict__ grad_out, const int* __restrict__ count_dev, int count_host,
    const float* __restrict__ label, const uint8_t* __restrict__ mask, const float* __restrict__ p,
    const float* __restrict__ g, int64_t V, int n, int gl2, float* __restrict__ gp) {
    using E = typename Row<kVec>::E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = 1 << gl2, l = lane & (G - 1), sub = lane >> gl2, S = 32 >> gl2;
    const int cnt = count_dev ? *count_dev : count_host;
    const float inv_count = cnt > 0 ? 1.0f / (float)cnt : 0.0f;
    const float scale = *grad_out * inv_count;
    const E* P = reinterpret_cast<const E*>(p);
    const E* Q = reinterpret_cast<const E*>(g);
    E* O = reinterpret_cast<E*>(gp);
    const int64_t step = (int64_t)gridDim.x * kLossWarps * 32;
    __shared__ int lists[kLossWarps][32];
    int* list = lists[warp];
    int64_t win = ((int64_t)blockIdx.x * kLossWarps + warp) * 32;
    bool flag = voxel_valid(label, mask, win + lane, V);
    RowIO<kVec, kK> io;
    for (; win < V; win += step) {
        int ni;
        const int nv = window_list(list, flag, win + lane < V, lane, &ni);
        flag = voxel_valid(label, mask, win + step + lane, V);  // next window, in flight meanwhile
        for (int j = 0; j < nv; j += S) {
            const int slot = j + sub;
            const bool act = slot < nv;
            const int64_t v = win + (act ? list[slot] : 0);
            const E* pr = P + v * n;
            const E* gr = Q + v * n;
            float d, a, b;
            io.sums(pr, gr, act, l, G, n, d, a, b);
            group_sum3(d, a, b, G);
            if (act) {
                const float ra = sqrtf(fmaxf(a, kEps)), rb = sqrtf(fmaxf(b, kEps));
                const float D = ra * rb + kEps;
                const float c1 = (-1.0f / D) * scale;                               // multiplies g
                const float c2 = (a > kEps ? (d * rb) / (ra * D * D) : 0.0f) * scale;  // multiplies p
                io.write_grad(O + v * n, pr, gr, l, G, n, c1, c2);
            }
        }
        for (int j = sub; j < ni; j += S) RowIO<kVec, kK>::write_zero(O + (win + list[nv + j]) * n, l, G, n);
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
    int kk;   // elements per lane held in registers (1, 2, 4, 8) or 0 (strided loop)
};

// G = the power of two near n / 4 (at most 32), so that a lane holds about 4 elements of a row.
RowShape row_shape(int C, const void* a, const void* b, const void* c) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    RowShape r;
    r.vec = C % 4 == 0 && al(a) && al(b) && al(c);
    r.n = r.vec ? C / 4 : C;
    const int want = (r.n + 3) / 4;
    r.gl2 = 0;
    while (r.gl2 < 5 && (1 << r.gl2) < want) ++r.gl2;
    const int need = (r.n + (1 << r.gl2) - 1) >> r.gl2;
    r.kk = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 0;
    return r;
}

// Enough CTAs to cover the windows, at most one resident wave (occupancy of this instance), capped.
template <typename K>
int loss_grid(K kernel, int64_t V) {
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kLossThreads, 0) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int64_t need = (V + kLossWarps * 32 - 1) / (kLossWarps * 32);
    return (int)std::max<int64_t>(1, std::min<int64_t>(need, std::min(sm_count() * per_sm, kMaxLossParts)));
}

template <bool kVec, int kK>
int fwd_k(const float* label, const uint8_t* mask, const float* p, const float* g, int64_t V, const RowShape& r,
          float* loss, int* count, void* ws, cudaStream_t s) {
    float* part_loss = static_cast<float*>(ws);
    int* part_count = reinterpret_cast<int*>(part_loss + kMaxLossParts);
    const int grid = loss_grid(cosine_loss_fwd_kernel<kVec, kK>, V);
    G2V_TIMED("cosine_loss_fwd_kernel", s,
              (cosine_loss_fwd_kernel<kVec, kK><<<grid, kLossThreads, 0, s>>>(label, mask, p, g, V, r.n, r.gl2,
                                                                              part_loss, part_count)));
    G2V_LAUNCH_CHECK("cosine_loss_fwd_kernel");
    G2V_TIMED("cosine_loss_final_kernel", s,
              (cosine_loss_final_kernel<<<1, kLossThreads, 0, s>>>(part_loss, part_count, grid, loss, count)));
    G2V_LAUNCH_CHECK("cosine_loss_final_kernel");
    return 0;
}

template <bool kVec, int kK>
int bwd_k(const float* grad_out, const int* count_dev, int count_host, const float* label, const uint8_t* mask,
          const float* p, const float* g, int64_t V, const RowShape& r, float* gp, cudaStream_t s) {
    const int grid = loss_grid(cosine_loss_bwd_kernel<kVec, kK>, V);
    G2V_TIMED("cosine_loss_bwd_kernel", s,
              (cosine_loss_bwd_kernel<kVec, kK><<<grid, kLossThreads, 0, s>>>(grad_out, count_dev, count_host, label,
                                                                              mask, p, g, V, r.n, r.gl2, gp)));
    G2V_LAUNCH_CHECK("cosine_loss_bwd_kernel");
    return 0;
}

template <bool kVec>
int fwd_dispatch(const float* label, const uint8_t* mask, const float* p, const float* g, int64_t V,
                 const RowShape& r, float* loss, int* count, void* ws, cudaStream_t s) {
    switch (r.kk) {
        case 1: return fwd_k<kVec, 1>(label, mask, p, g, V, r, loss, count, ws, s);
        case 2: return fwd_k<kVec, 2>(label, mask, p, g, V, r, loss, count, ws, s);
        case 4: return fwd_k<kVec, 4>(label, mask, p, g, V, r, loss, count, ws, s);
        case 8: return fwd_k<kVec, 8>(label, mask, p, g, V, r, loss, count, ws, s);
        default: return fwd_k<kVec, 0>(label, mask, p, g, V, r, loss, count, ws, s);
    }
}

template <bool kVec>
int bwd_dispatch(const float* grad_out, const int* count_dev, int count_host, const float* label,
                 const uint8_t* mask, const float* p, const float* g, int64_t V, const RowShape& r, float* gp,
                 cudaStream_t s) {
    switch (r.kk) {
        case 1: return bwd_k<kVec, 1>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s);
        case 2: return bwd_k<kVec, 2>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s);
        case 4: return bwd_k<kVec, 4>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s);
        case 8: return bwd_k<kVec, 8>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s);
        default: return bwd_k<kVec, 0>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s);
    }
}
}  // namespace

size_t cosine_loss_workspace_bytes() { return (size_t)kMaxLossParts * (sizeof(float) + sizeof(int)); }

int launch_cosine_loss_fwd(const float* label, const uint8_t* mask, const float* p, const float* g, int64_t V, int C,
                           float* loss, int* count, void* ws, cudaStream_t s) {
    const RowShape r = row_shape(C, p, g, nullptr);
    return r.vec ? fwd_dispatch<true>(label, mask, p, g, V, r, loss, count, ws, s)
                 : fwd_dispatch<false>(label, mask, p, g, V, r, loss, count, ws, s);
}

int launch_cosine_loss_bwd(const float* grad_out, const int* count_dev, int count_host, const float* label,
                           const uint8_t* mask, const float* p, const float* g, int64_t V, int C, float* gp,
                           cudaStream_t s) {
    if (V <= 0 || C <= 0) return 0;
    const RowShape r = row_shape(C, p, g, gp);
    return r.vec ? bwd_dispatch<true>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s)
                 : bwd_dispatch<false>(grad_out, count_dev, count_host, label, mask, p, g, V, r, gp, s);
}

}  // namespace g2v
