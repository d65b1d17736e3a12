// g2v_splat_tc.cu -- forward splat on the 5th-generation tensor cores (tcgen05, kind::f16).
//
// grid_feats[v][c] = sum_g w_gv f_gc / max(D_v, 1e-6), D_v = sum_g w_gv (reference TileGaussianVoxelizer
// forward, src/cuda_gaussian_voxelizer.cu:857-926), as the contraction over the Gaussians of
//     S[c][v] = sum_k F[g_k][c] * w[v][k]       (C x K) . (K x 128)
// computed as D^T in TMEM: M = 128 channels per MMA (two M-blocks = 256 channels per job), N = the 128
// voxels of a unit, K = 16 Gaussians per step.  fp32-level accuracy comes from splitting both operands
// into a half pair, x = hi + lo (~22 bits), and accumulating hi*hi + hi*lo + lo*hi in fp32 (the dropped
// lo*lo term is ~2^-22 relative).  Range: features are scaled per channel by a power of two so that a
// channel's max |f| lies in [2^14, 2^15); weights by a per-unit power of two from the unit's max
// |opacity| (w <= |opacity|), folded into the weight's base-2 exponent.  The epilogue undoes both
// exactly and divides by max(D_v, 1e-6).
//
// Unit of work: a pair of z-adjacent tiles (4 x 4 x 8 voxels) with the union of their Gaussian lists
// (ascending ids): each feature row gathered serves 128 voxels.  Persistent CTAs (one per SM) walk the
// units with a fixed stride; a job is (unit, 256-channel group) and its accumulator takes half of TMEM,
// so the epilogue of one job overlaps the main loop of the next.
//
// Operands in shared memory (per stage):
//   A = F^T slice (256 channels x 16 Gaussians) MN-major, 128-byte swizzle: 64-channel x 8-Gaussian
//       atoms of 1 KB (LBO = 1 KB between channel atoms, SBO = 2 KB between Gaussian octets), gathered
//       row by row from the split features with 16-byte cp.async (L2 evict_last);
//   B = w slice (128 voxels x 16 Gaussians) MN-major, 128-byte swizzle, same atom geometry: one thread
//       writes the 8 z-voxels of a line for one Gaussian as one 16-byte store (conflict-free).
// Roles (544 threads with 4 weight warps): warps 0-3 gather feature rows and stage the step's Gaussian
// records; warps 4-7 evaluate the weights (thread = z-line of 8 voxels x Gaussian pair; along z the
// exponent is a quadratic, so each weight is two FMAs and one exp2) and, in a unit's first job, the
// density; warp 8 (one thread) issues the 6 MMAs of a step; warps 9-16 run the epilogue (thread = channel): the scaled
// values of 16 voxels x 256 channels go to a shared-memory tile that one tiled TMA store writes out
// (L2 evict_first; the store clips the grid edges), double-buffered, or -- when the tensor map cannot be
// built (C % 4 != 0, unaligned output) -- straight to global memory with streaming stores.
// Weight cache: the weights of a unit do not depend on the channel group, so only its first job
// evaluates them; every weight thread also stores its 16-byte words to the CTA's region of a workspace
// buffer (the B stage's layout, kWcSteps steps per CTA; the working set of all CTAs stays in L2) and the
// unit's later jobs copy them back with cp.async.  Steps beyond kWcSteps (units of more than 512
// Gaussians) are evaluated in every job.
// Seven stages; every mbarrier wait is bounded.
#include <algorithm>
#include <cstddef>
#include <cstring>

#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kKStep = 16;                // Gaussians per pipeline step
constexpr int kCG = 256;                  // channels per job (two M-blocks)
constexpr int kUV = 128;                  // voxels per unit
constexpr int kStages = 7;
constexpr int kOutBytes = 16 * kCG * 4;  // epilogue staging tile: 16 voxels x 256 channels fp32
constexpr int kAHalf = 2 * 4096;          // 256 channels x 16 Gaussians, one half (hi or lo)
constexpr int kBHalf = 4096;              // 128 voxels x 16 Gaussians, one half
constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
constexpr uint32_t kTmemCols = 512;
constexpr int kBufCols = 256;             // one job: 2 M-blocks x 128 voxel columns
constexpr int kWarpW0 = 4;                // first weight warp
// Weight-cache capacity: steps (16 Gaussians each) of a unit whose weights are kept for the unit's later
// channel groups, per CTA, and the CTA count the cache is sized for.
constexpr int kWcSteps = 32;
constexpr int kMaxSplatCtas = 148;
constexpr size_t kWcStepBytes = 2 * (size_t)kBHalf;
// Roles for NW weight warps: warps 0-3 producers, 4 .. 4+NW-1 weights, then the MMA warp and 8 epilogue warps.
template <int NW>
struct Roles {
    static constexpr int kMmaWarp = kWarpW0 + NW;
    static constexpr int kEpiWarp0 = kMmaWarp + 1;
    static constexpr int kThreads = (kEpiWarp0 + 8) * 32;
    static constexpr int kGpt = kKStep * 16 / (NW * 32);  // Gaussians per weight thread and step
    static_assert(kGpt * NW * 32 == kKStep * 16, "weight threads must tile 16 Gaussians x 16 z-lines");
};
constexpr uint32_t kIdesc = tc::idesc_f16_f32(128, kUV, /*A MN-major*/ 1, /*B MN-major*/ 1);

// The Gaussian records of the 16 Gaussians of a step, staged with the step's features.
struct StepParams {
    GParams g[kKStep];
};

struct TcMisc {
    uint64_t full_a[kStages];   // the stage's features and Gaussian records landed (128 producer threads)
    uint64_t full_w[kStages];   // the stage's weights written (4 weight warps)
    uint64_t empty[kStages];    // the MMAs reading the stage completed
    uint64_t tfull[2];          // a job's accumulator is complete in TMEM buffer b
    uint64_t tempty[2];         // the epilogue has read buffer b (8 warps)
    uint64_t dready[2];         // a unit's vscale is written (128 weight threads)
    uint64_t dfree[2];          // the epilogue is done with a unit's vscale (8 warps)
    uint32_t tmem_base;
    float red[8];
    alignas(16) float vscale[2][kUV];  // per unit: 2^-kt / max(D_v, eps)
    alignas(16) float dpart[kKStep][kUV];  // density partials [Gaussian group of a thread][voxel], scaled by 2^kt
    alignas(16) StepParams prm[kStages];
};
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 2 * (size_t)kOutBytes + sizeof(TcMisc);
static_assert(kSmemBytes % 16 == 0, "dynamic shared memory size");
static_assert(kSmemBytes <= 227 * 1024, "splat_tc_kernel shared memory");
static_assert(offsetof(TcMisc, vscale) % 16 == 0 && offsetof(TcMisc, prm) % 16 == 0,
              "vector-accessed shared fields must be 16-byte aligned");

__device__ __forceinline__ int pow2_exponent(float m) {
    // floor(log2(m)) for a finite m > 0
    int e;
    frexpf(m, &e);
    return e - 1;
}

// Per-channel max |f| (as float bits; non-negative floats order like integers).  Row blocks of
// rows_per_block rows are walked with a stride of gridDim.y, so any row count fits the grid's y limit.
__global__ void __launch_bounds__(256) feature_colmax_kernel(const float* __restrict__ f, int64_t n, int C,
                                                             int rows_per_block, unsigned* __restrict__ colmax) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float m = 0.0f;
    for (int64_t r0 = (int64_t)blockIdx.y * rows_per_block; r0 < n; r0 += (int64_t)gridDim.y * rows_per_block) {
        const int64_t r1 = min(n, r0 + rows_per_block);
        for (int64_t r = r0; r < r1; ++r) m = fmaxf(m, fabsf(f[r * C + c]));
    }
    atomicMax(&colmax[c], __float_as_uint(m));
}

// features (N, C) fp32 -> hi / lo halves (N, Cp) scaled by 2^k_c, and unscale[c] = 2^-k_c.  The scaling
// is a product with the exact power of two (k_c in [-100, 100]: a normal float), which rounds like
// ldexpf; vec: C % 8 == 0 and a 16-byte aligned base, so a thread's 8 features are two float4 loads.
__global__ void __launch_bounds__(256) feature_split_kernel(const float* __restrict__ f, int64_t n, int C, int Cp,
                                                            int vec, const unsigned* __restrict__ colmax,
                                                            __half* __restrict__ hi, __half* __restrict__ lo,
                                                            float* __restrict__ unscale) {
    const int64_t chunks = (int64_t)Cp / 8;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n * chunks) return;
    const int64_t r = i / chunks;
    const int c8 = (int)(i - r * chunks) * 8;
    float x[8];
    if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(f + r * C + c8));
        const float4 b = __ldg(reinterpret_cast<const float4*>(f + r * C + c8 + 4));
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = c8 + j < C ? f[r * C + c8 + j] : 0.0f;
    }
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = c8 + j;
        int k = 0;
        if (c < C) {
            const float m = __uint_as_float(colmax[c]);
            k = (m > 0.0f) ? max(-100, min(100, 14 - pow2_exponent(m))) : 0;
        }
        tc::split_half(x[j] * __int_as_float((127 + k) << 23), h[j], l[j]);
        if (r == 0) unscale[c] = __int_as_float((127 - k) << 23);
    }
    *reinterpret_cast<uint4*>(hi + r * Cp + c8) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(lo + r * Cp + c8) = *reinterpret_cast<const uint4*>(l);
}

// Gaussian parameters packed as GParams records (the layout the weight threads read).
__global__ void __launch_bounds__(256) pack_params_kernel(const float* __restrict__ means,
                                                          const float* __restrict__ opacity,
                                                          const float* __restrict__ cov_inv,
                                                          const int32_t* __restrict__ lb, const int32_t* __restrict__ ub,
                                                          int64_t n, GParams* __restrict__ out) {
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float* P = cov_inv + g * 9;
    GParams r;
    r.w[0] = make_float4(means[g * 3], means[g * 3 + 1], means[g * 3 + 2], opacity[g]);
    r.w[1] = make_float4(P[0], P[1], P[2], P[3]);
    r.w[2] = make_float4(P[4], P[5], P[6], P[7]);
    r.w[3] = make_float4(P[8], __int_as_float(lb[g * 3]), __int_as_float(lb[g * 3 + 1]), __int_as_float(lb[g * 3 + 2]));
    r.w[4] = make_float4(__int_as_float(ub[g * 3]), __int_as_float(ub[g * 3 + 1]), __int_as_float(ub[g * 3 + 2]), 0.0f);
    out[g] = r;
}

// Named barrier of the NW weight warps (barrier 0 is __syncthreads).
template <int NW>
__device__ __forceinline__ void weight_barrier() {
    asm volatile("bar.sync 2, %0;" ::"n"(NW * 32) : "memory");
}

struct UnitGeom {
    int tx, ty, tzp;
};
__device__ __forceinline__ UnitGeom unit_geom(int u, int ty_n, int tzp_n, int tx_begin) {
    UnitGeom g;
    const int yz = ty_n * tzp_n;
    g.tx = tx_begin + u / yz;
    const int r = u - (u / yz) * yz;
    g.ty = r / tzp_n;
    g.tzp = r - g.ty * tzp_n;
    return g;
}

// The unit lists are those of z quads of tiles (tc_unit_shape, shared with the backward's tile pass):
// z pair u of the slab reads the list of its quad; the quad's Gaussians that miss the pair weigh zero
// there through the box test of the weight evaluation.
__device__ __forceinline__ int list_unit(int u, int tzp_n) {
    const int row = u / tzp_n;
    return row * ((tzp_n + 1) / 2) + (u - row * tzp_n) / 2;
}

// Named barrier of the 8 epilogue warps.
__device__ __forceinline__ void epi_barrier() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <bool kTmaStore, int NW>
__global__ void __launch_bounds__(Roles<NW>::kThreads, 1) splat_tc_kernel(
    const __grid_constant__ CUtensorMap omap, const __half* __restrict__ Fhi, const __half* __restrict__ Flo, const float* __restrict__ unscale, int C, int Cp,
    const GParams* __restrict__ gparams, const int32_t* __restrict__ unit_offsets,
    const int32_t* __restrict__ unit_lists, int num_units, int tx_begin, Grid G, float* __restrict__ density,
    float* __restrict__ grid_feats, unsigned char* __restrict__ wcache, int wc_steps, int* __restrict__ err) {
    constexpr int kNWW = NW;
    constexpr int kMmaWarp = Roles<NW>::kMmaWarp, kEpiWarp0 = Roles<NW>::kEpiWarp0, kGpt = Roles<NW>::kGpt;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    unsigned char* ostage = base + kStages * kStageBytes;  // 2 epilogue staging tiles
    TcMisc& ms = *reinterpret_cast<TcMisc*>(ostage + 2 * kOutBytes);
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {  // the swizzle atoms need 1 KB alignment; never expected
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tzp_n = (G.tiles[2] + 1) / 2;
    const int ngroups = (C + kCG - 1) / kCG;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&ms.full_a[i], 128);
            tc::mbar_init(&ms.full_w[i], kNWW * 32);
            tc::mbar_init(&ms.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&ms.tfull[i], 1);
            tc::mbar_init(&ms.tempty[i], 8);
            tc::mbar_init(&ms.dready[i], kNWW * 32);
            tc::mbar_init(&ms.dfree[i], 8);
        }
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    bool ok = true;
    auto a_stage = [&](int st, int hl) -> uint32_t { return tc::smem_u32(base + st * kStageBytes + hl * kAHalf); };
    auto b_stage = [&](int st, int hl) -> uint32_t {
        return tc::smem_u32(base + st * kStageBytes + 2 * kAHalf + hl * kBHalf);
    };

    if (warp < 4) {
        // ============ producers: feature rows (thread = half hl, row octet kh, 8-channel chunk jc) ============
        const int hl = tid >> 6, kh = (tid >> 5) & 1, jc = lane;
        const int mb = jc >> 4, a = (jc >> 3) & 1, j = jc & 7;
        const char* fbase = reinterpret_cast<const char*>(hl ? Flo : Fhi);
        const int64_t pitch = (int64_t)Cp * 2;
        const uint64_t pol = tc::l2_policy_evict_last();
        int it = 0;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
            const int lu = list_unit(u, tzp_n);
            const int s0 = unit_offsets[lu], K = unit_offsets[lu + 1] - s0;
            if (K == 0) continue;
            const int32_t* list = unit_lists + s0;
            const int nsteps = (K + kKStep - 1) / kKStep;
            for (int cg = 0; cg < ngroups && ok; ++cg) {
                const int c = cg * kCG + jc * 8;
                const bool cin = c < Cp;
                const char* fcol = fbase + (int64_t)(cin ? c : 0) * 2;
                // lanes 0..15 hold the Gaussian ids of a step; step i+1's ids load early
                int next_row = (lane < kKStep && lane < K) ? list[lane] : 0;
                for (int i = 0; i < nsteps && ok; ++i, ++it) {
                    const int st = it % kStages;
                    const int k0 = i * kKStep;
                    const int my_row = next_row;
                    next_row = (lane < kKStep && k0 + kKStep + lane < K) ? list[k0 + kKStep + lane] : 0;
                    if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                    if (!ok) break;
                    const uint32_t dbase = a_stage(st, hl) + mb * 4096 + a * 1024 + kh * 2048;
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const int k = kh * 8 + r;
                        const int row = __shfl_sync(0xffffffffu, my_row, k);
                        const bool valid = cin && (k0 + k < K);
                        tc::cp_async16_hint(dbase + r * 128 + ((j ^ r) << 4), fcol + (valid ? (int64_t)row * pitch : 0),
                                            valid ? 16u : 0u, pol);
                    }
                    // Gaussian records: 16 records of 5 x 16 bytes (zero fill for padding)
                    {
                        const int k = min(tid / 5, kKStep - 1), wq = tid - (tid / 5) * 5;
                        const int row = __shfl_sync(0xffffffffu, my_row, k);  // whole warp takes part
                        if (tid < kKStep * 5) {
                            const bool valid = k0 + k < K;
                            tc::cp_async16(tc::smem_u32(&ms.prm[st].g[k].w[wq]), &gparams[valid ? row : 0].w[wq],
                                           valid ? 16u : 0u);
                        }
                    }
                    tc::cp_async_mbar_arrive_noinc(&ms.full_a[st]);
                }
            }
        }
        tc::cp_async_wait<0>();  // no copy in flight when the shared memory is released
    } else if (warp < kMmaWarp) {
        // ============ weight warps: thread = (z-line o of 8 voxels, kGpt Gaussians kq*kGpt.. of the step) ============
        // With a weight cache, a unit's weights are evaluated in its first channel group only: each thread
        // also writes its 16-byte words to the CTA's region of the cache (same layout as the B stage) and,
        // in the later channel groups, copies them back with cp.async instead of evaluating them again.
        // A thread reads back only the words it wrote itself.
        const int t = tid - kWarpW0 * 32;
        const int o = t & 15, kq = t >> 4;
        const int lx = o >> 2, ly = o & 3;
        const float k2 = tc::kNegHalfLog2e;
        const float hz = G.h[2];
        unsigned char* wregion = wcache ? wcache + (size_t)blockIdx.x * wc_steps * kWcStepBytes : nullptr;
        // The named barriers below are reached the same number of times by every weight thread whatever
        // `ok` says (a wait that gave up only skips work), so a failed wait cannot split the barrier.
        int it = 0, nu = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
            const int lu = list_unit(u, tzp_n);
            const int s0 = unit_offsets[lu], K = unit_offsets[lu + 1] - s0;
            if (K == 0) continue;
            const int32_t* list = unit_lists + s0;
            const UnitGeom ug = unit_geom(u, G.tiles[1], tzp_n, tx_begin);
            const int x0 = ug.tx * kTile, y0 = ug.ty * kTile, z0 = ug.tzp * 8;
            const int vx = x0 + lx, vy = y0 + ly;
            const float cx = voxel_centre(G, 0, vx), cy = voxel_centre(G, 1, vy), cz0 = voxel_centre(G, 2, z0);
            // this thread's cache reads of the previous unit are complete before its words are rewritten
            tc::cp_async_wait<0>();
            // unit weight scale 2^kt from the largest |opacity| (w <= |opacity|)
            float om = 0.0f;
            for (int i = t; i < K; i += kNWW * 32) om = fmaxf(om, fabsf(gparams[list[i]].w[0].w));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) om = fmaxf(om, __shfl_xor_sync(0xffffffffu, om, off));
            if (lane == 0) ms.red[warp - kWarpW0] = om;
            weight_barrier<NW>();
            om = 0.0f;
#pragma unroll
            for (int w8 = 0; w8 < kNWW; ++w8) om = fmaxf(om, ms.red[w8]);
            weight_barrier<NW>();
            int kt = 0;
            if (om > 0.0f) {
                int e2;
                frexpf(om, &e2);
                kt = max(-100, min(100, 15 - e2));  // max scaled weight in [2^14, 2^15)
            }
            const float fkt = (float)kt;
            const int nsteps = (K + kKStep - 1) / kKStep;
            float dsum[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) dsum[i] = 0.0f;
            for (int cg = 0; cg < ngroups; ++cg) {
                for (int i = 0; i < nsteps && ok; ++i, ++it) {
                    const int st = it % kStages;
                    const bool cached = wregion != nullptr && i < wc_steps;
                    const bool reuse = cached && cg > 0;
                    if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                    if (!reuse) ok = ok && tc::mbar_wait(&ms.full_a[st], (it / kStages) & 1, err);
                    if (!ok) break;
                    unsigned char* bst = base + st * kStageBytes + 2 * kAHalf;
                    unsigned char* wstep = cached ? wregion + (size_t)i * kWcStepBytes : nullptr;
                    if (reuse) {
#pragma unroll
                        for (int u2 = 0; u2 < kGpt; ++u2) {
                            const int k = kq * kGpt + u2, r = k & 7;
                            const uint32_t off = (k >> 3) * 2048 + (o >> 3) * 1024 + r * 128 + (((o & 7) ^ r) << 4);
                            tc::cp_async16(tc::smem_u32(bst + off), wstep + off, 16u);
                            tc::cp_async16(tc::smem_u32(bst + kBHalf + off), wstep + kBHalf + off, 16u);
                        }
                        tc::cp_async_mbar_arrive_noinc(&ms.full_w[st]);
                        continue;
                    }
                    const int k0 = i * kKStep;
#pragma unroll
                    for (int u2 = 0; u2 < kGpt; ++u2) {
                        const int k = kq * kGpt + u2;
                        const GParams& gp = ms.prm[st].g[k];
                        const float4 A = gp.w[0], P0 = gp.w[1], P1 = gp.w[2], P2 = gp.w[3], U = gp.w[4];
                        const bool live = k0 + k < K && vx >= __float_as_int(P2.y) && vx <= __float_as_int(U.x) &&
                                          vy >= __float_as_int(P2.z) && vy <= __float_as_int(U.y);
                        const int zlo = __float_as_int(P2.w) - z0, zhi = __float_as_int(U.z) - z0;
                        const float dx = cx - A.x, dy = cy - A.y, dz = cz0 - A.z;
                        const float qx = fmaf(P0.z, dz, fmaf(P0.y, dy, P0.x * dx));
                        const float qy = fmaf(P1.y, dz, fmaf(P1.x, dy, P0.w * dx));
                        const float qz = fmaf(P2.x, dz, fmaf(P1.w, dy, P1.z * dx));
                        const float ptz = fmaf(P2.x, dz, fmaf(P1.y, dy, P0.z * dx));  // (P' d)_z
                        // base-2 exponent along the line: k2 (a + b lz + P8 hz^2 lz^2) + kt; -inf outside the box
                        const float a0 = live ? fmaf(k2, dx * qx + dy * qy + dz * qz, fkt) : -INFINITY;
                        const float b0 = k2 * hz * (qz + ptz), qq = k2 * hz * hz * P2.x;
                        // z pairs (lz, lz + 1) in packed f32x2 arithmetic
                        float w[8];
                        const float2 A2 = make_float2(a0, a0), B2 = make_float2(b0, b0), Q2 = make_float2(qq, qq);
                        const float2 O2 = make_float2(A.w, A.w);
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            const int l0 = 2 * p, l1 = l0 + 1;
                            const float2 mz = make_float2((l0 >= zlo && l0 <= zhi) ? 0.0f : -INFINITY,
                                                          (l1 >= zlo && l1 <= zhi) ? 0.0f : -INFINITY);
                            const float2 lz2 = make_float2((float)l0, (float)l1);
                            const float2 m = __fadd2_rn(__ffma2_rn(__ffma2_rn(Q2, lz2, B2), lz2, A2), mz);
                            const float2 wv = __fmul2_rn(O2, make_float2(tc::exp2_approx(m.x), tc::exp2_approx(m.y)));
                            w[l0] = wv.x;
                            w[l1] = wv.y;
                            if (cg == 0) {
                                const float2 d = __fadd2_rn(make_float2(dsum[l0], dsum[l1]), wv);
                                dsum[l0] = d.x;
                                dsum[l1] = d.y;
                            }
                        }
                        uint4 h, l;
                        tc::split_half2_v(w[0], w[1], h.x, l.x);
                        tc::split_half2_v(w[2], w[3], h.y, l.y);
                        tc::split_half2_v(w[4], w[5], h.z, l.z);
                        tc::split_half2_v(w[6], w[7], h.w, l.w);
                        const int r = k & 7;
                        const uint32_t off = (k >> 3) * 2048 + (o >> 3) * 1024 + r * 128 + (((o & 7) ^ r) << 4);
                        *reinterpret_cast<uint4*>(bst + off) = h;
                        *reinterpret_cast<uint4*>(bst + kBHalf + off) = l;
                        if (cached) {
                            *reinterpret_cast<uint4*>(wstep + off) = h;
                            *reinterpret_cast<uint4*>(wstep + kBHalf + off) = l;
                        }
                    }
                    tc::fence_async_smem();
                    tc::mbar_arrive(&ms.full_w[st]);
                }
                if (cg == 0) {
                    // density of the unit: sum over the thread groups; vscale for the epilogue
#pragma unroll
                    for (int lz = 0; lz < 8; ++lz) ms.dpart[kq][o * 8 + lz] = dsum[lz];
                    weight_barrier<NW>();
                    const int b = nu & 1;
                    if (nu >= 2 && ok) ok = tc::mbar_wait(&ms.dfree[b], ((nu / 2) + 1) & 1, err);
                    if (t < kUV) {
                        const int v = t;  // voxel of the unit: (v >> 5, (v >> 3) & 3, v & 7)
                        float Ds = 0.0f;
#pragma unroll
                        for (int q = 0; q < kNWW * 2; ++q) Ds += ms.dpart[q][v];
                        const float D = ldexpf(Ds, -kt);
                        ms.vscale[b][v] = ldexpf(1.0f, -kt) / fmaxf(D, kEps);
                        const int x = x0 + (v >> 5), y = y0 + ((v >> 3) & 3), z = z0 + (v & 7);
                        if (x < G.dims[0] && y < G.dims[1] && z < G.dims[2])
                            density[grid_row(G, x, y, z)] = D;
                    }
                    tc::mbar_arrive(&ms.dready[b]);
                    weight_barrier<NW>();  // dpart is reused by the next unit
                }
            }
            ++nu;
        }
        tc::cp_async_wait<0>();  // no copy in flight when the shared memory is released
    } else if (warp == kMmaWarp) {
        // ============ MMA thread ============
        if (lane == 0) {
            int it = 0, job = 0;
            const uint64_t adesc0 = tc::smem_desc(a_stage(0, 0), 1024, 2048, tc::kLayoutSw128);
            const uint64_t bdesc0 = tc::smem_desc(b_stage(0, 0), 1024, 2048, tc::kLayoutSw128);
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const int lu = list_unit(u, tzp_n);
                const int K = unit_offsets[lu + 1] - unit_offsets[lu];
                if (K == 0) continue;
                const int nsteps = (K + kKStep - 1) / kKStep;
                for (int cg = 0; cg < ngroups && ok; ++cg, ++job) {
                    const int buf = job & 1;
                    if (job >= 2) ok = tc::mbar_wait(&ms.tempty[buf], ((job / 2) + 1) & 1, err);
                    if (!ok) break;
                    tc::tc_fence_after();
                    for (int i = 0; i < nsteps && ok; ++i, ++it) {
                        const int st = it % kStages;
                        const uint32_t par = (it / kStages) & 1;
                        ok = tc::mbar_wait(&ms.full_a[st], par, err) && tc::mbar_wait(&ms.full_w[st], par, err);
                        if (!ok) break;
                        // the A operand was written by cp.async (generic proxy); the MMA reads it through the async proxy
                        tc::fence_async_smem();
                        tc::tc_fence_after();
                        // descriptors of the stage from the stage-0 ones (start address in 16-byte units)
                        const uint64_t soff = (uint64_t)((st * kStageBytes) >> 4);
                        const uint64_t bh = bdesc0 + soff, bl = bh + (uint64_t)(kBHalf >> 4);
#pragma unroll
                        for (int mb = 0; mb < 2; ++mb) {
                            const uint64_t ah = adesc0 + soff + (uint64_t)((mb * 4096) >> 4);
                            const uint64_t al = ah + (uint64_t)(kAHalf >> 4);
                            const uint32_t d = tmem + (uint32_t)(buf * kBufCols + mb * kUV);
                            tc::mma_f16_ss<tc::kColFill>(d, ah, bh, kIdesc, i > 0);
                            tc::mma_f16_ss<tc::kColLastUse>(d, ah, bl, kIdesc, true);
                            tc::mma_f16_ss(d, al, bh, kIdesc, true);
                        }
                        tc::mma_commit(tc::smem_u32(&ms.empty[st]));
                    }
                    tc::mma_commit(tc::smem_u32(&ms.tfull[buf]));
                }
            }
        }
    } else {
        // ============ epilogue warps: thread = channel (TMEM lane), streaming stores of grid_feats ============
        const int et = tid - kEpiWarp0 * 32;  // 0..255
        const int q = warp & 3;               // TMEM lane quarter of this warp
        const int mb = (warp - kEpiWarp0) >> 2;
        const int64_t sx = (int64_t)G.dims[1] * G.dims[2], sy = G.dims[2];
        const uint64_t opol = tc::l2_policy_evict_first();  // grid_feats is written once
        int job = 0, nu = 0, ochunk = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
            const int lu = list_unit(u, tzp_n);
            const int K = unit_offsets[lu + 1] - unit_offsets[lu];
            const UnitGeom ug = unit_geom(u, G.tiles[1], tzp_n, tx_begin);
            const int x0 = ug.tx * kTile, y0 = ug.ty * kTile, z0 = ug.tzp * 8;
            const int nx = min(kTile, G.dims[0] - x0), ny = min(kTile, G.dims[1] - y0), nz = min(8, G.dims[2] - z0);
            const int64_t row0 = grid_row(G, x0, y0, z0);
            if (K == 0) {  // no Gaussian reaches the unit: zeros
                for (int v = 0; v < kUV; ++v) {
                    const int lx = v >> 5, ly = (v >> 3) & 3, lz = v & 7;
                    if (lx >= nx || ly >= ny || lz >= nz) continue;
                    const int64_t row = row0 + lx * sx + ly * sy + lz;
                    for (int c = et; c < C; c += 256) __stcs(&grid_feats[row * C + c], 0.0f);
                    if (et == 0) density[row] = 0.0f;
                }
                continue;
            }
            const int b = nu & 1;
            bool good = ok && tc::mbar_wait(&ms.dready[b], (nu / 2) & 1, err);
            for (int cg = 0; cg < ngroups; ++cg, ++job) {
                const int buf = job & 1;
                good = good && ok && tc::mbar_wait(&ms.tfull[buf], (job / 2) & 1, err);
                if (!good) ok = false;
                tc::tc_fence_after();
                const int c = cg * kCG + mb * 128 + q * 32 + lane;
                const bool cok = c < C;
                const float us = cok ? unscale[c] : 0.0f;
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kBufCols + mb * kUV);
                if (kTmaStore) {
                    // all 8 warps take part in every chunk (the staging tile spans the job's 256 channels)
                    const int cl = mb * 128 + q * 32 + lane;  // channel within the job
#pragma unroll 1
                    for (int ch = 0; ch < 8; ++ch, ++ochunk) {  // x-slice lx = ch / 2, ly = 2 (ch % 2) + e / 8
                        float vals[16];
                        if (good) {
                            tc::tmem_ld16(taddr + ch * 16, vals);
                        } else {
#pragma unroll
                            for (int e = 0; e < 16; ++e) vals[e] = 0.0f;
                        }
                        const float4* vs4 = reinterpret_cast<const float4*>(&ms.vscale[b][ch * 16]);
                        const int sb = ochunk & 1;
                        float* st = reinterpret_cast<float*>(ostage + sb * kOutBytes);
                        if (et == 0) tc::bulk_wait_group_read<1>();  // the store that last read tile sb is done
                        epi_barrier();
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4) {
                            const float4 r4 = vs4[e4];
                            st[(4 * e4 + 0) * kCG + cl] = vals[4 * e4 + 0] * (us * r4.x);
                            st[(4 * e4 + 1) * kCG + cl] = vals[4 * e4 + 1] * (us * r4.y);
                            st[(4 * e4 + 2) * kCG + cl] = vals[4 * e4 + 2] * (us * r4.z);
                            st[(4 * e4 + 3) * kCG + cl] = vals[4 * e4 + 3] * (us * r4.w);
                        }
                        tc::fence_async_smem();
                        epi_barrier();
                        if (et == 0 && good) {
                            tc::tma_store_4d_hint(&omap, tc::smem_u32(st), cg * kCG, z0, y0 + 2 * (ch & 1),
                                                  x0 + (ch >> 1) - G.xoff, opol);
                            tc::bulk_commit_group();
                        }
                    }
                } else if (good) {
#pragma unroll 1
                    for (int ch = 0; ch < 8; ++ch) {  // 16 columns: x-slice lx = ch / 2, ly = 2 (ch % 2) + (e / 8)
                        float vals[16];
                        tc::tmem_ld16(taddr + ch * 16, vals);
                        const int lx = ch >> 1;
                        const float4* vs4 = reinterpret_cast<const float4*>(&ms.vscale[b][ch * 16]);
                        float vs[16];
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4) {
                            const float4 r4 = vs4[e4];
                            vs[4 * e4] = r4.x;
                            vs[4 * e4 + 1] = r4.y;
                            vs[4 * e4 + 2] = r4.z;
                            vs[4 * e4 + 3] = r4.w;
                        }
                        if (cok && lx < nx) {
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                const int ly = (ch & 1) * 2 + (e >> 3), lz = e & 7;
                                if (ly < ny && lz < nz)
                                    __stcs(&grid_feats[(row0 + lx * sx + ly * sy + lz) * C + c], vals[e] * (us * vs[e]));
                            }
                        }
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&ms.tempty[buf]);
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&ms.dfree[b]);
            ++nu;
        }
        if (kTmaStore && et == 0) tc::bulk_wait_group_all();  // the output is written before the CTA exits
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}
}  // namespace

int launch_pack_params(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                       const int32_t* ub, int64_t n, GParams* out, cudaStream_t s) {
    if (n <= 0) return 0;
    G2V_TIMED("pack_params_kernel", s,
              pack_params_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(means, opacity, cov_inv, lb, ub, n, out));
    G2V_LAUNCH_CHECK("pack_params_kernel");
    return 0;
}

size_t splat_tc_split_bytes(int64_t n, int64_t C) {
    const int64_t Cp = (C + 7) / 8 * 8;
    return 2 * ((size_t)n * Cp * sizeof(__half) + 256) + 2 * ((size_t)Cp * 4 + 256) +
           ((size_t)(n > 0 ? n : 1) * sizeof(GParams) + 256) + ((size_t)kMaxSplatCtas * kWcSteps * kWcStepBytes + 256);
}

namespace {
// Weight warps of the splat kernel: with one channel group (C <= 256) every step evaluates weights and
// eight warps hide their latency better (cfg5: splat 32.6 vs 36.7 ms); with several groups the weight
// cache leaves the evaluation to the first group and four warps are faster (cfg3: 1.16 vs 1.22 ms).
// G2V_SPLAT_WW=4 or 8 overrides.  G2V_SPLAT_WCACHE=0 turns the weight cache off (cfg3: 1.60 / 1.46 ms).
int splat_weight_warps(int ngroups) {
    const char* e = getenv("G2V_SPLAT_WW");
    if (e && atoi(e) == 8) return 8;
    if (e && atoi(e) == 4) return 4;
    return ngroups == 1 ? 8 : 4;
}
bool splat_weight_cache() {
    const char* e = getenv("G2V_SPLAT_WCACHE");
    return !(e && e[0] == '0');
}
template <int NW>
int launch_splat_kernel(bool tma, const CUtensorMap& omap, const __half* hi, const __half* lo, const float* unscale,
                        int C, int Cp, const GParams* gp, const int32_t* unit_offsets, const int32_t* unit_lists,
                        int num_units, int tile_x_begin, const Grid& G, float* density, float* grid_feats,
                        unsigned char* wcache, int* err, cudaStream_t s) {
    auto kern = tma ? splat_tc_kernel<true, NW> : splat_tc_kernel<false, NW>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    int dev = 0, sms = 148;
    G2V_CUDA(cudaGetDevice(&dev));
    G2V_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    int grid = num_units < sms ? num_units : sms;
    if (grid > kMaxSplatCtas) grid = kMaxSplatCtas;  // the weight cache holds kMaxSplatCtas regions
    G2V_TIMED("splat_tc_kernel", s,
              kern<<<(unsigned)grid, Roles<NW>::kThreads, kSmemBytes, s>>>(
                  omap, hi, lo, unscale, C, Cp, gp, unit_offsets, unit_lists, num_units, tile_x_begin, G, density,
                  grid_feats, wcache, kWcSteps, err));
    G2V_LAUNCH_CHECK("splat_tc_kernel");
    return 0;
}
}  // namespace

// Splits the features (per-channel power-of-two scale) into `split` (splat_tc_split_bytes) and runs the
// tensor-core splat over the units (z pairs of tiles) of the slab [tile_x_begin, tile_x_end), whose
// Gaussians come from the z-quad unit lists (unit_offsets / unit_lists, tc_unit_shape cells).
int launch_splat_tc(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                    const int32_t* ub, const float* features, int64_t n, int C, const int32_t* unit_offsets,
                    const int32_t* unit_lists, int tile_x_begin, int tile_x_end, const Grid& G, float* density,
                    float* grid_feats, void* split, int* err, cudaStream_t s) {
    const int num_units = (tile_x_end - tile_x_begin) * G.tiles[1] * ((G.tiles[2] + 1) / 2);
    if (num_units <= 0) return 0;
    const int Cp = (C + 7) / 8 * 8;
    Carver cv(split);
    __half* hi = cv.take<__half>((size_t)n * Cp);
    __half* lo = cv.take<__half>((size_t)n * Cp);
    unsigned* colmax = cv.take<unsigned>((size_t)Cp);
    float* unscale = cv.take<float>((size_t)Cp);
    if (n > 0) {
        G2V_CUDA(cudaMemsetAsync(colmax, 0, sizeof(unsigned) * Cp, s));
        const int rows = 64;  // rows per block: enough blocks in flight to stream the features
        const int64_t row_blocks = (n + rows - 1) / rows;
        dim3 g1((C + 255) / 256, (unsigned)std::min<int64_t>(row_blocks, 65535));
        G2V_TIMED("feature_colmax_kernel", s, feature_colmax_kernel<<<g1, 256, 0, s>>>(features, n, C, rows, colmax));
        G2V_LAUNCH_CHECK("feature_colmax_kernel");
        const int64_t total = n * (Cp / 8);
        G2V_TIMED("feature_split_kernel", s,
                  feature_split_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
                      features, n, C, Cp, (C % 8 == 0 && (reinterpret_cast<uintptr_t>(features) & 15) == 0) ? 1 : 0,
                      colmax, hi, lo, unscale));
        G2V_LAUNCH_CHECK("feature_split_kernel");
    }
    GParams* gp = cv.take<GParams>((size_t)(n > 0 ? n : 1));
    unsigned char* wcache = cv.take<unsigned char>((size_t)kMaxSplatCtas * kWcSteps * kWcStepBytes);
    int rc = launch_pack_params(means, opacity, cov_inv, lb, ub, n, gp, s);
    if (rc) return rc;
    CUtensorMap omap;
    memset(&omap, 0, sizeof(omap));
    const int ldims[3] = {G.xlen, G.dims[1], G.dims[2]};
    const bool tma = C > 0 && encode_grid_rows_f32(&omap, grid_feats, ldims, C, kCG, 8, 2, 1);
    // the cache serves a unit's later channel groups: with one group (C <= 256) nothing would read it
    const int ngroups = (C + kCG - 1) / kCG;
    unsigned char* wc = (splat_weight_cache() && ngroups > 1) ? wcache : nullptr;
    if (splat_weight_warps(ngroups) == 4)
        return launch_splat_kernel<4>(tma, omap, hi, lo, unscale, C, Cp, gp, unit_offsets, unit_lists, num_units,
                                      tile_x_begin, G, density, grid_feats, wc, err, s);
    return launch_splat_kernel<8>(tma, omap, hi, lo, unscale, C, Cp, gp, unit_offsets, unit_lists, num_units,
                                  tile_x_begin, G, density, grid_feats, wc, err, s);
}

}  // namespace g2v

