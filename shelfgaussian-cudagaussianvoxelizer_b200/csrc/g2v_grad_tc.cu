// g2v_grad_tc.cu -- feature gradient of the backward on the tensor cores (tcgen05, kind::f16, bf16).
//
// For a block of tiles b and its Gaussians (the block's list, up to 256 "slots" per pass):
//     dF[slot][c] = sum_{v in b} w_slot,v / max(D_v, 1e-6) * gF[v][c]
// computed as D^T in TMEM: M = 128 channels (2 M-blocks = 256 channels per CTA), N = 256 slots,
// K = 32 voxels per pipeline step (half a tile: the 16 voxels of each of two x-slices, two MMA K-steps).  Accuracy: both operands
// are split into bf16 pairs (x = hi + lo to ~2^-17) and hi*hi + hi*lo + lo*hi is accumulated in fp32;
// bf16 keeps the fp32 exponent range, so no scaling is needed.
//
// Operands in shared memory (per stage):
//   A = gF^T slices (256 channels x 32 voxels) MN-major, 128-byte swizzle (64-channel x 8-voxel atoms),
//       converted from the fp32 gradient rows by the producer warps;
//   B = weights (256 slots x 16 voxels, one block per x-slice) K-major, 32-byte swizzle (a row = one slot's 16 voxels), evaluated by the weight
//       warps from the slot's parameters: over the 4x4 voxels of an x-slice the Mahalanobis distance is a
//       quadratic in (ly, lz), so each weight costs a few FMAs and one exp.
// The fp32 gradient rows of a step (32 voxels x 256 channels, 32 KB) arrive in a staging ring through
// one tiled TMA load of the 4-D tensor map {C, Z, Y, X} (zero fill beyond the grid and beyond C); when
// the map cannot be built (C % 4 != 0, unaligned base) the converting threads load the rows themselves.
// log2(1 / max(D, eps)) of the block's voxels is computed once per CTA into shared memory and folded,
// with the box masks (-inf), into the base-2 exponent of each weight: w / den = o * 2^(quadratic + L_v).
// Roles (576 threads): warps 0-7 convert A (two voxel rows each), warps 8-15 produce B (one Gaussian
// slot per thread), warp 16 (one thread) issues the 6 MMAs of a step, warp 17 (one thread) issues the
// TMA loads; two warps of each producer role per scheduler hide the latency of the dependent math.  Two
// operand stages and two staging stages of two x-slices each are handed over through mbarriers (a step of
// two slices halves the barrier round trips per voxel, which the pipeline's hand-offs are bound by); every
// wait is bounded.  The epilogue writes the
// per-(Gaussian, block) partial rows of the reference's dL/dfeatures; a deterministic CSR-order reduction
// sums them per Gaussian.
#include <cstddef>

#include <cstring>

#include "g2v.h"
#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 576;
constexpr int kSlots = 256;
constexpr int kMB = 2;                          // M-blocks of 128 channels per CTA
constexpr int kCG = kMB * 128;                  // channels per CTA
constexpr int kStages = 2;                      // operand stages of two x-slices (K = 32 voxels) each
constexpr int kASub = kMB * 4096;               // one operand half of one x-slice
constexpr int kAHalf = 2 * kASub;               // one operand half, one stage
constexpr int kBSub = kSlots * 16 * 2;
constexpr int kBHalf = 2 * kBSub;
constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
constexpr uint32_t kTmemCols = 512;
constexpr int kGS = 2;                          // staging stages of the fp32 gradient
constexpr int kGBytes = 32 * kCG * 4;           // 32 KB: [lx][ly][lz][256 channels]
constexpr int kMaxBlockTiles = 32;              // tiles per block (default 4 x 2 x 4)
constexpr int kMaskPasses = 32;                 // passes with a step mask; later passes take every step
// N of a pass = its slot count rounded up to 16 (a pass that is not full issues narrower MMAs)

struct FMisc {
    uint64_t full[kStages];   // 8 converter-warp + 8 weight-warp arrivals: both operands of the stage written
    uint64_t empty[kStages];  // MMA commit: the stage has been read
    uint64_t mma_done;
    uint32_t tmem_base;
    int fail;
    uint32_t smask[kMaskPasses][2];  // per pass: the steps that meet a slot's box (bit j = step j)
    uint64_t gfull[kGS];   // TMA bytes of a staged step
    uint64_t gempty[kGS];  // 8 converter-warp arrivals
    alignas(16) GParams prm[kSlots];  // slot records of the pass (each weight thread stages its own)
    int64_t rowoff[kSlots];
    alignas(16) float lrd[kMaxBlockTiles * kVoxPerTile];  // log2(1 / max(D, eps)), -inf outside the grid
    int4 org[kMaxBlockTiles];  // voxel origin of each tile of the block, in step order
};
// Walks the set bits of a step mask (at most 64 steps: 32 tiles x 2 x-slice pairs) in ascending order.
struct StepList {
    uint64_t bits;
    __device__ __forceinline__ int next() {
        const int j = __ffsll((long long)bits) - 1;
        bits &= bits - 1;
        return j;
    }
};
static_assert(kMaxBlockTiles * 2 <= 64, "a pass's steps fit one 64-bit mask");
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + (size_t)kGS * kGBytes + sizeof(FMisc);
static_assert(kSmemBytes <= 227 * 1024, "fpass_tc_kernel shared memory");
static_assert(offsetof(FMisc, lrd) % 16 == 0, "lrd is read as float4");

template <bool kTma>
__global__ void __launch_bounds__(kThreads, 1) fpass_tc_kernel(
    const __grid_constant__ CUtensorMap gmap, const float* __restrict__ grad_feats, int C, const float* __restrict__ density, const GParams* __restrict__ gparams,
    const int32_t* __restrict__ block_offsets, const int32_t* __restrict__ block_lists,
    const int32_t* __restrict__ g2b_offsets, int bx_begin, int nby, int nbz, int BX, int BY, int BZ, int tx_begin,
    int tx_end, int ngroups, int vec, Grid G, float* __restrict__ partialF, int64_t block_pair_cap,
    int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    unsigned char* gstage = base + kStages * kStageBytes;
    FMisc& ms = *reinterpret_cast<FMisc*>(gstage + kGS * kGBytes);
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bl = blockIdx.x / ngroups, cg = blockIdx.x - bl * ngroups;
    const int bxr = bl / (nby * nbz), rem = bl - bxr * nby * nbz;
    const int by = rem / nbz, bz = rem - (rem / nbz) * nbz;
    const int bx = bx_begin + bxr;
    const int s0 = block_offsets[bl], Kb = block_offsets[bl + 1] - s0;
    if (Kb == 0) return;
    const int c0 = cg * kCG;
    const int txa = max(bx * BX, tx_begin), txb = min(bx * BX + BX, min(tx_end, G.tiles[0]));
    const int tya = by * BY, tyb = min(tya + BY, G.tiles[1]);
    const int tza = bz * BZ, tzb = min(tza + BZ, G.tiles[2]);
    const int nty = tyb - tya, ntz = tzb - tza;
    const int ntiles = max(0, txb - txa) * nty * ntz;
    if (ntiles == 0) {  // no tile of this block in the slab: its partial rows are zero
        for (int sl = 0; sl < Kb; ++sl) {
            const int g = block_lists[s0 + sl];
            const GParams& gp = gparams[g];
            const int blx = (__float_as_int(gp.w[3].y) / kTile) / BX, bly = (__float_as_int(gp.w[3].z) / kTile) / BY;
            const int blz = (__float_as_int(gp.w[3].w) / kTile) / BZ;
            const int ey = (__float_as_int(gp.w[4].y) / kTile) / BY - bly + 1;
            const int ez = (__float_as_int(gp.w[4].z) / kTile) / BZ - blz + 1;
            const int64_t ro = (int64_t)g2b_offsets[g] + ((bx - blx) * ey + (by - bly)) * ez + (bz - blz);
            if (ro >= block_pair_cap) continue;
            for (int c = c0 + threadIdx.x; c < min(C, c0 + kCG); c += kThreads) partialF[ro * C + c] = 0.0f;
        }
        return;
    }
    if (ntiles > kMaxBlockTiles) {  // the host sizes blocks within the limit
        if (tid == 0) atomicOr(err, 4);
        return;
    }
    for (int t = tid; t < ntiles; t += kThreads) {
        const int tzi = t % ntz, tyi = (t / ntz) % nty, txi = t / (ntz * nty);
        ms.org[t] = make_int4((txa + txi) * kTile, (tya + tyi) * kTile, (tza + tzi) * kTile, 0);
    }

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&ms.full[i], 16);
            tc::mbar_init(&ms.empty[i], 1);
        }
        tc::mbar_init(&ms.mma_done, 1);
        for (int i = 0; i < kMaskPasses * 2; ++i) ms.smask[i >> 1][i & 1] = 0u;
        for (int i = 0; i < kGS; ++i) {
            tc::mbar_init(&ms.gfull[i], 1);
            tc::mbar_init(&ms.gempty[i], 8);
        }
        tc::mbar_fence_init();
        ms.fail = 0;
    }
    if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    bool ok = true;

    // The steps of each pass whose pair of x-slices meets at least one of its slots' voxel boxes; every role
    // walks the same list, so the others (no weight of the pass is non-zero there) are skipped.  The
    // block lists are ordered by the boxes' lower x, so a pass's slots lie close together along x.
    // A warp's 32 slots belong to one pass (576 and 256 are multiples of 32).
    {
        const int nmask = min(Kb, kMaskPasses * kSlots);
        for (int sl0 = 0; sl0 < nmask; sl0 += kThreads) {
            const int sl = sl0 + tid;
            uint64_t mlo = 0;  // 2 bits (x-slice pairs) per tile, at most 32 tiles
            if (sl < nmask) {
                const GParams& gp = gparams[block_lists[s0 + sl]];
                const float4 d = gp.w[3], e4 = gp.w[4];
                const int lx = __float_as_int(d.y), ly = __float_as_int(d.z), lz = __float_as_int(d.w);
                const int ux = __float_as_int(e4.x), uy = __float_as_int(e4.y), uz = __float_as_int(e4.z);
                for (int ti = 0; ti < ntiles; ++ti) {
                    const int4 o = ms.org[ti];
                    const int a = max(lx - o.x, 0), b = min(ux - o.x, 3);
                    if (a > b || ly > o.y + 3 || uy < o.y || lz > o.z + 3 || uz < o.z) continue;
                    const int pa = a >> 1, pb = b >> 1;  // slice pairs of x-slices a..b
                    mlo |= (uint64_t)(((2u << (pb - pa)) - 1u) << pa) << (ti * 2);
                }
            }
            const uint32_t w0 = __reduce_or_sync(0xffffffffu, (uint32_t)mlo);
            const uint32_t w1 = __reduce_or_sync(0xffffffffu, (uint32_t)(mlo >> 32));
            if (lane == 0 && sl < nmask) {
                uint32_t* m = ms.smask[sl / kSlots];
                if (w0) atomicOr(&m[0], w0);
                if (w1) atomicOr(&m[1], w1);
            }
        }
    }
    __syncthreads();

    auto a_stage = [&](int st, int hl) -> unsigned char* { return base + st * kStageBytes + hl * kAHalf; };
    auto b_stage = [&](int st, int hl) -> unsigned char* {
        return base + st * kStageBytes + 2 * kAHalf + hl * kBHalf;
    };
    // tile and first x-slice of step j (a pair of x-slices) of a pass
    auto step_geom = [&](int j, int& x0, int& y0, int& z0, int& ks) {
        const int4 o = ms.org[j >> 1];
        ks = (j & 1) * 2;
        x0 = o.x;
        y0 = o.y;
        z0 = o.z;
    };

    int it = 0;  // global step counter across passes (stage / parity bookkeeping)
    int issued = 0;  // TMA thread: staged steps issued
    const int npass = (Kb + kSlots - 1) / kSlots;
    for (int pass = 0; pass < npass; ++pass) {
        const int p0 = pass * kSlots, ns = min(kSlots, Kb - p0);
        const int nn = (ns + 15) & ~15;  // MMA N of this pass
        // A pass of at most 128 slots runs transposed: the slots' weights are the A operand (M = 128, K-major)
        // and the converted gradient the B operand (N = 256 channels, MN-major), so a step issues three
        // MMAs of N = 256 instead of six narrow ones; the accumulator then holds slots in lanes, channels
        // in columns.
        const bool tr = ns <= 128;
        const uint32_t idesc = tr ? tc::idesc_bf16_f32(128, 256, /*A K-major*/ 0, /*B MN-major*/ 1)
                                  : tc::idesc_bf16_f32(128, nn, /*A MN-major*/ 1, /*B K-major*/ 0);
        // the pass's step list, padded to whole rounds of the operand ring with skipped steps (their
        // weights are zero) so that the MMA loop keeps one register set of descriptors per stage
        const int nsteps = ntiles * 2;
        uint64_t step_bits = nsteps >= 64 ? ~0ull : (1ull << nsteps) - 1;
        if (pass < kMaskPasses) {
            const uint64_t all = step_bits;
            step_bits = ((uint64_t)ms.smask[pass][1] << 32) | ms.smask[pass][0];
            if (__popcll(step_bits) & (kStages - 1)) {  // nsteps is even, so a skipped step exists
                const uint64_t skipped = all & ~step_bits;
                step_bits |= skipped & (~skipped + 1);  // the lowest one
            }
        }
        const int nact = __popcll(step_bits);
        StepList steps{step_bits};
        if (warp < 8) {
            // ---------------- converters: A = gF^T, thread = (8-channel chunk jc, 2 voxel rows) ----------
            const int jc = lane;                                     // channels c0 + 8 jc .. + 7
            const int mb = jc >> 4, a = (jc >> 3) & 1, jj = jc & 7;
            for (int sk = 0; sk < nact && ok; ++sk, ++it) {
                const int j = steps.next();
                const int st = it % kStages, gs = it % kGS;
                int x0, y0, z0, ks;
                step_geom(j, x0, y0, z0, ks);
                if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                if (kTma && ok) ok = tc::mbar_wait(&ms.gfull[gs], (it / kGS) & 1, err);
                if (!ok) break;
#pragma unroll
                for (int i4 = 0; i4 < 4; ++i4) {
                    const int kk = i4 >> 1;                // x-slice of the pair
                    const int r = warp * 2 + (i4 & 1);     // voxel row of the slice: (ly, lz) = (r / 4, r % 4)
                    const int v = kk * 16 + r;             // K index within the stage
                    float f[8];
                    if (kTma) {
                        const float4* src = reinterpret_cast<const float4*>(gstage + gs * kGBytes + v * (kCG * 4) + jc * 32);
                        const float4 u = src[0], w4 = src[1];
                        f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
                        f[4] = w4.x; f[5] = w4.y; f[6] = w4.z; f[7] = w4.w;
                    } else {
                        const int x = x0 + ks + kk, y = y0 + (r >> 2), z = z0 + (r & 3);
                        const bool vok = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
                        const int c = c0 + jc * 8;
                        const float* src = grad_feats + grid_row(G, x, y, z) * C + c;
                        if (vok && c + 7 < C && vec) {
                            const float4 u = *reinterpret_cast<const float4*>(src);
                            const float4 w4 = *reinterpret_cast<const float4*>(src + 4);
                            f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
                            f[4] = w4.x; f[5] = w4.y; f[6] = w4.z; f[7] = w4.w;
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) f[e] = (vok && c + e < C) ? src[e] : 0.0f;
                        }
                    }
                    uint4 h, l;
                    tc::split_bf16x2_p(make_float2(f[0], f[1]), h.x, l.x);
                    tc::split_bf16x2_p(make_float2(f[2], f[3]), h.y, l.y);
                    tc::split_bf16x2_p(make_float2(f[4], f[5]), h.z, l.z);
                    tc::split_bf16x2_p(make_float2(f[6], f[7]), h.w, l.w);
                    const int g8 = v >> 3, rr = v & 7;
                    // channel atom n = 2 mb + a at n KB, voxel octet g8 at 4 g8 KB: uniform strides, so the
                    // stage is both the A operand (two M-blocks of 128 channels) and a B operand of N = 256
                    const int off = mb * 2048 + a * 1024 + g8 * 4096 + rr * 128 + ((jj ^ rr) << 4);
                    *reinterpret_cast<uint4*>(a_stage(st, 0) + off) = h;
                    *reinterpret_cast<uint4*>(a_stage(st, 1) + off) = l;
                }
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&ms.full[st]);
                    if (kTma) tc::mbar_arrive(&ms.gempty[gs]);
                }
            }
            // partial-row offsets of the pass's slots for the epilogue, while the last MMAs run
            {
                const int sl = tid;  // 256 converter threads, one slot each
                int64_t ro = -1;
                if (sl < ns) {
                    const int g = block_lists[s0 + p0 + sl];
                    const GParams& gp = gparams[g];
                    const int lbx = __float_as_int(gp.w[3].y), lby = __float_as_int(gp.w[3].z), lbz = __float_as_int(gp.w[3].w);
                    const int uby = __float_as_int(gp.w[4].y), ubz = __float_as_int(gp.w[4].z);
                    const int blx = (lbx / kTile) / BX, bly = (lby / kTile) / BY, blz = (lbz / kTile) / BZ;
                    const int ey = (uby / kTile) / BY - bly + 1, ez = (ubz / kTile) / BZ - blz + 1;
                    ro = (int64_t)g2b_offsets[g] + ((bx - blx) * ey + (by - bly)) * ez + (bz - blz);
                    if (ro >= block_pair_cap) ro = -1;  // offsets come from the caller
                }
                ms.rowoff[sl] = ro;
            }
        } else if (warp < 16) {
            // ---------------- weight warps: thread = slot t, the 16 voxels of each of the step's x-slices -----
            // Over a tile the base-2 exponent of the weight is a quadratic in the local voxel (ks, ly, lz):
            //   k (d0 + h l)^T P (d0 + h l),  k = -log2(e) / 2,  d0 = tile-origin voxel centre - mean,
            // so its 10 coefficients are formed once per tile (its first step of the pass) and each x-slice
            // only adds the ks terms.  The y / z box masks of the tile are 0 / -inf terms added per
            // (ly, lz), the x mask decides the whole slice.  Voxel centres are linear within a tile (a tile
            // never spans two stacked scenes).
            const int t = tid - 256;
            const bool trow = t < (tr ? 128 : nn);  // rows the MMAs read (zero beyond the pass's slots)
            const bool slot = t < ns;
            if (pass == 0) {
                // log2(1 / max(D, eps)) of every voxel of the block's tiles (tile order of the steps); only
                // the weight warps read it, so only they wait for it (named barrier 2)
                for (int i = t; i < ntiles * kVoxPerTile; i += 256) {
                    const int ti = i >> 6;
                    int lx, ly, lz;
                    local_voxel(i & 63, lx, ly, lz);
                    const int tzi = ti % ntz, tyi = (ti / ntz) % nty, txi = ti / (ntz * nty);
                    const int x = (txa + txi) * kTile + lx, y = (tya + tyi) * kTile + ly, z = (tza + tzi) * kTile + lz;
                    float r = -INFINITY;
                    if (x < G.dims[0] && y < G.dims[1] && z < G.dims[2])
                        r = -log2f(fmaxf(density[grid_row(G, x, y, z)], kEps));
                    ms.lrd[i] = r;
                }
                asm volatile("bar.sync 2, 256;" ::: "memory");
            }
            if (trow) {  // this thread's slot record, read at each tile of the pass
                const GParams& src = gparams[slot ? block_lists[s0 + p0 + t] : 0];
#pragma unroll
                for (int wq = 0; wq < 5; ++wq) ms.prm[t].w[wq] = src.w[wq];
            }
            const float k = tc::kNegHalfLog2e;
            const float hx = G.h[0], hy = G.h[1], hz = G.h[2];
            float opa = 0.0f, A0 = 0.0f, Bx = 0.0f, By = 0.0f, Bz = 0.0f;
            float Qxx = 0.0f, Qyy = 0.0f, Qzz = 0.0f, Qxy = 0.0f, Qxz = 0.0f, Qyz = 0.0f;
            float my[4];
            float2 Zq01 = make_float2(0.f, 0.f), Zq23 = make_float2(0.f, 0.f);  // Qzz lz^2 + z box mask
            int xlo = 1, xhi = 0;
            bool yz_in = false;  // the slot's box meets the tile's y and z ranges
            int cur_tile = -1;
            for (int sk = 0; sk < nact && ok; ++sk, ++it) {
                const int j = steps.next();
                const int st = it % kStages;
                const int tj = j >> 1;  // tile of the step
                if (tj != cur_tile && trow) {  // first step of the pass in this tile
                    const int4 o = ms.org[tj];
                    const GParams& gp = ms.prm[t];
                    const float4 a = gp.w[0], b = gp.w[1], c = gp.w[2], d = gp.w[3], e4 = gp.w[4];
                    // P = [[b.x b.y b.z] [b.w c.x c.y] [c.z c.w d.x]]
                    const float dx = voxel_centre(G, 0, o.x) - a.x, dy = voxel_centre(G, 1, o.y) - a.y;
                    const float dz = voxel_centre(G, 2, o.z) - a.z;
                    const float qx = b.x * dx + b.y * dy + b.z * dz;    // (P d0)
                    const float qy = b.w * dx + c.x * dy + c.y * dz;
                    const float qz = c.z * dx + c.w * dy + d.x * dz;
                    const float ptx = b.x * dx + b.w * dy + c.z * dz;   // (P^T d0)
                    const float pty = b.y * dx + c.x * dy + c.w * dz;
                    const float ptz = b.z * dx + c.y * dy + d.x * dz;
                    opa = a.w;
                    A0 = k * (dx * qx + dy * qy + dz * qz);
                    Bx = k * hx * (qx + ptx);
                    By = k * hy * (qy + pty);
                    Bz = k * hz * (qz + ptz);
                    Qxx = k * hx * hx * b.x;
                    Qyy = k * hy * hy * c.x;
                    Qzz = k * hz * hz * d.x;
                    Qxy = k * hx * hy * (b.y + b.w);
                    Qxz = k * hx * hz * (b.z + c.z);
                    Qyz = k * hy * hz * (c.y + c.w);
                    xlo = __float_as_int(d.y) - o.x;
                    xhi = __float_as_int(e4.x) - o.x;
                    const int ylo = __float_as_int(d.z) - o.y, yhi = __float_as_int(e4.y) - o.y;
                    const int zlo = __float_as_int(d.w) - o.z, zhi = __float_as_int(e4.z) - o.z;
                    yz_in = ylo <= 3 && yhi >= 0 && zlo <= 3 && zhi >= 0;
                    float mz[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        my[i] = (i >= ylo && i <= yhi) ? 0.0f : -INFINITY;
                        mz[i] = (i >= zlo && i <= zhi) ? Qzz * (float)(i * i) : -INFINITY;
                    }
                    Zq01 = make_float2(mz[0], mz[1]);
                    Zq23 = make_float2(mz[2], mz[3]);
                }
                cur_tile = tj;
                if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                if (!ok) break;
#pragma unroll 1
                for (int kk = 0; kk < 2; ++kk) {
                const int ks = (j & 1) * 2 + kk;
                const bool act = slot && yz_in && ks >= xlo && ks <= xhi;
                if (trow) {
                    // pairs of z-consecutive voxels (lz = 0,1 and 2,3) in packed f32x2 arithmetic:
                    //   m = (Ay + Qzz lz^2 + z mask) + lz Bz2 + log2(1 / den_v),  w = o 2^m
                    float2 w[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) w[e] = make_float2(0.0f, 0.0f);
                    if (act) {
                        const float fk = (float)ks;
                        const float Ak = fmaf(fmaf(Qxx, fk, Bx), fk, A0);
                        const float Byk = fmaf(Qxy, fk, By), Bzk = fmaf(Qxz, fk, Bz);
                        const float4* L4 = reinterpret_cast<const float4*>(&ms.lrd[tj * kVoxPerTile + ks * 16]);
                        const float2 o2 = make_float2(opa, opa);
#pragma unroll
                        for (int ly = 0; ly < 4; ++ly) {
                            const float4 L = L4[ly];  // log2(1 / den) of the voxels (ly, 0..3); -inf outside the grid
                            const float Ay = fmaf(fmaf(Qyy, (float)ly, Byk), (float)ly, Ak) + my[ly];
                            const float Bz2 = fmaf(Qyz, (float)ly, Bzk);
                            const float2 A2 = make_float2(Ay, Ay), B2 = make_float2(Bz2, Bz2);
                            const float2 m01 = __fadd2_rn(__ffma2_rn(make_float2(0.0f, 1.0f), B2, __fadd2_rn(A2, Zq01)),
                                                          make_float2(L.x, L.y));
                            const float2 m23 = __fadd2_rn(__ffma2_rn(make_float2(2.0f, 3.0f), B2, __fadd2_rn(A2, Zq23)),
                                                          make_float2(L.z, L.w));
                            w[2 * ly] = __fmul2_rn(make_float2(tc::exp2_approx(m01.x), tc::exp2_approx(m01.y)), o2);
                            w[2 * ly + 1] = __fmul2_rn(make_float2(tc::exp2_approx(m23.x), tc::exp2_approx(m23.y)), o2);
                        }
                    }
                    uint4 h0, h1, l0, l1;
                    tc::split_bf16x2_p(w[0], h0.x, l0.x);
                    tc::split_bf16x2_p(w[1], h0.y, l0.y);
                    tc::split_bf16x2_p(w[2], h0.z, l0.z);
                    tc::split_bf16x2_p(w[3], h0.w, l0.w);
                    tc::split_bf16x2_p(w[4], h1.x, l1.x);
                    tc::split_bf16x2_p(w[5], h1.y, l1.y);
                    tc::split_bf16x2_p(w[6], h1.z, l1.z);
                    tc::split_bf16x2_p(w[7], h1.w, l1.w);
                    // K-major, 32-byte swizzle: row t = the slot's 16 voxels (32 bytes), chunk c at c ^ ((t / 4) % 2)
                    const int sw = (t >> 2) & 1;
                    const int off0 = (t >> 3) * 256 + (t & 7) * 32 + (sw << 4), off1 = off0 ^ 16;
                    *reinterpret_cast<uint4*>(b_stage(st, 0) + kk * kBSub + off0) = h0;
                    *reinterpret_cast<uint4*>(b_stage(st, 0) + kk * kBSub + off1) = h1;
                    *reinterpret_cast<uint4*>(b_stage(st, 1) + kk * kBSub + off0) = l0;
                    *reinterpret_cast<uint4*>(b_stage(st, 1) + kk * kBSub + off1) = l1;
                }
                }
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&ms.full[st]);
            }
        } else if (kTma && warp == 17 && lane == 0) {
            // ---------------- TMA thread: the step's gradient rows (two x-slices) into the staging ring -----
            for (int sk = 0; sk < nact && ok; ++sk, ++it) {
                const int j = steps.next();
                const int gs = it % kGS;
                int x0, y0, z0, ks;
                step_geom(j, x0, y0, z0, ks);
                if (it >= kGS) ok = tc::mbar_wait(&ms.gempty[gs], ((it / kGS) + 1) & 1, err);
                if (!ok) break;
                tc::mbar_arrive_expect_tx(&ms.gfull[gs], kGBytes);
                tc::tma_load_4d(tc::smem_u32(gstage + gs * kGBytes), &gmap, c0, z0, y0, x0 + ks - G.xoff, &ms.gfull[gs]);
                issued = it + 1;
            }
        } else if (warp == 16 && lane == 0) {
            // ---------------- MMA thread ----------------
            // Every stage's descriptors are formed once and kept in registers: the step loop is unrolled by
            // the stage count (a pass's step list comes in whole rounds of the ring, so stage s of a round
            // is its step j0 + s), and each step is one wait and two blocks of six MMAs (one per x-slice)
            // plus the commit that frees the stage.
            static_assert(kStages == 2 && kMB == 2, "the MMA loop is unrolled for two stages of two M-blocks");
            const uint64_t ao = (uint64_t)(kASub >> 4), bo = (uint64_t)(kBSub >> 4);  // the second x-slice
            const uint64_t adesc0 = tc::smem_desc(tc::smem_u32(a_stage(0, 0)), 1024, 4096, tc::kLayoutSw128);
            const uint64_t bdesc0 = tc::smem_desc(tc::smem_u32(b_stage(0, 0)), 16, 256, tc::kLayoutSw32);
            uint64_t dah[kStages][kMB], dal[kStages][kMB], dbh[kStages], dbl[kStages];
#pragma unroll
            for (int st = 0; st < kStages; ++st) {
                // the start-address field counts 16-byte units
                const uint64_t soff = (uint64_t)((st * kStageBytes) >> 4);
                dbh[st] = bdesc0 + soff;
                dbl[st] = dbh[st] + (uint64_t)(kBHalf >> 4);
#pragma unroll
                for (int mb = 0; mb < kMB; ++mb) {
                    dah[st][mb] = adesc0 + soff + (uint64_t)((mb * 2048) >> 4);
                    dal[st][mb] = dah[st][mb] + (uint64_t)(kAHalf >> 4);
                }
            }
            for (int j0 = 0; j0 < nact && ok; j0 += kStages) {
                const uint32_t par = (uint32_t)((it + j0) / kStages) & 1;
#pragma unroll
                for (int st = 0; st < kStages; ++st) {
                    ok = ok && tc::mbar_wait(&ms.full[st], par, err);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const bool acc = (j0 + st) > 0;
                    if (tr) {
                        tc::mma_f16_ss<tc::kColFill>(tmem, dbh[st], dah[st][0], idesc, acc);
                        tc::mma_f16_ss<tc::kColLastUse>(tmem, dbh[st], dal[st][0], idesc, true);
                        tc::mma_f16_ss(tmem, dbl[st], dah[st][0], idesc, true);
                        tc::mma_step1x3_commit(tmem, dbh[st] + bo, dbl[st] + bo, dah[st][0] + ao, dal[st][0] + ao, idesc,
                                               true, tc::smem_u32(&ms.empty[st]));
                    } else {
#pragma unroll
                        for (int mb = 0; mb < kMB; ++mb) {
                            const uint32_t d = tmem + (uint32_t)(mb * kSlots);
                            tc::mma_f16_ss<tc::kColFill>(d, dah[st][mb], dbh[st], idesc, acc);
                            tc::mma_f16_ss<tc::kColLastUse>(d, dah[st][mb], dbl[st], idesc, true);
                            tc::mma_f16_ss(d, dal[st][mb], dbh[st], idesc, true);
                        }
                        tc::mma_step2x3_commit(tmem, tmem + kSlots, dah[st][0] + ao, dal[st][0] + ao, dah[st][1] + ao,
                                               dal[st][1] + ao, dbh[st] + bo, dbl[st] + bo, idesc, true,
                                               tc::smem_u32(&ms.empty[st]));
                    }
                }
            }
            it += nact;
            tc::mma_commit(tc::smem_u32(&ms.mma_done));
        } else {
            it += nact;
        }

        ok = tc::mbar_wait_drain(&ms.mma_done, pass & 1, err) && ok;
        if (!ok) ms.fail = 1;
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
        // epilogue: warp w < 16 reads lanes 32*(w%4).. (channels) of M-block (w/4)%2, slot columns
        // 128*(w/8) .. +127; the next 16 columns load from TMEM while the current ones are stored
        if (warp < 16 && !ms.fail && tr) {
            // transposed pass: warp w reads lanes 32*(w%4).. (slots) and the 64 channel columns of (w/4);
            // a thread stores 16 consecutive channels of its slot's partial row per TMEM load
            const int q = warp & 3, cb = warp >> 2;
            const int sl = q * 32 + lane;
            const int64_t ro = sl < ns ? ms.rowoff[sl] : -1;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + cb * 64;
#pragma unroll 1
            for (int jc = 0; jc < 4; ++jc) {
                const int cc = c0 + cb * 64 + jc * 16;
                if (cc >= C) break;  // warp-uniform
                float v[16];
                if (nact > 0) {
                    tc::tmem_ld16(tbase + jc * 16, v);
                } else {  // no step of the pass: the accumulator was never written
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[e] = 0.0f;
                }
                if (ro >= 0) {
                    float* dst = partialF + ro * C + cc;
                    if (vec && cc + 16 <= C) {
#pragma unroll
                        for (int e = 0; e < 16; e += 4)
                            *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (cc + e < C) dst[e] = v[e];
                    }
                }
            }
        } else if (warp < 16 && !ms.fail) {
            const int q = warp & 3, mb = (warp >> 2) & 1, half = warp >> 3;
            const int c = c0 + mb * 128 + q * 32 + lane;
            const int jc0 = half * 8, jc1 = min(half * 8 + 8, (ns + 15) >> 4);  // warp-uniform
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + mb * kSlots;
            if (jc0 < jc1 && nact == 0) {  // no step of the pass: the accumulator was never written
                if (c < C)
                    for (int sl = jc0 * 16; sl < min(jc1 * 16, ns); ++sl) {
                        const int64_t ro = ms.rowoff[sl];
                        if (ro >= 0) partialF[ro * C + c] = 0.0f;
                    }
            } else if (jc0 < jc1) {
                float va[16], vb[16];
                tc::tmem_ld16(tbase + jc0 * 16, va);
                for (int jc = jc0; jc < jc1; ++jc) {
                    const bool more = jc + 1 < jc1;
                    if (more) tc::tmem_ld16_nowait(tbase + (jc + 1) * 16, vb);
                    if (c < C) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const int64_t ro = ms.rowoff[jc * 16 + e];
                            if (ro >= 0) partialF[ro * C + c] = va[e];
                        }
                    }
                    if (more) {
                        tc::tmem_wait_ld16(vb);
#pragma unroll
                        for (int e = 0; e < 16; ++e) va[e] = vb[e];
                    }
                }
            }
        }
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
    }
    // no copy may still be in flight when the CTA's shared memory is released (matters after a wait gave up)
    if (kTma && warp == 17 && lane == 0)
        for (int k = max(0, issued - kGS); k < issued; ++k) tc::mbar_wait_drain(&ms.gfull[k % kGS], (k / kGS) & 1, err);
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}
}  // namespace

// The feature-gradient pass: one CTA per (block, 256-channel group) with passes of 256 slots.
int launch_fpass_tc(const float* grad_feats, int C, const float* density, const GParams* gparams,
                    const int32_t* block_offsets, const int32_t* block_lists, const int32_t* g2b_offsets, int bx_begin,
                    int nbx, int nby, int nbz, const int B[3], int tx_begin, int tx_end, const Grid& G, float* partialF,
                    int64_t block_pair_cap, int* err, cudaStream_t s) {
    const int64_t nblocks = (int64_t)nbx * nby * nbz;
    if (nblocks <= 0 || C <= 0) return 0;
    const int ngroups = (C + kCG - 1) / kCG;
    const int vec = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(grad_feats) % 16 == 0);
    if (B[0] * B[1] * B[2] > kMaxBlockTiles) {
        set_error("fpass_tc: block of %dx%dx%d tiles exceeds %d", B[0], B[1], B[2], kMaxBlockTiles);
        return G2V_ERROR_INVALID_VALUE;
    }
    CUtensorMap gmap;
    memset(&gmap, 0, sizeof(gmap));
    const int ldims[3] = {G.xlen, G.dims[1], G.dims[2]};
    const bool tma = encode_grid_rows_f32(&gmap, grad_feats, ldims, C, kCG, kTile, kTile, 2);  // x-slice pairs
    auto kern = tma ? fpass_tc_kernel<true> : fpass_tc_kernel<false>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    const int64_t grid = nblocks * ngroups;
    G2V_TIMED("fpass_tc_kernel", s,
              kern<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(
                  gmap, grad_feats, C, density, gparams, block_offsets, block_lists, g2b_offsets, bx_begin, nby, nbz, B[0],
                  B[1], B[2], tx_begin, tx_end, ngroups, vec, G, partialF, block_pair_cap, err));
    G2V_LAUNCH_CHECK("fpass_tc_kernel");
    return 0;
}

}  // namespace g2v
