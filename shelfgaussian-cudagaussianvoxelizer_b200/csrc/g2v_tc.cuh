// g2v_tc.cuh -- sm_100a building blocks: shared-memory descriptors, tcgen05 MMA / TMEM, mbarriers,
// cp.async.  Inline PTX, following the operand encodings of the PTX ISA for tcgen05 (the bit layout
// of the descriptors matches cute/arch/mma_sm100_desc.hpp).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <cstring>

namespace g2v {
namespace tc {

// Error bit set in the caller-provided device error word when a bounded wait gives up.
constexpr int kErrWaitTimeout = 1;
// Suspend-time hint of one try_wait (ns) and the limit of one bounded wait (ns).
constexpr uint32_t kWaitHintNs = 1000000u;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05): start address, leading / stride byte offsets (16-byte
// units), version 1, layout type in bits 61-63 (0 = no swizzle, 2 = 128-byte, 4 = 64-byte, 6 = 32-byte
// swizzle).  In a swizzled layout the 16-byte chunk index of an address (bits 4..) is XORed with its
// 128-byte row index (bits 7..): 3 bits for 128-byte, 2 for 64-byte, 1 for 32-byte swizzle, repeating
// every 1024 / 512 / 256 bytes, so atoms start on those boundaries.
constexpr int kLayoutNone = 0;
constexpr int kLayoutSw128 = 2;
constexpr int kLayoutSw64 = 4;
constexpr int kLayoutSw32 = 6;

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, int layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(layout & 7) << 61;
    return d;
}

// Instruction descriptor of kind::f16 with f16 A/B and f32 accumulation.
// a_mn / b_mn: operand stored MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, int a_mn, int b_mn) {
    return (1u << 4)                      // D format f32
           | (0u << 7) | (0u << 10)       // A, B format f16
           | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// A-operand collector use of an MMA: kColNone reads A from shared memory; kColFill reads it and keeps it
// in the tensor core's collector buffer; kColLastUse takes A from the collector (the previous MMA's A,
// which the descriptor must repeat) and releases it.  hi*hi + hi*lo of a split contraction share A_hi.
constexpr int kColNone = 0, kColFill = 1, kColLastUse = 2;

// D[tmem] (+)= A[smem] * B[smem], issued by one thread.
template <int kCol = kColNone>
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
    if constexpr (kCol == kColFill)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
    else if constexpr (kCol == kColLastUse)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void mma_commit(uint32_t mbar_saddr) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar_saddr)
                 : "memory");
}

// One pipeline step of a split-operand contraction over two accumulators: for m = 0, 1
//     D_m (+)= Ah_m * Bh + Ah_m * Bl + Al_m * Bh
// (six MMAs, the first of each accumulator overwriting it when `accumulate` is false), then a commit
// that arrives on `mbar` once they have completed.  One asm block, so the issuing thread spends no
// instructions between the MMAs.
__device__ __forceinline__ void mma_step2x3_commit(uint32_t d0, uint32_t d1, uint64_t ah0, uint64_t al0, uint64_t ah1,
                                                   uint64_t al1, uint64_t bh, uint64_t bl, uint32_t idesc,
                                                   bool accumulate, uint32_t mbar) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t"
        "setp.ne.b32 p, %9, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%0], %2, %6, %8, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%0], %2, %7, %8, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %6, %8, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%1], %4, %6, %8, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%1], %4, %7, %8, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %5, %6, %8, t;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%10];\n\t}\n" ::"r"(d0),
        "r"(d1), "l"(ah0), "l"(al0), "l"(ah1), "l"(al1), "l"(bh), "l"(bl), "r"(idesc), "r"((uint32_t)accumulate),
        "r"(mbar)
        : "memory");
}

// One pipeline step over one accumulator: D (+)= Ah * Bh + Ah * Bl + Al * Bh, then the commit that
// arrives on `mbar` once the three MMAs have completed (one asm block, like mma_step2x3_commit).
__device__ __forceinline__ void mma_step1x3_commit(uint32_t d, uint64_t ah, uint64_t al, uint64_t bh, uint64_t bl,
                                                   uint32_t idesc, bool accumulate, uint32_t mbar) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%0], %1, %3, %5, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%0], %1, %4, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %3, %5, t;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t}\n" ::"r"(d),
        "l"(ah), "l"(al), "l"(bh), "l"(bl), "r"(idesc), "r"((uint32_t)accumulate), "r"(mbar)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM allocation by one full warp; the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 16 columns of 32-bit words from TMEM (thread i of the warp gets lane base+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// tmem_ld16 without the wait: the registers are valid only after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Waits for this thread's TMEM loads; v (the registers of the last tmem_ld16_nowait) is passed through
// the wait so that the compiler cannot read it before the load has completed.
__device__ __forceinline__ void tmem_wait_ld16(float (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
                 :
                 : "memory");
}

// ---------------------------------------------------------------------------------------------
// mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Global nanosecond timer (bounds of the waits below).
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// One try_wait with a suspend-time hint: the thread sleeps until the phase completes (or the hint
// elapses) instead of returning at once, so hand-offs cost no polling loop.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_saddr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar_saddr), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    return done != 0;
}

// Non-blocking test of the phase: true when it has already completed.  A phase that is complete by the
// time a consumer reaches it is the common case of a deep ring; the test avoids try_wait's suspend path.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar_saddr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar_saddr), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait until the phase with the given parity has completed.  Bounded: after kWaitLimitNs of waiting it
// records kErrWaitTimeout in *err and returns false instead of waiting forever; once any wait of any CTA
// has given up (*err != 0), later waits that do not complete at once return false, so that the whole
// grid drains quickly.  The error word (global memory) is read only on that slow path.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    const uint32_t a = smem_u32(bar);
    if (mbar_test_wait(a, parity)) return true;
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(a, parity)) return true;
        if (*reinterpret_cast<volatile int*>(err) != 0) return false;
        if (global_ns() - t0 > kWaitLimitNs) break;
    }
    atomicOr(err, kErrWaitTimeout);
    return false;
}

// Wait for a commit that is always issued (the end-of-work commit of the MMA thread, the completion of
// a copy already issued), also after another wait has given up, so that nothing is in flight when the
// kernel frees its TMEM or shared memory.  Bounded like mbar_wait; returns false when *err is set.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, int* err) {
    const uint32_t a = smem_u32(bar);
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(a, parity)) return *reinterpret_cast<volatile int*>(err) == 0;
        if (global_ns() - t0 > kWaitLimitNs) break;
    }
    atomicOr(err, kErrWaitTimeout);
    return false;
}

// ---------------------------------------------------------------------------------------------
// cp.async (16 bytes; src_bytes = 0 fills zeros) and the async-proxy fence for operands written with
// ordinary stores.
__device__ __forceinline__ void cp_async16(uint32_t dst_saddr, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst_saddr), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// float -> (hi, lo) half pair with x ~= hi + lo to ~22 bits (values must be within the half range).
__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

// float -> (hi, lo) bf16 pair with x ~= hi + lo to ~2^-17 relative (full float range, no scaling needed).
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// Two floats -> packed bf16x2 hi / lo words (element x0 in the low half, like consecutive bf16 in
// memory) with x ~= hi + lo as in split_bf16; three instructions per element.
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
    const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xffff0000u);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(x1 - h1), "f"(x0 - h0));
}

// split_bf16x2 of a float pair with the remainder formed by one packed f32x2 operation (sm_100):
// x.x goes to the low half of each word.
__device__ __forceinline__ void split_bf16x2_p(float2 x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x.y), "f"(x.x));
    const float2 h = make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u));
    const float2 r = __ffma2_rn(h, make_float2(-1.0f, -1.0f), x);  // x - h, exact
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r.y), "f"(r.x));
}

// Two floats -> packed f16x2 hi / lo words (x0 in the low half) with x ~= hi + lo as in split_half.
__device__ __forceinline__ void split_half2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
    __half2 h2;
    memcpy(&h2, &hi, 4);
    const float2 hf = __half22float2(h2);
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(x1 - hf.y), "f"(x0 - hf.x));
}

// split_half2 with the hi half rounded to 11 significant bits by Veltkamp's splitting, c = (2^13 + 1) x,
// h = c - (c - x) (packed f32x2 operations on the FMA pipes), so that converting h to f16 is exact (for
// |x| >= 2^-14; below, f16 subnormals round h once more, an error under 2^-24 of the 2^14..2^15 range the
// splat scales its weights to) and no f16 -> f32 conversion is needed for the remainder: two conversions per
// pair instead of four.
__device__ __forceinline__ void split_half2_v(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const float2 x = make_float2(x0, x1), m1 = make_float2(-1.0f, -1.0f);
    const float2 c = __fmul2_rn(x, make_float2(8193.0f, 8193.0f));
    const float2 h = __ffma2_rn(__ffma2_rn(x, m1, c), m1, c);  // c - (c - x)
    const float2 r = __ffma2_rn(h, m1, x);                      // x - h, exact
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(h.y), "f"(h.x));
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r.y), "f"(r.x));
}

// 2^x with the hardware approximation (ex2.approx.ftz).
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// -1/2 * log2(e): exp(-m/2) = 2^(kNegHalfLog2e * m).
constexpr float kNegHalfLog2e = -0.72134752044448170368f;

// Instruction descriptor of kind::f16 with bf16 A/B and f32 accumulation.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace tc
}  // namespace g2v

namespace g2v {
namespace tc {

// ---------------------------------------------------------------------------------------------
// TMA and mbarrier transaction helpers (single CTA, this CTA's own shared memory only).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// The mbarrier receives one arrival when all cp.async issued so far by this thread have completed.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst_saddr, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst_saddr), "l"(src) : "memory");
}
// Four rows (row0..row3) x one box width starting at column `col` of a 2-D tensor map, written as four
// consecutive box rows at dst; completion is counted in bytes on `bar`.
__device__ __forceinline__ void tma_gather4(uint32_t dst_saddr, const void* tmap, int col, int r0, int r1, int r2,
                                            int r3, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst_saddr),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
        : "memory");
}

// Tiled 4-D load of one box at coordinates (c0 innermost .. c3) into shared memory; completion is
// counted in bytes on `bar`.  c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_4d(uint32_t dst_saddr, const void* tmap, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst_saddr),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

// L2 eviction-priority policies (createpolicy) for the cache-hinted copies below.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// cp_async16 with an L2 cache policy.
__device__ __forceinline__ void cp_async16_hint(uint32_t dst_saddr, const void* src, uint32_t src_bytes,
                                                uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(dst_saddr), "l"(src),
                 "r"(src_bytes), "l"(policy)
                 : "memory");
}
// tma_load_4d with an L2 cache policy.
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst_saddr, const void* tmap, int c0, int c1, int c2, int c3,
                                                 uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst_saddr),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Tiled 4-D store of a box from shared memory to global memory (bulk-group completion) with an L2
// cache policy.  c0 * element size must be a multiple of 16 bytes and no coordinate may be negative;
// the parts of the box beyond the tensor are not written.
__device__ __forceinline__ void tma_store_4d_hint(const void* tmap, uint32_t src_saddr, int c0, int c1, int c2, int c3,
                                                  uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group.L2::cache_hint"
        " [%0, {%2, %3, %4, %5}], [%1], %6;" ::"l"(reinterpret_cast<uint64_t>(tmap)),
        "r"(src_saddr), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N bulk groups of this thread still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until all bulk groups of this thread have completed (writes visible).
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace tc
}  // namespace g2v

namespace g2v {
// Parameters of one Gaussian as five 16-byte words: (mean, opacity), P[0..3], P[4..7], (P[8], lb.xyz),
// (ub.xyz, pad); lb/ub are int32 bit patterns.  Built by launch_pack_params, read by the tensor-core
// kernels with 16-byte loads.
struct __align__(16) GParams {
    float4 w[5];
};
int launch_pack_params(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                       const int32_t* ub, int64_t n, GParams* out, cudaStream_t s);
}  // namespace g2v

namespace g2v {
namespace tc {
// ---------------------------------------------------------------------------------------------
// CTA pairs (a cluster of two CTAs sharing one tcgen05 MMA, cta_group::2).  The even CTA of the pair
// (rank 0, the leader) issues the MMAs; the A operand's M rows and the B operand's N rows are split
// between the two CTAs' shared memory at the same offsets, and each CTA's TMEM holds the accumulator
// rows of its own A rows over all N columns.  Producers of the other CTA reach the leader's mbarriers
// through shared::cluster addresses; the leader's commits arrive on the same barrier offset in both
// CTAs.  Every load of the pair is a plain per-CTA load (no multicast).
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the variable at shared::cta address `saddr` in the cluster's CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
// Arrive (release at cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Relaxed arrive on another CTA's mbarrier: no release fence.  For hand-offs whose data is already in
// place and visible within its own CTA when the arrive is issued (the arriving thread acquired it), where
// a cluster-scope release costs ~1600 cycles per arrive.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// try_wait with acquire at cluster scope: for phases completed by arrivals or transfers of the other CTA.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_saddr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar_saddr), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    return done != 0;
}
// Bounded wait like mbar_wait, with cluster-scope acquire.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait_cluster(a, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_cluster(a, parity)) return true;
        if (*reinterpret_cast<volatile int*>(err) != 0) return false;
        if (global_ns() - t0 > kWaitLimitNs) break;
    }
    atomicOr(err, kErrWaitTimeout);
    return false;
}
// 4-byte store into the other CTA's shared memory whose completion counts 4 bytes on that CTA's mbarrier
// (both given as shared::cluster addresses).
__device__ __forceinline__ void st_async_f32(uint32_t cluster_addr, float v, uint32_t cluster_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(cluster_addr),
                 "r"(__float_as_uint(v)), "r"(cluster_bar)
                 : "memory");
}
// TMEM allocation for a CTA pair: one warp of each CTA (same warp index, same destination offset).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A * B over the pair (M = 256: rows 0-127 from the leader's A, 128-255 from the other
// CTA's; B's N rows: the first N/2 from the leader, the rest from the other CTA); one leader thread.
template <int kCol = kColNone>
__device__ __forceinline__ void mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                bool accumulate) {
    if constexpr (kCol == kColFill)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16.collector::a::fill [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
    else if constexpr (kCol == kColLastUse)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16.collector::a::lastuse [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
}
// Arrive on the mbarrier at shared::cta offset `mbar_saddr` in every CTA of `cta_mask` once all prior
// pair MMAs of this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t mbar_saddr, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            mbar_saddr),
        "h"(cta_mask)
        : "memory");
}
// All threads of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 32 lanes x 8 columns of 32-bit words from TMEM (thread i of the warp gets lane base + i).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
}  // namespace tc
}  // namespace g2v
