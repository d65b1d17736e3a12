// tc_pipe_probe2.cu -- pipeline probe with per-stage operands: every stage holds its own A and B, which the
// producer warps rewrite (16-byte stores) before arriving, like the kernels' producers; optionally 13 more
// warps run dependent FMA chains on all schedulers while the MMA thread works.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "g2v_tc.cuh"
using namespace g2v;

template <int N, int S, int R, int WRITE, int EXTRA_KB, int BUSY>
__global__ void __launch_bounds__(576, 1) pipe(int steps, unsigned long long* out, int* err) {
    extern __shared__ __align__(1024) unsigned char sm[];
    __shared__ uint64_t full[8], empty[8], done;
    __shared__ uint32_t tbase;
    constexpr int kA = 4096 * (S >= 12 ? 2 : 1);   // one or two M-blocks of A
    constexpr int kB = N * 32;
    constexpr int kStage = kA + kB;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < R * kStage / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sm)[i] = 0;
    if (tid == 0) {
        for (int i = 0; i < R; ++i) { tc::mbar_init(&full[i], 4); tc::mbar_init(&empty[i], 1); }
        tc::mbar_init(&done, 1);
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(&tbase, 512);
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tbase;
    bool ok = true;
    if (warp < 4) {
        unsigned char* scratch = sm + R * kStage;
        for (int it = 0; it < steps && ok; ++it) {
            const int st = it % R;
            if (it >= R) ok = tc::mbar_wait(&empty[st], ((it / R) + 1) & 1, err);
            if (!ok) break;
            if (WRITE) {
                uint4 v = make_uint4(0, 0, 0, 0);
                for (int q = tid; q < kStage / 16; q += 128) *reinterpret_cast<uint4*>(sm + st * kStage + q * 16) = v;
            }
            for (int q = tid; q < EXTRA_KB * 64; q += 128) *reinterpret_cast<uint4*>(scratch + (q * 16) % 16384) = make_uint4(it, 0, 0, 0);
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&full[st]);
        }
    } else if (warp >= 5 && BUSY) {
        // busy warps: dependent FMA chains until the MMA thread is done (bounded by a step count)
        float x = (float)tid, y = 1.0001f;
        for (int i = 0; i < steps * 40; ++i) { x = fmaf(x, y, 1e-7f); y = fmaf(y, 0.99999f, 1e-6f); }
        if (x == 12345.f) out[2] = 1;
    } else if (tid == 128) {
        const uint32_t idesc = tc::idesc_bf16_f32(128, N, 1, 1);
        const long long t0 = clock64();
        for (int it = 0; it < steps && ok; ++it) {
            const int st = it % R;
            ok = tc::mbar_wait(&full[st], (it / R) & 1, err);
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t a = tc::smem_u32(sm + st * kStage), b = a + kA;
            const uint64_t bd = tc::smem_desc(b, 1024, 2048, tc::kLayoutSw128);
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const int mb = (S >= 12) ? ((s / 3) & 1) : 0;
                const uint64_t ad = tc::smem_desc(a + mb * 4096, 1024, 2048, tc::kLayoutSw128);
                tc::mma_f16_ss(tmem + (uint32_t)(((s / 3) & 1) * N), ad, bd, idesc, it > 0 || s > 5);
            }
            tc::mma_commit(tc::smem_u32(&empty[st]));
        }
        tc::mma_commit(tc::smem_u32(&done));
        tc::mbar_wait_drain(&done, 0, err);
        atomicAdd(out, (unsigned long long)(clock64() - t0));
        atomicAdd(out + 1, 1ull);
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

template <int N, int S, int R, int WRITE, int EXTRA_KB, int BUSY>
void run(const char* name, int sms) {
    unsigned long long* out; int* err;
    cudaMalloc(&out, 24); cudaMalloc(&err, 4);
    cudaMemset(out, 0, 24); cudaMemset(err, 0, 4);
    auto k = pipe<N, S, R, WRITE, EXTRA_KB, BUSY>;
    const int smem = 200 * 1024;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const int steps = 4000;
    k<<<sms, BUSY ? 576 : 160, smem>>>(100, out, err);
    cudaDeviceSynchronize();
    cudaMemset(out, 0, 24);
    k<<<sms, BUSY ? 576 : 160, smem>>>(steps, out, err);
    cudaError_t ce = cudaDeviceSynchronize();
    unsigned long long h[2]; int herr; cudaMemcpy(h, out, 16, cudaMemcpyDeviceToHost); cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
    const double cyc = (double)h[0] / (double)(h[1] ? h[1] : 1) / steps;
    const double ideal = (double)S * 128 * N * 16 / 4096.0;
    printf("%-60s cycles/step %7.1f  (MMA ideal %5.0f, %3.0f%%)  %s err %d\n", name, cyc, ideal, 100.0 * ideal / cyc,
           cudaGetErrorString(ce), herr);
    cudaFree(out); cudaFree(err);
}

int main() {
    int sms = 0; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    run<128, 6, 7, 0, 0, 0>("N128 S6 R7 per-stage operands, static", sms);
    run<128, 6, 7, 1, 0, 0>("N128 S6 R7 per-stage operands, rewritten (8 KB)", sms);
    run<128, 6, 7, 1, 16, 0>("N128 S6 R7 rewritten + 16 KB other stores", sms);
    run<128, 6, 7, 1, 16, 1>("N128 S6 R7 rewritten + 16 KB, + 13 busy FMA warps", sms);
    run<128, 12, 4, 0, 0, 0>("N128 S12 R4 per-stage (2 M-blocks), static", sms);
    run<128, 12, 4, 1, 0, 0>("N128 S12 R4 per-stage, rewritten (12 KB)", sms);
    run<128, 12, 4, 1, 32, 0>("N128 S12 R4 rewritten + 32 KB other stores", sms);
    run<128, 12, 4, 1, 32, 1>("N128 S12 R4 rewritten + 32 KB, + 13 busy FMA warps", sms);
    run<256, 6, 4, 0, 0, 0>("N256 S6 R4 per-stage, static", sms);
    run<256, 6, 4, 1, 0, 0>("N256 S6 R4 per-stage, rewritten (12 KB)", sms);
    run<256, 6, 4, 1, 32, 0>("N256 S6 R4 rewritten + 32 KB other stores", sms);
    run<256, 6, 4, 1, 32, 1>("N256 S6 R4 rewritten + 32 KB, + 13 busy FMA warps", sms);
    return 0;
}
