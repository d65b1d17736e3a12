// g2v_selftest.cu -- exercise of the bounded-wait failure path (g2v_debug_wait_timeout).
//
// One CTA waits on an mbarrier that nothing ever arrives at, with the same bounded wait the tensor-core
// kernels use; the wait gives up after its time limit, records kErrWaitTimeout in the device error word
// and the kernel returns, leaving the context usable.  No trap, no fault, no unbounded spin, and no
// device allocation (the result flag is a library variable).
#include "g2v_internal.cuh"
#include "g2v_tc.cuh"

namespace g2v {

__device__ int g_wait_gave_up = 0;

namespace {
__global__ void wait_timeout_kernel(int* err) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);  // expects one arrival that never comes
        tc::mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) g_wait_gave_up = tc::mbar_wait(&bar, 0, err) ? 0 : 1;
}
}  // namespace

int launch_wait_timeout(int* err, cudaStream_t s, int* gave_up_host) {
    wait_timeout_kernel<<<1, 32, 0, s>>>(err);
    G2V_LAUNCH_CHECK("wait_timeout_kernel");
    G2V_CUDA(cudaMemcpyFromSymbolAsync(gave_up_host, g_wait_gave_up, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
    G2V_CUDA(cudaStreamSynchronize(s));
    return 0;
}

}  // namespace g2v
