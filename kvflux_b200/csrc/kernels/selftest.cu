// Self-test of device-side failure detection: the bounded mbarrier waits that
// every TMA/tcgen05 kernel here uses, run on a barrier that nothing completes.
// Nothing is in flight on that barrier (no copy, no MMA), so giving up is
// clean: each wait raises KVFX_FLAG_TIMEOUT and returns false, the kernel
// exits, and the context stays usable.
#include "common.cuh"
#include "launch.h"

namespace kvfx {
namespace {

__device__ int g_wait_result[2];

// Warp 0: the inline wait (mbar_wait); warp 1: the out-of-line one
// (mbar_wait_lean). Lane 0 of each records whether its wait completed.
__global__ void wait_timeout_kernel(unsigned* status) {
    __shared__ uint64_t bar;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);  // one arrival expected; none is ever made
        fence_mbarrier_init();
    }
    __syncthreads();
    if (lane == 0) {
        const bool done = warp == 0 ? mbar_wait(&bar, 0, status) : mbar_wait_lean(&bar, 0, status);
        g_wait_result[warp] = done ? 1 : 0;
    }
}

}  // namespace

cudaError_t launch_wait_selftest(unsigned* status, cudaStream_t s, int* completed) {
    const int init[2] = {-1, -1};
    cudaError_t e = cudaMemcpyToSymbolAsync(g_wait_result, init, sizeof(init), 0, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return e;
    wait_timeout_kernel<<<1, 64, 0, s>>>(status);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = cudaMemcpyFromSymbolAsync(completed, g_wait_result, sizeof(init), 0, cudaMemcpyDeviceToHost, s)) !=
        cudaSuccess)
        return e;
    return cudaStreamSynchronize(s);
}

}  // namespace kvfx
