// esa_selftest.cu -- a device-side check of the bounded-wait machinery.
//
// Every spin-wait in the scan kernels is bounded: a wait on an mbarrier phase
// (the TMA copies, mbar_wait_bounded) or on another CTA's flag gives up after
// kWaitBudgetNs of %globaltimer (or kWaitMaxIters polls), ORs a bit into the
// device status word and lets the kernel return, so the context stays usable.
// This entry point runs the strip kernels' own mbar_wait_bounded on an
// mbarrier that nothing ever arrives on, so that a test can see the wait run
// out, the status bit set and the next launch succeed -- without a fault, a
// trap or a hang.
#include "../../include/esa_b200.h"
#include "esa_internal.h"
#include "esa_scan_common.cuh"

namespace esa {
namespace {

__device__ unsigned g_selftest_out[2];

__global__ void wait_selftest_kernel(unsigned* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    const unsigned long long t0 = globaltimer_ns();
    const bool ok = mbar_wait_bounded(&bar, 0u, status);  // no arrival: runs out
    const unsigned long long t1 = globaltimer_ns();
    if (threadIdx.x == 0) {
        g_selftest_out[0] = ok ? 1u : 0u;
        g_selftest_out[1] = (unsigned)((t1 - t0) / 1000000ull);
    }
}

}  // namespace

int wait_selftest(unsigned* completed, unsigned* waited_ms, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned* status = status_ptr(dev);
    if (status == nullptr) return set_error(ESA_ERR_CUDA, "cannot resolve the device status word");
    wait_selftest_kernel<<<1, 32, 0, s>>>(status);
    cudaError_t e = cudaGetLastError();
    unsigned out[2] = {0, 0};
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(out, g_selftest_out, sizeof(out));
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("wait self-test: ") + cudaGetErrorString(e));
    if (completed) *completed = out[0];
    if (waited_ms) *waited_ms = out[1];
    return ESA_OK;
}

}  // namespace esa
