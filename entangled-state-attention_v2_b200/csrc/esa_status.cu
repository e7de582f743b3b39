// esa_status.cu -- the per-device status word of the scan kernels.
//
// Kernels OR ESA_STATUS_* bits into it when a bounded wait runs out.  A
// __device__ variable lives once in each device's context; kernels in the
// other translation units receive its address (status_ptr) as an argument.
#include <mutex>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"

namespace esa {

__device__ unsigned int g_device_status = 0;

unsigned* status_ptr(int device) {
    static unsigned* cache[64] = {nullptr};
    static std::mutex mu;
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[device] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) cache[device] = static_cast<unsigned*>(p);
    }
    return cache[device];
}

int device_status(int device, int clear, unsigned* status) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned));
    if (e == cudaSuccess && clear) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned));
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("device status: ") + cudaGetErrorString(e));
    return ESA_OK;
}

}  // namespace esa
