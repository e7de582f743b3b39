// esa_noalloc.cu -- esa_scan_fwd_noalloc: the forward scan for callers that
// cannot allocate device memory.
//
// esa_scan_fwd needs a caller-provided workspace whenever it takes the
// time-parallel (decoupled-lookback) kernel.  Some callers have no device
// allocator to get one from: a C host program or a foreign-language binding
// that receives its input and output buffers from elsewhere, or code whose
// device memory plan is fixed before it runs and must not grow per call.
// This entry point runs that same lookback kernel with its scratch taken from
// a fixed array in this file instead, so it allocates nothing.
//
// The array is a file-scope __device__ object: every GPU on which the library
// is loaded holds its ESA_NOALLOC_SCRATCH_BYTES until the process exits.  Host
// code cannot use the array's name as a device address, so the first call on
// each device looks the address up with cudaGetSymbolAddress (with that device
// current) and caches it; make that first call before any stream capture.
// All calls share the one array, and it keeps the previous call's contents:
// the launch clears the part that must start at zero (the tile ticket and the
// lookback flags) before the kernel runs.  Calls that overlap on the GPU (for
// example on two streams at once) would race on the array.
#include <mutex>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_scan_common.cuh"

#define ESA_EXPORT __attribute__((visibility("default")))

namespace esa {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[ESA_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device (looked up once
// per device); null, with the error recorded, if the lookup fails.
void* noalloc_scratch(int dev) {
    static void* cache[64] = {nullptr};
    static std::mutex mu;
    if (dev < 0 || dev >= 64) {
        set_error(ESA_ERR_CUDA, "device index out of range for the scratch table");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            set_error(ESA_ERR_CUDA, std::string("scratch address lookup: ") + cudaGetErrorString(e));
            return nullptr;
        }
        cache[dev] = p;
    }
    return cache[dev];
}

bool rows_aligned16(const void* p, int64_t hd, int es) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && ((hd * es) % 16 == 0);
}

}  // namespace
}  // namespace esa

using namespace esa;

extern "C" ESA_EXPORT int esa_scan_fwd_noalloc(const void* A, const void* B, void* E, int64_t nb,
                                               int64_t T, int64_t hd, int dtype, int compass,
                                               const void* e0, void* e_last, void* stream) {
    clear_error();
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    if (nb < 0 || T < 0 || hd < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "negative dimension");
    if (compass <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "compass must be a positive integer");
    if (T > 0x7fffffffLL || nb > 0x7fffffffLL || hd > 0x7fffffffLL)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "dimension exceeds 2^31 - 1");
    const size_t need = lookback_workspace_bytes(nb, T, hd, es, compass);
    if (need > (size_t)ESA_NOALLOC_SCRATCH_BYTES)
        return set_error(ESA_ERR_WORKSPACE,
                         "esa_scan_fwd_noalloc: this problem needs " + std::to_string(need) +
                             " bytes of scratch, more than the fixed " +
                             std::to_string((size_t)ESA_NOALLOC_SCRATCH_BYTES) +
                             " bytes it has; use esa_scan_fwd with a workspace instead");
    if (nb * T * hd == 0) return ESA_OK;
    if (!A || !B || !E) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");

    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
    void* scratch = noalloc_scratch(dev);
    if (scratch == nullptr) return ESA_ERR_CUDA;

    ScanCall c{};
    c.kind = Kind::FwdPlain;
    c.tin = c.te = dtype;
    c.a.in[0] = {static_cast<const char*>(A), hd};
    c.a.in[1] = {static_cast<const char*>(B), hd};
    c.a.out[0] = {static_cast<char*>(E), hd};
    c.a.nb = nb;
    c.a.T = T;
    c.a.hd = hd;
    c.a.e0 = e0;
    c.a.e_last = e_last;
    c.a.status = status_ptr(dev);
    if (c.a.status == nullptr) return set_error(ESA_ERR_CUDA, "cannot resolve the device status word");
    c.compass = compass;
    c.ws = scratch;
    c.ws_bytes = ESA_NOALLOC_SCRATCH_BYTES;
    c.stream = static_cast<cudaStream_t>(stream);
    c.bulk_ok = rows_aligned16(A, hd, es) && rows_aligned16(B, hd, es) && rows_aligned16(E, hd, es);
    // rows the bulk copies cannot stage need no scratch: one thread per channel
    if (!c.bulk_ok) return sequential_scan_launch(c);
    return lookback_scan_launch(c);
}
