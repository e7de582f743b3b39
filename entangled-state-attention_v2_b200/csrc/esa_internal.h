// esa_internal.h -- host-side declarations shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace esa {

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
// Clears this thread's last error.
void clear_error();
// Number of SMs of `device` (cached).
int device_sm_count(int device);

size_t scan_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass);
int device_status(int device, int clear, unsigned* status);

int scan_fwd(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd, int dtype,
             int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes, cudaStream_t s);
int scan_rev(const void* A, const void* E, const void* dE, void* dA, void* dB, int64_t nb, int64_t T,
             int64_t hd, int dtype, int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
             cudaStream_t s);
int gated_scan_fwd(const void* g, const void* v, int64_t rrs, int raw_dtype, void* E, int e_dtype,
                   int64_t nb, int64_t T, int64_t hd, float gmin, float gmax, int round_ab,
                   int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes,
                   cudaStream_t s);
int gated_scan_bwd(const void* g, const void* v, int64_t rrs, int raw_dtype, const void* E,
                   const void* dE, int e_dtype, void* dg, void* dv, int64_t drs, int draw_dtype,
                   int64_t nb, int64_t T, int64_t hd, float gmin, float gmax, int round_ab,
                   int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
                   cudaStream_t s);
int lightning_step(const void* qgv, int64_t qrs, int qdt, const void* state, void* new_state,
                   int sdt, void* z, int zdt, int64_t nb, int64_t C, float gmin, float gmax,
                   float eps, cudaStream_t s);

inline int dtype_size(int dtype) {
    switch (dtype) {
        case 0: return 2;
        case 1: return 2;
        case 2: return 4;
        case 3: return 8;
        default: return 0;
    }
}

}  // namespace esa
