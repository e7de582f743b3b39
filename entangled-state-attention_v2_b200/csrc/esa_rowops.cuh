// esa_rowops.cuh -- row-wise element access for the readout and layer-norm
// kernels: loads and stores of one element or of 8 consecutive elements of
// a runtime dtype code (ESA_DTYPE_*), widened to / rounded from the
// accumulator type, and a warp-shuffle sum.
#pragma once

#include "esa_scan_common.cuh"

namespace esa {
namespace rowops {

// ---- element access by runtime dtype code ----------------------------------
template <typename A>
__device__ __forceinline__ A load1(const char* p, int dt) {
    switch (dt) {
        case ESA_DTYPE_F16: return A(__half2float(*reinterpret_cast<const __half*>(p)));
        case ESA_DTYPE_BF16: return A(__bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p)));
        case ESA_DTYPE_F32: return A(*reinterpret_cast<const float*>(p));
        default: return A(*reinterpret_cast<const double*>(p));
    }
}

template <typename A>
__device__ __forceinline__ void store1(char* p, int dt, A x) {
    switch (dt) {
        case ESA_DTYPE_F16: *reinterpret_cast<__half*>(p) = __float2half_rn(float(x)); break;
        case ESA_DTYPE_BF16: *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(float(x)); break;
        case ESA_DTYPE_F32: *reinterpret_cast<float*>(p) = float(x); break;
        default: *reinterpret_cast<double*>(p) = double(x); break;
    }
}

// 8 consecutive elements at p (16-byte aligned), widened to A
template <typename A>
__device__ __forceinline__ void load8(const char* p, int dt, A (&x)[8]) {
    if (dt == ESA_DTYPE_F16 || dt == ESA_DTYPE_BF16) {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f;
            if (dt == ESA_DTYPE_F16)
                f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            else
                f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
            x[2 * i] = A(f.x);
            x[2 * i + 1] = A(f.y);
        }
    } else if (dt == ESA_DTYPE_F32) {
        const float4 a = reinterpret_cast<const float4*>(p)[0];
        const float4 b = reinterpret_cast<const float4*>(p)[1];
        x[0] = A(a.x), x[1] = A(a.y), x[2] = A(a.z), x[3] = A(a.w);
        x[4] = A(b.x), x[5] = A(b.y), x[6] = A(b.z), x[7] = A(b.w);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const double2 d = reinterpret_cast<const double2*>(p)[i];
            x[2 * i] = A(d.x);
            x[2 * i + 1] = A(d.y);
        }
    }
}

// 8 consecutive elements to p (16-byte aligned), rounded to the element type
template <typename A>
__device__ __forceinline__ void store8(char* p, int dt, const A (&x)[8]) {
    if (dt == ESA_DTYPE_F16 || dt == ESA_DTYPE_BF16) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (dt == ESA_DTYPE_F16) {
                const __half2 h = __floats2half2_rn(float(x[2 * i]), float(x[2 * i + 1]));
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            } else {
                const __nv_bfloat162 h = __floats2bfloat162_rn(float(x[2 * i]), float(x[2 * i + 1]));
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if (dt == ESA_DTYPE_F32) {
        reinterpret_cast<float4*>(p)[0] = make_float4(float(x[0]), float(x[1]), float(x[2]), float(x[3]));
        reinterpret_cast<float4*>(p)[1] = make_float4(float(x[4]), float(x[5]), float(x[6]), float(x[7]));
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            reinterpret_cast<double2*>(p)[i] = make_double2(double(x[2 * i]), double(x[2 * i + 1]));
    }
}

// 8 elements of one row at channel c0: vector access, or element by element
// (rows whose length or alignment the 16-byte path cannot take)
template <typename A, bool VECT>
__device__ __forceinline__ void row_load(const char* row, int dt, int es, int64_t c0, int64_t C, A (&x)[8]) {
    if constexpr (VECT) {
        load8(row + c0 * es, dt, x);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = (c0 + i < C) ? load1<A>(row + (c0 + i) * es, dt) : A(0);
    }
}

template <typename A, bool VECT>
__device__ __forceinline__ void row_store(char* row, int dt, int es, int64_t c0, int64_t C, const A (&x)[8]) {
    if constexpr (VECT) {
        store8(row + c0 * es, dt, x);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (c0 + i < C) store1<A>(row + (c0 + i) * es, dt, x[i]);
    }
}

template <typename A>
__device__ __forceinline__ A warp_sum(A x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// x rounded to the element type `dt` (returned widened again)
__device__ __forceinline__ float round_dt(float x, int dt) {
    if (dt == ESA_DTYPE_F16) return __half2float(__float2half_rn(x));
    if (dt == ESA_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(x));
    return x;
}

__device__ __forceinline__ float rsqrt_acc(float x) { return 1.0f / sqrtf(x); }
__device__ __forceinline__ double rsqrt_acc(double x) { return 1.0 / sqrt(x); }

}  // namespace rowops
}  // namespace esa
