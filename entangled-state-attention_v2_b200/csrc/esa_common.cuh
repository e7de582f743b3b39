// esa_common.cuh -- shared device helpers for the ESA sm_100a kernels.
//
// Element types, 16-byte vector conversion, the PTX wrappers the scan kernels
// need (mbarrier, bulk async copy global->shared, acquire/release flags,
// %globaltimer), bounded waits and the device error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/esa_b200.h"

namespace esa {

// Wall-clock budget of every spin-wait in these kernels: one second.
constexpr unsigned long long kWaitBudgetNs = 1000000000ull;
// Iteration cap as a backstop in case %globaltimer does not advance.
constexpr unsigned int kWaitMaxIters = 1u << 26;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// Element types and 16-byte vectors.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<__half> {
    using acc = float;
    static __device__ __forceinline__ float to_acc(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_acc(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
    using acc = float;
    static __device__ __forceinline__ float to_acc(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_acc(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<float> {
    using acc = float;
    static __device__ __forceinline__ float to_acc(float x) { return x; }
    static __device__ __forceinline__ float from_acc(float x) { return x; }
};
template <> struct Elem<double> {
    using acc = double;
    static __device__ __forceinline__ double to_acc(double x) { return x; }
    static __device__ __forceinline__ double from_acc(double x) { return x; }
};

// VEC elements of T packed in 16 bytes.
template <typename T> struct alignas(16) Vec16 {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

template <typename T, typename A>
__device__ __forceinline__ void unpack(const Vec16<T>& p, A (&out)[Vec16<T>::N]) {
#pragma unroll
    for (int i = 0; i < Vec16<T>::N; ++i) out[i] = static_cast<A>(Elem<T>::to_acc(p.v[i]));
}

template <typename T, typename A>
__device__ __forceinline__ Vec16<T> pack(const A (&in)[Vec16<T>::N]) {
    Vec16<T> p;
#pragma unroll
    for (int i = 0; i < Vec16<T>::N; ++i) p.v[i] = Elem<T>::from_acc(in[i]);
    return p;
}

__device__ __forceinline__ uint4 ld_shared_v4(const void* p) {
    uint4 r;
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}

// Streaming 16-byte global store (E is written once and not re-read here).
__device__ __forceinline__ void st_global_cs_v4(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ uint4 ld_global_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// ---------------------------------------------------------------------------
// Flags for the decoupled lookback: release store / acquire load at gpu scope.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (the TMA engine's non-tensor form).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" :: "r"(a) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 :: "r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" :: "r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(a), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}

// Non-blocking test of an mbarrier phase (no suspension).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(a), "r"(parity) : "memory");
    return ok != 0;
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing on `bar`.  L2 evict-first:
// every input byte is read exactly once.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, unsigned bytes,
                                         uint64_t* bar, uint64_t policy) {
    uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;"
        :: "r"(d), "l"(gsrc), "r"(bytes), "r"(b), "l"(policy) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------------------
// Gate nonlinearity, from the definitions sigmoid(x) = 1 / (1 + e^-x) and
// tanh(x) = 2 sigmoid(2x) - 1, evaluated with expf / tanhf of the CUDA math
// library (accuracy tested against torch in tests/test_gpu_*.py).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ double sigmoid_(double x) { return 1.0 / (1.0 + exp(-x)); }
__device__ __forceinline__ float sigmoid_(float x) { return sigmoidf_(x); }
__device__ __forceinline__ float tanh_(float x) { return tanhf(x); }
__device__ __forceinline__ double tanh_(double x) { return tanh(x); }

// Gate nonlinearity of 16-bit logits feeding a 16-bit scan, on the hardware
// approximations of PTX: sigmoid(x) = 1 / (1 + 2^(-x log2 e)) with
// ex2.approx.ftz.f32 and rcp.approx.ftz.f32 (relative errors near 2^-22), and
// tanh.approx.f32 (relative error below 2^-10.98).  Their errors sit at or
// below the half-precision rounding (2^-11 relative) that the logits carry in
// and that A, B and E get on the way out; the exact forms above cost the
// fused gated scans a third of their speed (the [16,2048,768] fp16 forward:
// 115.7 vs 75.4 us).  Wider logits or scans keep the exact forms.
__device__ __forceinline__ float sigmoid_fast(float x) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return r;
}
__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// The forward gate A = lo + span sigmoid(x) of 16-bit scans, from
// sigmoid(x) = (1 + tanh(x / 2)) / 2: one tanh.approx instead of ex2 + rcp.
// Its error (under 2^-11 of span / 2) moves about 2 % of the fp16-rounded A
// by one unit in the last place; the scan output's relative error grows from
// 2.1e-4 (its own rounding) to 3.4e-4 on [4, 2048, 256] random logits.  The
// reverse scans keep sigmoid_fast, whose derivative s (1 - s) needs the
// relative accuracy tanh.approx lacks near saturation.
__device__ __forceinline__ float gate_a_fast(float x, float lo_half_span, float half_span) {
    return fmaf(half_span, tanh_fast(0.5f * x), lo_half_span);
}
template <bool FAST, typename A>
__device__ __forceinline__ A gate_sigmoid(A x) {
    if constexpr (FAST && std::is_same<A, float>::value)
        return sigmoid_fast(x);
    else
        return sigmoid_(x);
}
template <bool FAST, typename A>
__device__ __forceinline__ A gate_tanh(A x) {
    if constexpr (FAST && std::is_same<A, float>::value)
        return tanh_fast(x);
    else
        return tanh_(x);
}

}  // namespace esa
