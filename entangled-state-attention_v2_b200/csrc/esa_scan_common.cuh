// esa_scan_common.cuh -- definitions shared by the scan kernels.
//
// The recurrence E_t = A_t E_{t-1} + B_t runs over independent channels
// (b, c), c < hd, of [nb, T, hd] data (hd contiguous, the reference's
// [B,T,H,D]).  Four kinds of scan share one per-step contract:
//
//   FwdPlain  staged {A, B}                 -> E
//   FwdGated  staged {g, v} (logits)         -> E, with A = gmin + span*sigmoid(g),
//                                               B = (1 - A) tanh(v) computed in-kernel
//   RevPlain  staged {A, E_{t-1}, dE}        -> dA, dB
//   RevGated  staged {g, v, E_{t-1}, dE}     -> d g, d v  (gate chain rule fused)
//
// Every kind is an affine scan x_t = a_t x_{t-1} + b_t (forward in t) or
// x_t = a_t x_{t+1} + b_t (reverse, with x = H = A*G, a = A_t, b = A_t dE_t).
// Phase 1 of a kernel produces (a_t, b_t) per step ("step_coef"); phase 3
// re-runs the steps from the exact incoming state and writes the outputs
// ("step_apply").
#pragma once

#include <type_traits>

#include <string>

#include "esa_common.cuh"
#include "esa_internal.h"

namespace esa {

// Calls f(T{}) with T the element type of dtype code `dtype`.
template <typename F>
int dispatch_dtype(int dtype, F&& f) {
    switch (dtype) {
        case ESA_DTYPE_F16: return f(__half{});
        case ESA_DTYPE_BF16: return f(__nv_bfloat16{});
        case ESA_DTYPE_F32: return f(float{});
        case ESA_DTYPE_F64: return f(double{});
        default: return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    }
}

template <typename T, int N>
struct alignas(sizeof(T) * N) VecN {
    T v[N];
};

template <typename T>
__device__ __forceinline__ float round_to(float x) {
    return Elem<T>::to_acc(Elem<T>::from_acc(x));
}
template <typename T>
__device__ __forceinline__ double round_to(double x) {
    return static_cast<double>(Elem<T>::from_acc(static_cast<typename Elem<T>::acc>(x)));
}

// VN > 0 overrides the channels per thread vector (the narrow strip scan's
// two-channel lanes); 0 keeps one 16-byte vector of the widest type.
template <Kind K, typename Tin, typename Te, int VN = 0>
struct Policy {
    static constexpr bool REV = (K == Kind::RevPlain || K == Kind::RevGated);
    static constexpr bool GATED = (K == Kind::FwdGated || K == Kind::RevGated);
    static constexpr int NIN = (K == Kind::RevGated) ? 4 : (K == Kind::RevPlain ? 3 : 2);
    using acc = typename std::conditional<(sizeof(Tin) == 8 || sizeof(Te) == 8), double, float>::type;
    static constexpr int WIDE = (sizeof(Tin) > sizeof(Te)) ? sizeof(Tin) : sizeof(Te);
    static constexpr int VEC = VN > 0 ? VN : 16 / WIDE;  // channels per thread vector
    // element size of staged array i
    static __host__ __device__ constexpr int es(int i) {
        return (K == Kind::RevGated) ? (i < 2 ? (int)sizeof(Tin) : (int)sizeof(Te))
               : (K == Kind::RevPlain) ? (int)sizeof(Te)
                                       : (int)sizeof(Tin);
    }
    // staged array i holds row t + shift(i) at step t (E_{t-1} for the reverse scans)
    static __host__ __device__ constexpr int shift(int i) {
        return (K == Kind::RevPlain && i == 1) || (K == Kind::RevGated && i == 2) ? -1 : 0;
    }
    // element size of the outputs (E, dA/dB: Te; d gate/d value: Tin)
    static constexpr int OES = (K == Kind::RevGated) ? (int)sizeof(Tin) : (int)sizeof(Te);
    // phase-1 values kept in registers for phase 3 (S rows x VEC channels):
    // forward: (A, B); reverse: (A or sigmoid(g), dE).  Phase 3 then needs no
    // shared-memory reload or conversion of them.
    template <int S>
    struct Cache {
        acc c0[S][VEC];
        acc c1[S][VEC];
    };
};

// ---------------------------------------------------------------------------
// Lane-vector arithmetic, one scalar IEEE round-to-nearest instruction per
// channel.  (Blackwell's packed FP32x2 forms measured slower in these kernels:
// their register-pair operands cost more moves than the pairing saves.)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_rn(double a, double b, double c) { return __fma_rn(a, b, c); }
// d = a * b + c
template <typename A, int N>
__device__ __forceinline__ void vfma(A (&d)[N], const A (&a)[N], const A (&b)[N], const A (&c)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = fma_rn(a[i], b[i], c[i]);
}
// d = a * b
template <typename A, int N>
__device__ __forceinline__ void vmul(A (&d)[N], const A (&a)[N], const A (&b)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = a[i] * b[i];
}
// d = a + b
template <typename A, int N>
__device__ __forceinline__ void vadd(A (&d)[N], const A (&a)[N], const A (&b)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) d[i] = a[i] + b[i];
}
// Compose the affine pair (qa, qb) (earlier) with (pa, pb) (later):
// (pa, pb) <- (pa*qa, pa*qb + pb).
template <typename A, int N>
__device__ __forceinline__ void vcompose(A (&pa)[N], A (&pb)[N], const A (&qa)[N], const A (&qb)[N]) {
    vfma(pb, pa, qb, pb);
    vmul(pa, pa, qa);
}

// Load N elements of T from shared memory and widen them to the accumulator
// type (16-bit types in pairs: one conversion per channel pair).
template <typename T, int N, typename A>
__device__ __forceinline__ void load_smem(const char* p, A (&out)[N]) {
    if constexpr (std::is_same<T, __half>::value && std::is_same<A, float>::value && N % 2 == 0) {
        const VecN<__half2, N / 2> v = *reinterpret_cast<const VecN<__half2, N / 2>*>(p);
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const float2 f = __half22float2(v.v[i]);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value && std::is_same<A, float>::value && N % 2 == 0) {
        const VecN<__nv_bfloat162, N / 2> v = *reinterpret_cast<const VecN<__nv_bfloat162, N / 2>*>(p);
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const float2 f = __bfloat1622float2(v.v[i]);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    } else {
        VecN<T, N> v = *reinterpret_cast<const VecN<T, N>*>(p);
#pragma unroll
        for (int i = 0; i < N; ++i) out[i] = static_cast<A>(Elem<T>::to_acc(v.v[i]));
    }
}

// Vector load / store of N accumulators (one thread's channels) in shared
// memory: a warp touches one contiguous span, so no bank conflicts beyond the
// span's width.
template <typename A, int N>
__device__ __forceinline__ void lds_vec(const A* p, A (&out)[N]) {
    const VecN<A, N> v = *reinterpret_cast<const VecN<A, N>*>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = v.v[i];
}
template <typename A, int N>
__device__ __forceinline__ void sts_vec(A* p, const A (&in)[N]) {
    VecN<A, N> v;
#pragma unroll
    for (int i = 0; i < N; ++i) v.v[i] = in[i];
    *reinterpret_cast<VecN<A, N>*>(p) = v;
}

// One vector store of W 32-bit words (W = 1, 2, 4): a single st.global.v4 /
// v2 / b32 (a struct copy of __half2 elements would be split per element).
template <int W>
__device__ __forceinline__ void store_words(char* p, const uint32_t (&w)[W]) {
    if constexpr (W == 4) {
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if constexpr (W == 2) {
        *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    } else {
#pragma unroll
        for (int i = 0; i < W; ++i) reinterpret_cast<uint32_t*>(p)[i] = w[i];
    }
}

template <typename T, int N, typename A>
__device__ __forceinline__ void store_global(char* p, const A (&in)[N]) {
    if constexpr (std::is_same<T, __half>::value && std::is_same<A, float>::value && N % 2 == 0) {
        uint32_t w[N / 2];
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const __half2 h = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        store_words<N / 2>(p, w);
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value && std::is_same<A, float>::value && N % 2 == 0) {
        uint32_t w[N / 2];
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        store_words<N / 2>(p, w);
    } else {
        VecN<T, N> v;
#pragma unroll
        for (int i = 0; i < N; ++i) v.v[i] = Elem<T>::from_acc(static_cast<typename Elem<T>::acc>(in[i]));
        *reinterpret_cast<VecN<T, N>*>(p) = v;
    }
}

// Channel pairs of 16-bit data: two elements widened with one conversion,
// and a float pair rounded to the 16-bit type and widened back (the value
// A.to(scan_dtype) takes) with one packing conversion.
template <typename T>
__device__ __forceinline__ float2 pair_load(const char* p) {
    if constexpr (std::is_same<T, __half>::value)
        return __half22float2(*reinterpret_cast<const __half2*>(p));
    else
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <typename T>
__device__ __forceinline__ float2 pair_round(float x, float y) {
    if constexpr (std::is_same<T, __half>::value)
        return __half22float2(__floats2half2_rn(x, y));
    else
        return __bfloat1622float2(__floats2bfloat162_rn(x, y));
}
template <typename T>
constexpr bool is_16bit = std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value;

// Per-step coefficients (a, b) of step row `rows` (phase 1).  `rows[i]` points
// at this thread's first channel in staged array i.
template <Kind K, typename Tin, typename Te, int S, typename P = Policy<K, Tin, Te>>
__device__ __forceinline__ void step_coef(const char* const (&rows)[4], const KArgs& prm,
                                          typename P::acc (&a)[P::VEC],
                                          typename P::acc (&b)[P::VEC],
                                          typename P::template Cache<S>& cache, int s) {
    using acc = typename P::acc;
    constexpr int VEC = P::VEC;
    constexpr bool FASTG = sizeof(Tin) == 2 && sizeof(Te) == 2;  // 16-bit gates (gate_sigmoid)
    constexpr bool PAIR16 = is_16bit<Tin> && std::is_same<Tin, Te>::value && VEC % 2 == 0;
    if constexpr (K == Kind::FwdPlain || K == Kind::FwdSummary) {
        load_smem<Tin, VEC>(rows[0], a);
        load_smem<Tin, VEC>(rows[1], b);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            cache.c0[s][i] = a[i];
            cache.c1[s][i] = b[i];
        }
    } else if constexpr (K == Kind::FwdGated && PAIR16) {
        // 16-bit logits and scan: channel pairs, B = (1 - A) tanh(v) as
        // fma(-A, t, t) (1 - A is exact for A in [0.5, 1])
        const float hs = 0.5f * float(prm.span), c = float(prm.gmin) + hs;
#pragma unroll
        for (int i = 0; i < VEC; i += 2) {
            const float2 g = pair_load<Tin>(rows[0] + i * 2);
            const float2 v = pair_load<Tin>(rows[1] + i * 2);
            float A0 = gate_a_fast(g.x, c, hs), A1 = gate_a_fast(g.y, c, hs);
            const float t0 = tanh_fast(v.x), t1 = tanh_fast(v.y);
            float B0 = fmaf(-A0, t0, t0), B1 = fmaf(-A1, t1, t1);
            if (prm.round_ab) {
                const float2 ra = pair_round<Te>(A0, A1), rb = pair_round<Te>(B0, B1);
                A0 = ra.x;
                A1 = ra.y;
                B0 = rb.x;
                B1 = rb.y;
            }
            a[i] = A0;
            a[i + 1] = A1;
            b[i] = B0;
            b[i + 1] = B1;
            cache.c0[s][i] = A0;
            cache.c0[s][i + 1] = A1;
            cache.c1[s][i] = B0;
            cache.c1[s][i + 1] = B1;
        }
    } else if constexpr (K == Kind::FwdGated) {
        acc g[VEC], v[VEC];
        load_smem<Tin, VEC>(rows[0], g);
        load_smem<Tin, VEC>(rows[1], v);
        const acc lo = acc(prm.gmin), span = acc(prm.span);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            acc A;
            if constexpr (FASTG)
                A = gate_a_fast(g[i], float(prm.gmin + 0.5 * prm.span), float(0.5 * prm.span));
            else
                A = lo + span * gate_sigmoid<FASTG>(g[i]);
            acc B = (acc(1) - A) * gate_tanh<FASTG>(v[i]);
            if (prm.round_ab) {
                A = round_to<Te>(A);
                B = round_to<Te>(B);
            }
            a[i] = A;
            b[i] = B;
            cache.c0[s][i] = A;
            cache.c1[s][i] = B;
        }
    } else if constexpr (K == Kind::RevPlain) {
        acc d[VEC];
        load_smem<Te, VEC>(rows[0], a);
        load_smem<Te, VEC>(rows[2], d);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            b[i] = a[i] * d[i];
            cache.c0[s][i] = a[i];
            cache.c1[s][i] = d[i];
        }
    } else if constexpr (PAIR16) {  // RevGated, 16-bit pairs
        const float lo = float(prm.gmin), span = float(prm.span);
#pragma unroll
        for (int i = 0; i < VEC; i += 2) {
            const float2 g = pair_load<Tin>(rows[0] + i * 2);
            const float2 d = pair_load<Te>(rows[3] + i * 2);
            const float s0 = sigmoid_fast(g.x), s1 = sigmoid_fast(g.y);
            float A0 = fmaf(span, s0, lo), A1 = fmaf(span, s1, lo);
            if (prm.round_ab) {
                const float2 ra = pair_round<Te>(A0, A1);
                A0 = ra.x;
                A1 = ra.y;
            }
            cache.c0[s][i] = s0;
            cache.c0[s][i + 1] = s1;
            cache.c1[s][i] = d.x;
            cache.c1[s][i + 1] = d.y;
            a[i] = A0;
            a[i + 1] = A1;
            b[i] = A0 * d.x;
            b[i + 1] = A1 * d.y;
        }
    } else {  // RevGated
        acc g[VEC], d[VEC];
        load_smem<Tin, VEC>(rows[0], g);
        load_smem<Te, VEC>(rows[3], d);
        const acc lo = acc(prm.gmin), span = acc(prm.span);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const acc sg = gate_sigmoid<FASTG>(g[i]);
            acc A = lo + span * sg;
            if (prm.round_ab) A = round_to<Te>(A);
            cache.c0[s][i] = sg;
            cache.c1[s][i] = d[i];
            a[i] = A;
            b[i] = A * d[i];
        }
    }
}

// Phase-3 step: advance the state `e` over step t and write this step's
// outputs for VEC channels starting at global channel `gc` (when `valid`).
// Forward: e = E_{t-1} in, E_t out.  Reverse: e = H_{t+1} in, H_t out.
// MAY_T0 = false promises t > 0 (the reverse kinds then read E_{t-1} from
// shared memory with no branch on t).
template <Kind K, typename Tin, typename Te, int S, typename P = Policy<K, Tin, Te>, bool MAY_T0 = true>
__device__ __forceinline__ void step_apply(const char* const (&rows)[4], const KArgs& prm,
                                           int64_t b, int64_t t, int64_t gc, bool valid,
                                           typename P::acc (&e)[P::VEC],
                                           typename P::template Cache<S>& cache, int s, char* o0,
                                           char* o1) {
    using acc = typename P::acc;
    constexpr int VEC = P::VEC;
    constexpr bool FASTG = sizeof(Tin) == 2 && sizeof(Te) == 2;  // 16-bit gates (gate_sigmoid)
    constexpr bool PAIR16 = is_16bit<Tin> && std::is_same<Tin, Te>::value && VEC % 2 == 0;
    if constexpr (K == Kind::FwdPlain) {
        vfma(e, cache.c0[s], e, cache.c1[s]);
        if (valid)
            store_global<Te, VEC>(o0, e);
    } else if constexpr (K == Kind::FwdGated) {
        vfma(e, cache.c0[s], e, cache.c1[s]);
        if (valid)
            store_global<Te, VEC>(o0, e);
    } else {
        acc ep[VEC], d[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) d[i] = cache.c1[s][i];
        if (!MAY_T0 || t > 0) {
            load_smem<Te, VEC>(K == Kind::RevPlain ? rows[1] : rows[2], ep);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) ep[i] = acc(0);
            if (prm.e0 != nullptr && valid) {
                const acc* e0 = static_cast<const acc*>(prm.e0) + b * prm.hd + gc;
#pragma unroll
                for (int i = 0; i < VEC; ++i) ep[i] = e0[i];
            }
        }
        if constexpr (K == Kind::RevPlain) {
            acc ga[VEC];
            vadd(d, d, e);            // G_t = dE_t + H_{t+1}  (= dB)
            vmul(ga, d, ep);          // dA = G_t E_{t-1}
            vmul(e, cache.c0[s], d);  // H_t = A_t G_t
            if (valid) {
                store_global<Te, VEC>(o0, ga);
                store_global<Te, VEC>(o1, d);
            }
        } else if constexpr (PAIR16) {
            acc dg[VEC], dv[VEC];
            const float lo = float(prm.gmin), span = float(prm.span);
#pragma unroll
            for (int i = 0; i < VEC; i += 2) {
                const float2 v = pair_load<Tin>(rows[1] + i * 2);
                const float V[2] = {tanh_fast(v.x), tanh_fast(v.y)};
                float A[2], Ar[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) A[u] = fmaf(span, cache.c0[s][i + u], lo);
                if (prm.round_ab) {
                    const float2 r = pair_round<Te>(A[0], A[1]);
                    Ar[0] = r.x;
                    Ar[1] = r.y;
                } else {
                    Ar[0] = A[0];
                    Ar[1] = A[1];
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const float sg = cache.c0[s][i + u];
                    const float g = d[i + u] + e[i + u];
                    const float dA = g * ep[i + u];
                    dg[i + u] = fmaf(-g, V[u], dA) * (span * sg * (1.0f - sg));
                    dv[i + u] = g * (1.0f - A[u]) * fmaf(-V[u], V[u], 1.0f);
                    e[i + u] = Ar[u] * g;
                }
            }
            if (valid) {
                store_global<Tin, VEC>(o0, dg);
                store_global<Tin, VEC>(o1, dv);
            }
        } else {
            acc v[VEC], dg[VEC], dv[VEC];
            load_smem<Tin, VEC>(rows[1], v);
            const acc lo = acc(prm.gmin), span = acc(prm.span);
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                const acc sg = cache.c0[s][i];
                const acc A = lo + span * sg;
                const acc Ar = prm.round_ab ? round_to<Te>(A) : A;
                const acc V = gate_tanh<FASTG>(v[i]);
                const acc g = d[i] + e[i];
                const acc dA = g * ep[i];
                dg[i] = (dA - g * V) * span * sg * (acc(1) - sg);
                dv[i] = g * (acc(1) - A) * (acc(1) - V * V);
                e[i] = Ar * g;
            }
            if (valid) {
                store_global<Tin, VEC>(o0, dg);
                store_global<Tin, VEC>(o1, dv);
            }
        }
    }
}

// Bounded wait on an mbarrier phase.  Returns false (and raises `status`) if
// the phase did not complete within the wait budget.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, unsigned* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned it = 0; it < kWaitMaxIters; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitBudgetNs) break;
    }
    atomicOr(status, ESA_STATUS_COPY_TIMEOUT);
    return false;
}

}  // namespace esa
