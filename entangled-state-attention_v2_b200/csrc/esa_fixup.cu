// esa_fixup.cu -- the two short passes of the single-pass sequence-parallel
// scan: the product of A over a time slice, and the rescan of the head of a
// slice that was scanned from a zero state, once its incoming state is known.
//
// A slice scanned from zero, x^0_t = A_t x^0_{t-1} + B_t with x^0_{-1} = 0,
// differs from the scan from the true incoming state c by a term that only
// decays:  x_t = x^0_t + P_t c,  P_t = A_0 A_1 ... A_t.  So the ranks holding
// consecutive slices scan their slices at once (one pass over A, B, E),
// exchange the per-channel summaries (end state from zero, P_{T-1}), compose
// each rank's incoming state, and then rescan only the head of the slice from
// it: once P_t is exactly zero in the accumulator type every later P_t is
// zero too, and the outputs from the zero state equal those from c (to the
// rounding of the fp32 state).  The head is rescanned from A and B rather
// than corrected from E, so each output is rounded once, from the fp32
// state.  With gates below one P_t reaches zero after a few thousand steps at
// most (A = 0.95: ~1700 steps in fp32), so both passes read a short head of
// the slice; with A = 1 they walk the whole slice (bounded by T).
//
// CTA = 8 warps over 32*V channels of one batch row (V = 2 for 16-bit data
// with an even channel count and 4-byte aligned rows, else 1): per round each
// warp takes 32 consecutive steps (all loads issued before any use) and
// composes them from a zero state in registers; the warps combine their
// chunks through shared memory in warp order, and each warp re-runs its chunk
// from its incoming state to write E.  A round covers 256 steps; the CTA
// stops after the first round whose running product is zero for every
// channel it holds.  No waits on other CTAs.
// Roofline: HBM, but the passes are short; latency per round dominates.
#include <string>

#include "esa_common.cuh"
#include "esa_internal.h"

namespace esa {

namespace {

constexpr int kFixWarps = 8;
constexpr int kFixSteps = 32;  // steps per warp per round

template <typename T, int V>
struct LaneVec;
template <typename T>
struct LaneVec<T, 1> {
    static __device__ __forceinline__ void load(const T* p, typename Elem<T>::acc (&v)[1]) {
        v[0] = Elem<T>::to_acc(*p);
    }
    static __device__ __forceinline__ void store(T* p, const typename Elem<T>::acc (&v)[1]) {
        *p = Elem<T>::from_acc(v[0]);
    }
};
template <typename T>
struct LaneVec<T, 2> {  // two 16-bit channels in one 4-byte word
    static __device__ __forceinline__ void load(const T* p, float (&v)[2]) {
        const unsigned w = *reinterpret_cast<const unsigned*>(p);
        const T* h = reinterpret_cast<const T*>(&w);
        v[0] = Elem<T>::to_acc(h[0]);
        v[1] = Elem<T>::to_acc(h[1]);
    }
    static __device__ __forceinline__ void store(T* p, const float (&v)[2]) {
        T h[2] = {Elem<T>::from_acc(v[0]), Elem<T>::from_acc(v[1])};
        *reinterpret_cast<unsigned*>(p) = *reinterpret_cast<const unsigned*>(h);
    }
};

// FIX = false: prod[b*hd + c] = product of A[b, t, c] over t < T.
// FIX = true:  E[b, t, c] = the scan from x_{-1} = carry[b*hd + c] over the
//              head of the slice, i.e. while the product of A from t = 0 is
//              not yet zero for some channel of the block (E written once,
//              from the fp32 state, as by the scan kernels).
template <typename T, int V, bool FIX>
__global__ void __launch_bounds__(32 * kFixWarps) fixup_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                               T* __restrict__ E,
                                                               const typename Elem<T>::acc* __restrict__ carry,
                                                               typename Elem<T>::acc* __restrict__ prod,
                                                               int64_t T_len, int64_t hd, int64_t groups) {
    using acc = typename Elem<T>::acc;
    __shared__ acc tot_a[kFixWarps][32 * V];
    __shared__ acc tot_b[FIX ? kFixWarps : 1][32 * V];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = blockIdx.x / groups;
    const int64_t c0 = (blockIdx.x - b * groups) * (32 * V) + (int64_t)lane * V;
    const bool live = c0 < hd;  // V = 2 only when hd is even: both channels or none
    const int64_t base = b * T_len * hd + c0;
    // running product of A and (FIX) running state before the round
    acc run[V], xr[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        run[i] = acc(1);
        xr[i] = (FIX && live) ? carry[b * hd + c0 + i] : acc(0);
    }
    for (int64_t t0 = 0; t0 < T_len; t0 += (int64_t)kFixWarps * kFixSteps) {
        const int64_t tw = t0 + (int64_t)warp * kFixSteps;
        acc a[kFixSteps][V], bv[FIX ? kFixSteps : 1][V];
#pragma unroll
        for (int s = 0; s < kFixSteps; ++s) {
            const int64_t t = tw + s;
            if (live && t < T_len) {
                LaneVec<T, V>::load(A + base + t * hd, a[s]);
                if constexpr (FIX) LaneVec<T, V>::load(B + base + t * hd, bv[s]);
            } else {
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    a[s][i] = acc(1);
                    if constexpr (FIX) bv[s][i] = acc(0);
                }
            }
        }
        // the warp's chunk composed from a zero state: product pa, state pb
        acc pa[V], pb[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
            pa[i] = acc(1);
            pb[i] = acc(0);
        }
#pragma unroll
        for (int s = 0; s < kFixSteps; ++s)
#pragma unroll
            for (int i = 0; i < V; ++i) {
                if constexpr (FIX) pb[i] = a[s][i] * pb[i] + bv[s][i];
                pa[i] = pa[i] * a[s][i];
            }
#pragma unroll
        for (int i = 0; i < V; ++i) {
            tot_a[warp][lane * V + i] = pa[i];
            if constexpr (FIX) tot_b[warp][lane * V + i] = pb[i];
        }
        __syncthreads();
        if constexpr (FIX) {
            // state entering this warp's chunk: the running state through the
            // earlier warps' chunks in warp order, then the chunk re-run from it
            acc x[V];
#pragma unroll
            for (int i = 0; i < V; ++i) x[i] = xr[i];
            for (int w = 0; w < warp; ++w)
#pragma unroll
                for (int i = 0; i < V; ++i) x[i] = tot_a[w][lane * V + i] * x[i] + tot_b[w][lane * V + i];
#pragma unroll
            for (int s = 0; s < kFixSteps; ++s) {
                const int64_t t = tw + s;
#pragma unroll
                for (int i = 0; i < V; ++i) x[i] = a[s][i] * x[i] + bv[s][i];
                if (live && t < T_len) LaneVec<T, V>::store(E + base + t * hd, x);
            }
        }
        // running product (and state) after the round, same order on every warp
        bool nonzero = false;
#pragma unroll
        for (int i = 0; i < V; ++i) {
            for (int w = 0; w < kFixWarps; ++w) {
                if constexpr (FIX) xr[i] = tot_a[w][lane * V + i] * xr[i] + tot_b[w][lane * V + i];
                run[i] = run[i] * tot_a[w][lane * V + i];
            }
            nonzero = nonzero || (live && !(run[i] == acc(0)));
        }
        // every warp has read the chunk totals; stop once the product is zero
        // for every channel: later outputs no longer depend on the carry
        if (!__syncthreads_or(nonzero)) break;
    }
    if constexpr (!FIX) {
        if (warp == 0 && live)
#pragma unroll
            for (int i = 0; i < V; ++i) prod[b * hd + c0 + i] = run[i];
    }
}

template <typename F>
int dispatch_fix(int dtype, F&& f) {
    switch (dtype) {
        case ESA_DTYPE_F16: return f(__half{});
        case ESA_DTYPE_BF16: return f(__nv_bfloat16{});
        case ESA_DTYPE_F32: return f(float{});
        case ESA_DTYPE_F64: return f(double{});
        default: return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    }
}

template <bool FIX>
int launch_fix(const void* A, const void* B, void* E, const void* carry, void* prod, int64_t nb, int64_t T,
               int64_t hd, int dtype, cudaStream_t s, const char* what) {
    if (nb < 0 || T < 0 || hd < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(what) + ": negative size");
    if (dtype_size(dtype) == 0)
        return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    if (nb * hd == 0) return ESA_OK;
    if (FIX ? (!A || !B || !E || !carry) : (!A || !prod))
        return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(what) + ": null pointer");
    return dispatch_fix(dtype, [&](auto tag) -> int {
        using T_ = decltype(tag);
        using acc = typename Elem<T_>::acc;
        const bool pair = sizeof(T_) == 2 && hd % 2 == 0 && (reinterpret_cast<uintptr_t>(A) & 3u) == 0 &&
                          (!FIX || ((reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(E)) & 3u) == 0);
        const int width = pair ? 64 : 32;
        const int64_t groups = (hd + width - 1) / width;
        const int64_t blocks = nb * groups;
        if (blocks > 0x7fffffffLL) return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(what) + ": too many channels");
        const dim3 grid((unsigned)blocks), block(32 * kFixWarps);
        const T_* a = static_cast<const T_*>(A);
        const T_* bb = static_cast<const T_*>(B);
        T_* e = static_cast<T_*>(E);
        const acc* cr = static_cast<const acc*>(carry);
        acc* pr = static_cast<acc*>(prod);
        if constexpr (sizeof(T_) == 2) {
            if (pair)
                fixup_kernel<T_, 2, FIX><<<grid, block, 0, s>>>(a, bb, e, cr, pr, T, hd, groups);
            else
                fixup_kernel<T_, 1, FIX><<<grid, block, 0, s>>>(a, bb, e, cr, pr, T, hd, groups);
        } else {
            fixup_kernel<T_, 1, FIX><<<grid, block, 0, s>>>(a, bb, e, cr, pr, T, hd, groups);
        }
        const cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string(what) + " launch: " + cudaGetErrorString(err));
        return ESA_OK;
    });
}

}  // namespace

int scan_prod(const void* A, void* prod, int64_t nb, int64_t T, int64_t hd, int dtype, cudaStream_t s) {
    return launch_fix<false>(A, nullptr, nullptr, nullptr, prod, nb, T, hd, dtype, s, "esa_scan_prod");
}

int scan_fixup(const void* A, const void* B, void* E, const void* carry, int64_t nb, int64_t T, int64_t hd,
               int dtype, cudaStream_t s) {
    return launch_fix<true>(A, B, E, carry, nullptr, nb, T, hd, dtype, s, "esa_scan_fixup");
}

}  // namespace esa
