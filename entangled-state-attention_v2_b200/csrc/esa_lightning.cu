// esa_lightning.cu -- the fused ESA-Lightning one-token decode step on sm_100a.
//
// One CTA per batch row.  Per channel c of the row (C = H*D channels):
//   A  = gmin + (gmax - gmin) * sigmoid(g_c),   B = (1 - A) * tanh(v_c)
//   S' = A * S_c + B                       (rounded to the state dtype)
//   z_c = sigmoid(q_c) * S'_c * rsqrt(mean_c(S'^2) + eps)
// The RMS runs over all C channels of the row (the reference normalises across
// heads), so the whole row lives in one CTA and the reduction is a CTA
// reduction.  Arithmetic in fp32 (fp64 for fp64 states).  Replaces the ~10
// eager launches of esa/generation.py:443-458 with one; the qgv GEMV before it
// and out_proj after it stay on cuBLAS.
#include <string>

#include "esa_common.cuh"
#include "esa_internal.h"

namespace esa {

template <typename Tq, typename Ts, typename Tz>
__global__ void __launch_bounds__(256) lightning_step_kernel(const Tq* __restrict__ qgv, int64_t qrs,
                                                             const Ts* state, Ts* new_state,
                                                             Tz* __restrict__ z, int64_t C,
                                                             double gmin, double gspan, double eps) {
    using acc = typename std::conditional<(sizeof(Ts) == 8 || sizeof(Tq) == 8), double, float>::type;
    __shared__ acc red[32];
    const int64_t b = blockIdx.x;
    const Tq* q = qgv + b * qrs;
    const Tq* g = q + C;
    const Tq* v = q + 2 * C;
    const Ts* s_in = state + b * C;
    Ts* s_out = new_state + b * C;
    Tz* zr = z + b * C;
    const acc lo = acc(gmin), span = acc(gspan);

    acc ss = acc(0);
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
        const acc A = lo + span * sigmoid_(static_cast<acc>(Elem<Tq>::to_acc(g[c])));
        const acc B = (acc(1) - A) * tanh_(static_cast<acc>(Elem<Tq>::to_acc(v[c])));
        // the reference casts A and B to the state dtype before the update
        const acc Ar = static_cast<acc>(Elem<Ts>::to_acc(Elem<Ts>::from_acc(static_cast<typename Elem<Ts>::acc>(A))));
        const acc Br = static_cast<acc>(Elem<Ts>::to_acc(Elem<Ts>::from_acc(static_cast<typename Elem<Ts>::acc>(B))));
        const acc sp = Ar * static_cast<acc>(Elem<Ts>::to_acc(s_in[c])) + Br;
        const Ts spr = Elem<Ts>::from_acc(static_cast<typename Elem<Ts>::acc>(sp));
        s_out[c] = spr;  // s_out may alias s_in: each element is read then written by this thread
        const acc e = static_cast<acc>(Elem<Ts>::to_acc(spr));
        ss += e * e;
    }
    // CTA reduction of the sum of squares
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        acc x = lane < nw ? red[lane] : acc(0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane == 0) red[0] = x;
    }
    __syncthreads();
    const acc r = acc(1) / sqrt(red[0] / acc(C) + acc(eps));
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
        const acc e = static_cast<acc>(Elem<Ts>::to_acc(s_out[c]));
        const acc sq = sigmoid_(static_cast<acc>(Elem<Tq>::to_acc(q[c])));
        zr[c] = Elem<Tz>::from_acc(static_cast<typename Elem<Tz>::acc>(sq * e * r));
    }
}

template <typename F>
static int dispatch_t(int dtype, F&& f) {
    switch (dtype) {
        case ESA_DTYPE_F16: return f(__half{});
        case ESA_DTYPE_BF16: return f(__nv_bfloat16{});
        case ESA_DTYPE_F32: return f(float{});
        case ESA_DTYPE_F64: return f(double{});
        default: return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    }
}

int lightning_step(const void* qgv, int64_t qrs, int qdt, const void* state, void* new_state,
                   int sdt, void* z, int zdt, int64_t nb, int64_t C, double gmin, double gmax,
                   double eps, cudaStream_t s) {
    if (nb < 0 || C <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "lightning step needs nb >= 0 and C > 0");
    if (qrs < 3 * C) return set_error(ESA_ERR_INVALID_ARGUMENT, "qgv row stride smaller than 3*C");
    if (nb == 0) return ESA_OK;
    if (!qgv || !state || !new_state || !z) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (nb > 0x7fffffff) return set_error(ESA_ERR_INVALID_ARGUMENT, "too many rows");
    return dispatch_t(qdt, [&](auto qt) -> int {
        using Tq = decltype(qt);
        return dispatch_t(sdt, [&](auto st) -> int {
            using Ts = decltype(st);
            return dispatch_t(zdt, [&](auto zt) -> int {
                using Tz = decltype(zt);
                int threads = 256;
                if (C < 256) threads = (int)((C + 31) / 32 * 32);
                lightning_step_kernel<Tq, Ts, Tz><<<(unsigned)nb, threads, 0, s>>>(
                    static_cast<const Tq*>(qgv), qrs, static_cast<const Ts*>(state),
                    static_cast<Ts*>(new_state), static_cast<Tz*>(z), C, gmin, gmax - gmin, eps);
                cudaError_t e = cudaGetLastError();
                if (e != cudaSuccess)
                    return set_error(ESA_ERR_CUDA, std::string("lightning launch: ") + cudaGetErrorString(e));
                return ESA_OK;
            });
        });
    });
}

}  // namespace esa
