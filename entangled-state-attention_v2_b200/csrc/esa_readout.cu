// esa_readout.cu -- the ESA layer readout, fused: forward and backward.
//
//   n = E * rsqrt(mean_C(E^2) + eps),   y = sigmoid(q) * n
//
// (the reference's `sigmoid(q) * E * rsqrt(E.pow(2).mean(-1) + eps)`,
// esa/backends/thunder.py:304-311, esa/generation.py:270-293), one warp per
// row of C channels: a pass for the sum of squares (warp-shuffle reduction),
// a pass for the outputs; the row's rsqrt is kept for the backward.  The
// backward of the same row:
//
//   dq = dy * n * s * (1 - s),   dn = dy * s,   s = sigmoid(q)
//   dE = r * (dn - n * mean_C(dn * n)),   r = rsqrt(mean_C(E^2) + eps)
//
// Arithmetic in fp32 (fp64 when any operand is fp64) with one rounding per
// output.  q, dq may be row-strided views (the q slice of the qgv projection
// and of its gradient, row stride 3C); every operand has its own element type.
// Roofline: HBM -- forward reads q and E and writes y (plus 4 bytes a row);
// backward reads dy, q, E and writes dq and dE.
#include <initializer_list>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"
#include "esa_rowops.cuh"

namespace esa {
namespace {

using namespace rowops;

// One operand: base, row stride (elements), element type code and size.
struct Opnd {
    const char* p;
    int64_t rs;
    int dt, es;
};
struct MutOpnd {
    char* p;
    int64_t rs;
    int dt, es;
};

struct ReadoutArgs {
    Opnd q, E, dy;
    MutOpnd y, dq, dE;
    void* rstd;  // acc [rows]
    int64_t rows, C;
    double eps;
};

constexpr int kReadoutWarps = 8;

// FIX >= 0: every operand of the call has the 16-bit dtype code FIX (the
// autocast training layer), so loads and stores resolve at compile time and
// the sigmoid takes its fast 16-bit form (gate_sigmoid); FIX < 0: per-operand
// dtypes read at run time, exact sigmoid.
template <int FIX>
__device__ __forceinline__ int dt_of(int dt) { return FIX >= 0 ? FIX : dt; }
template <int FIX>
__device__ __forceinline__ int es_of(int es) { return FIX >= 0 ? 2 : es; }

template <typename A, bool VECT, int FIX>
__global__ void __launch_bounds__(32 * kReadoutWarps) readout_fwd_kernel(const ReadoutArgs a) {
    constexpr bool FAST = FIX >= 0;
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kReadoutWarps;
    const A inv_c = A(1) / A(a.C), eps = A(a.eps);
    const int edt = dt_of<FIX>(a.E.dt), qdt = dt_of<FIX>(a.q.dt), ydt = dt_of<FIX>(a.y.dt);
    const int ees = es_of<FIX>(a.E.es), qes = es_of<FIX>(a.q.es), yes = es_of<FIX>(a.y.es);
    for (int64_t row = (int64_t)blockIdx.x * kReadoutWarps + (threadIdx.x >> 5); row < a.rows; row += nw) {
        const char* er = a.E.p + row * a.E.rs * ees;
        const char* qr = a.q.p + row * a.q.rs * qes;
        char* yr = a.y.p + row * a.y.rs * yes;
        A ss = A(0);
        for (int64_t c0 = lane * 8; c0 < a.C; c0 += 256) {
            A e[8];
            row_load<A, VECT>(er, edt, ees, c0, a.C, e);
#pragma unroll
            for (int i = 0; i < 8; ++i) ss = fma_rn(e[i], e[i], ss);
        }
        const A r = rsqrt_acc(warp_sum(ss) * inv_c + eps);
        for (int64_t c0 = lane * 8; c0 < a.C; c0 += 256) {
            A e[8], q[8], y[8];
            row_load<A, VECT>(er, edt, ees, c0, a.C, e);
            row_load<A, VECT>(qr, qdt, qes, c0, a.C, q);
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = gate_sigmoid<FAST>(q[i]) * (e[i] * r);
            row_store<A, VECT>(yr, ydt, yes, c0, a.C, y);
        }
        if (lane == 0) static_cast<A*>(a.rstd)[row] = r;
    }
}

template <typename A, bool VECT, int FIX>
__global__ void __launch_bounds__(32 * kReadoutWarps) readout_bwd_kernel(const ReadoutArgs a) {
    constexpr bool FAST = FIX >= 0;
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kReadoutWarps;
    const A inv_c = A(1) / A(a.C);
    const int edt = dt_of<FIX>(a.E.dt), qdt = dt_of<FIX>(a.q.dt), dydt = dt_of<FIX>(a.dy.dt);
    const int dqdt = dt_of<FIX>(a.dq.dt), dedt = dt_of<FIX>(a.dE.dt);
    const int ees = es_of<FIX>(a.E.es), qes = es_of<FIX>(a.q.es), dyes = es_of<FIX>(a.dy.es);
    const int dqes = es_of<FIX>(a.dq.es), dees = es_of<FIX>(a.dE.es);
    for (int64_t row = (int64_t)blockIdx.x * kReadoutWarps + (threadIdx.x >> 5); row < a.rows; row += nw) {
        const char* er = a.E.p + row * a.E.rs * ees;
        const char* qr = a.q.p + row * a.q.rs * qes;
        const char* dyr = a.dy.p + row * a.dy.rs * dyes;
        char* dqr = a.dq.p + row * a.dq.rs * dqes;
        char* der = a.dE.p + row * a.dE.rs * dees;
        const A r = static_cast<const A*>(a.rstd)[row];
        // sum over the row of dn * n, dn = dy * s
        A dot = A(0);
        for (int64_t c0 = lane * 8; c0 < a.C; c0 += 256) {
            A e[8], q[8], dy[8];
            row_load<A, VECT>(er, edt, ees, c0, a.C, e);
            row_load<A, VECT>(qr, qdt, qes, c0, a.C, q);
            row_load<A, VECT>(dyr, dydt, dyes, c0, a.C, dy);
#pragma unroll
            for (int i = 0; i < 8; ++i) dot = fma_rn(dy[i] * gate_sigmoid<FAST>(q[i]), e[i] * r, dot);
        }
        const A mdot = warp_sum(dot) * inv_c;
        for (int64_t c0 = lane * 8; c0 < a.C; c0 += 256) {
            A e[8], q[8], dy[8], dq[8], de[8];
            row_load<A, VECT>(er, edt, ees, c0, a.C, e);
            row_load<A, VECT>(qr, qdt, qes, c0, a.C, q);
            row_load<A, VECT>(dyr, dydt, dyes, c0, a.C, dy);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const A s = gate_sigmoid<FAST>(q[i]);
                const A n = e[i] * r;
                const A dn = dy[i] * s;
                dq[i] = dy[i] * n * s * (A(1) - s);
                de[i] = r * (dn - n * mdot);
            }
            row_store<A, VECT>(dqr, dqdt, dqes, c0, a.C, dq);
            row_store<A, VECT>(der, dedt, dees, c0, a.C, de);
        }
    }
}

bool vec_ok(const void* p, int64_t rs, int es) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (rs * es) % 16 == 0;
}

// `fix`: the common 16-bit dtype code of every operand, or -1.
template <template <typename, bool, int> class Launch>
int readout_launch(const ReadoutArgs& a, bool wide, bool vect, int fix, cudaStream_t s) {
    const int64_t blocks_needed = (a.rows + kReadoutWarps - 1) / kReadoutWarps;
    const int grid = (int)(blocks_needed < 148 * 16 ? blocks_needed : 148 * 16);
    if (wide)
        vect ? Launch<double, true, -1>::go(a, grid, s) : Launch<double, false, -1>::go(a, grid, s);
    else if (fix == ESA_DTYPE_F16)
        vect ? Launch<float, true, ESA_DTYPE_F16>::go(a, grid, s) : Launch<float, false, ESA_DTYPE_F16>::go(a, grid, s);
    else if (fix == ESA_DTYPE_BF16)
        vect ? Launch<float, true, ESA_DTYPE_BF16>::go(a, grid, s)
             : Launch<float, false, ESA_DTYPE_BF16>::go(a, grid, s);
    else
        vect ? Launch<float, true, -1>::go(a, grid, s) : Launch<float, false, -1>::go(a, grid, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("readout launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

template <typename A, bool V, int FIX>
struct FwdLaunch {
    static void go(const ReadoutArgs& a, int grid, cudaStream_t s) {
        readout_fwd_kernel<A, V, FIX><<<grid, 32 * kReadoutWarps, 0, s>>>(a);
    }
};
template <typename A, bool V, int FIX>
struct BwdLaunch {
    static void go(const ReadoutArgs& a, int grid, cudaStream_t s) {
        readout_bwd_kernel<A, V, FIX><<<grid, 32 * kReadoutWarps, 0, s>>>(a);
    }
};

// The one 16-bit dtype code shared by every given code, or -1.
int common16(std::initializer_list<int> dts) {
    const int first = *dts.begin();
    if (first != ESA_DTYPE_F16 && first != ESA_DTYPE_BF16) return -1;
    for (int d : dts)
        if (d != first) return -1;
    return first;
}

int check_operand(const void* p, int64_t rs, int dt, int64_t C, const char* name, int* es) {
    *es = dtype_size(dt);
    if (*es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, std::string(name) + ": unsupported dtype code");
    if (p == nullptr) return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
    if (rs < C) return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(name) + ": row stride smaller than C");
    return ESA_OK;
}

}  // namespace

int readout_fwd(const void* q, int64_t qrs, int qdt, const void* E, int64_t ers, int edt, void* y,
                int64_t yrs, int ydt, void* rstd, int64_t rows, int64_t C, double eps, cudaStream_t s) {
    if (rows < 0 || C < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "negative dimension");
    if (rows == 0 || C == 0) return ESA_OK;
    ReadoutArgs a{};
    int es = 0;
    if (int rc = check_operand(q, qrs, qdt, C, "q", &es)) return rc;
    a.q = {static_cast<const char*>(q), qrs, qdt, es};
    if (int rc = check_operand(E, ers, edt, C, "E", &es)) return rc;
    a.E = {static_cast<const char*>(E), ers, edt, es};
    if (int rc = check_operand(y, yrs, ydt, C, "y", &es)) return rc;
    a.y = {static_cast<char*>(y), yrs, ydt, es};
    if (rstd == nullptr) return set_error(ESA_ERR_INVALID_ARGUMENT, "rstd is null");
    a.rstd = rstd;
    a.rows = rows;
    a.C = C;
    a.eps = eps;
    const bool wide = qdt == ESA_DTYPE_F64 || edt == ESA_DTYPE_F64 || ydt == ESA_DTYPE_F64;
    const bool vect = C % 8 == 0 && vec_ok(q, qrs, a.q.es) && vec_ok(E, ers, a.E.es) && vec_ok(y, yrs, a.y.es);
    return readout_launch<FwdLaunch>(a, wide, vect, common16({qdt, edt, ydt}), s);
}

int readout_bwd(const void* dy, int64_t dyrs, int dydt, const void* q, int64_t qrs, int qdt, const void* E,
                int64_t ers, int edt, const void* rstd, void* dq, int64_t dqrs, int dqdt, void* dE,
                int64_t ders, int dedt, int64_t rows, int64_t C, double eps, cudaStream_t s) {
    if (rows < 0 || C < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "negative dimension");
    if (rows == 0 || C == 0) return ESA_OK;
    ReadoutArgs a{};
    int es = 0;
    if (int rc = check_operand(dy, dyrs, dydt, C, "dy", &es)) return rc;
    a.dy = {static_cast<const char*>(dy), dyrs, dydt, es};
    if (int rc = check_operand(q, qrs, qdt, C, "q", &es)) return rc;
    a.q = {static_cast<const char*>(q), qrs, qdt, es};
    if (int rc = check_operand(E, ers, edt, C, "E", &es)) return rc;
    a.E = {static_cast<const char*>(E), ers, edt, es};
    if (int rc = check_operand(dq, dqrs, dqdt, C, "dq", &es)) return rc;
    a.dq = {static_cast<char*>(dq), dqrs, dqdt, es};
    if (int rc = check_operand(dE, ders, dedt, C, "dE", &es)) return rc;
    a.dE = {static_cast<char*>(dE), ders, dedt, es};
    if (rstd == nullptr) return set_error(ESA_ERR_INVALID_ARGUMENT, "rstd is null");
    a.rstd = const_cast<void*>(rstd);
    a.rows = rows;
    a.C = C;
    a.eps = eps;
    const bool wide = dydt == ESA_DTYPE_F64 || qdt == ESA_DTYPE_F64 || edt == ESA_DTYPE_F64 ||
                      dqdt == ESA_DTYPE_F64 || dedt == ESA_DTYPE_F64;
    const bool vect = C % 8 == 0 && vec_ok(dy, dyrs, a.dy.es) && vec_ok(q, qrs, a.q.es) &&
                      vec_ok(E, ers, a.E.es) && vec_ok(dq, dqrs, a.dq.es) && vec_ok(dE, ders, a.dE.es);
    return readout_launch<BwdLaunch>(a, wide, vect, common16({dydt, qdt, edt, dqdt, dedt}), s);
}

}  // namespace esa
