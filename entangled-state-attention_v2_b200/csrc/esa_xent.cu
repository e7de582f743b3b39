// esa_xent.cu -- cross-entropy of the LM head, the ESAModel training loss.
//
//   lse_i  = log sum_j exp(z_ij)                 (z = logits row i, V columns)
//   loss_i = lse_i - z_{i, t_i}                  (0 where t_i == ignore_index)
//   dz_ij  = g_i * (exp(z_ij - lse_i) - [j == t_i])   (0 where t_i is ignored)
//
// The reference computes `F.cross_entropy(logits.reshape(-1, V), targets,
// ignore_index=-1)` (esa/model.py); under fp16 autocast PyTorch runs it as an
// fp32 log-softmax of an fp32 copy of the logits, keeps that [rows, V] fp32
// result for the backward, and casts the fp32 gradient back to the logits'
// dtype -- about 20 % of the [16, 2048] x 32000 training step.  Here the
// forward reads the logits once (rows x 2 bytes x V) and keeps 4 bytes a row
// (lse); the backward reads them once more and writes the gradient in the
// logits' dtype.  Arithmetic in fp32; the mean over the rows that are not
// ignored is left to the caller (a sum of `loss` over rows divided by their
// count), whose per-row gradient g_i the backward takes.
//
// One CTA of 256 threads per row (a persistent grid over the rows): 16-byte
// vector loads, four in flight per thread; the forward's running (max, sum of
// exponentials) pairs combine across the CTA through warp shuffles and shared
// memory.  16-bit logits use __expf (error far below their 2^-11 rounding);
// fp32 logits use expf.
#include <cmath>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"
#include "esa_rowops.cuh"

namespace esa {
namespace {

constexpr int kXentThreads = 256;

template <typename T>
struct XentIo {
    static constexpr int PER = 16 / (int)sizeof(T);  // elements per 16-byte vector
    static __device__ __forceinline__ float ld(const T* p) { return Elem<T>::to_acc(*p); }
    static __device__ __forceinline__ void ldv(const T* p, float (&x)[PER]) {
        const VecN<T, PER> v = *reinterpret_cast<const VecN<T, PER>*>(p);
#pragma unroll
        for (int i = 0; i < PER; ++i) x[i] = Elem<T>::to_acc(v.v[i]);
    }
    static __device__ __forceinline__ void stv(T* p, const float (&x)[PER]) {
        VecN<T, PER> v;
#pragma unroll
        for (int i = 0; i < PER; ++i) v.v[i] = Elem<T>::from_acc(x[i]);
        *reinterpret_cast<VecN<T, PER>*>(p) = v;
    }
};

template <typename T>
__device__ __forceinline__ float xexp(float x) {
    if constexpr (sizeof(T) == 2)
        return __expf(x);
    else
        return expf(x);
}

// (m, s) pairs: s = sum exp(z - m).  Combine two, guarding m = -inf.
__device__ __forceinline__ void lse_combine(float& m, float& s, float m2, float s2) {
    const float mm = fmaxf(m, m2);
    if (mm == -INFINITY) {
        s = 0.f;
        m = mm;
        return;
    }
    s = s * expf(m - mm) + s2 * expf(m2 - mm);
    m = mm;
}

struct XentArgs {
    const char* z;
    int64_t ld;  // row stride of the logits (elements)
    const int64_t* t;
    int64_t ignore;
    float* lse;
    float* loss;
    const float* g;  // backward: per-row gradient of loss
    char* dz;
    int64_t dld;
    int64_t rows, V;
};

template <typename T, bool VECT>
__global__ void __launch_bounds__(kXentThreads) xent_fwd_kernel(const XentArgs a) {
    using Io = XentIo<T>;
    constexpr int PER = Io::PER;
    __shared__ float red_m[kXentThreads / 32], red_s[kXentThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const T* zr = reinterpret_cast<const T*>(a.z) + row * a.ld;
        float m = -INFINITY, s = 0.f;
        if constexpr (VECT) {
            const int64_t nvec = a.V / PER;
            int64_t v = tid;
            // four vectors in flight per thread
            for (; v + 3 * kXentThreads < nvec; v += 4 * kXentThreads) {
                float x[4][PER];
#pragma unroll
                for (int u = 0; u < 4; ++u) Io::ldv(zr + (v + u * kXentThreads) * PER, x[u]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float mv = x[u][0];
#pragma unroll
                    for (int i = 1; i < PER; ++i) mv = fmaxf(mv, x[u][i]);
                    if (mv > m) {
                        s *= xexp<T>(m - mv);
                        m = mv;
                    }
#pragma unroll
                    for (int i = 0; i < PER; ++i) s += xexp<T>(x[u][i] - m);
                }
            }
            for (; v < nvec; v += kXentThreads) {
                float x[PER];
                Io::ldv(zr + v * PER, x);
                float mv = x[0];
#pragma unroll
                for (int i = 1; i < PER; ++i) mv = fmaxf(mv, x[i]);
                if (mv > m) {
                    s *= xexp<T>(m - mv);
                    m = mv;
                }
#pragma unroll
                for (int i = 0; i < PER; ++i) s += xexp<T>(x[i] - m);
            }
        } else {
            for (int64_t j = tid; j < a.V; j += kXentThreads) {
                const float x = Io::ld(zr + j);
                if (x > m) {
                    s *= xexp<T>(m - x);
                    m = x;
                }
                s += xexp<T>(x - m);
            }
        }
        // CTA reduction of the (m, s) pairs
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
            const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
            lse_combine(m, s, m2, s2);
        }
        if (lane == 0) {
            red_m[warp] = m;
            red_s[warp] = s;
        }
        __syncthreads();
        if (tid == 0) {
            float mm = red_m[0], ss = red_s[0];
            for (int w = 1; w < kXentThreads / 32; ++w) lse_combine(mm, ss, red_m[w], red_s[w]);
            const float l = mm + logf(ss);
            a.lse[row] = l;
            const int64_t t = a.t[row];
            float loss = 0.f;
            if (t != a.ignore) loss = (t >= 0 && t < a.V) ? l - Io::ld(zr + t) : NAN;
            a.loss[row] = loss;
        }
        __syncthreads();
    }
}

template <typename T, bool VECT>
__global__ void __launch_bounds__(kXentThreads) xent_bwd_kernel(const XentArgs a) {
    using Io = XentIo<T>;
    constexpr int PER = Io::PER;
    const int tid = threadIdx.x;
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const T* zr = reinterpret_cast<const T*>(a.z) + row * a.ld;
        T* dr = reinterpret_cast<T*>(a.dz) + row * a.dld;
        const int64_t t = a.t[row];
        const bool ignored = t == a.ignore;
        // a target outside [0, V) that is not ignored gives a NaN gradient
        // row, as its loss is NaN (never a silently plausible gradient)
        const bool bad = !ignored && (t < 0 || t >= a.V);
        const float g = ignored ? 0.f : (bad ? __int_as_float(0x7fffffff) : a.g[row]);
        const float l = a.lse[row];
        if constexpr (VECT) {
            const int64_t nvec = a.V / PER;
            for (int64_t v = tid; v < nvec; v += kXentThreads) {
                float x[PER];
                Io::ldv(zr + v * PER, x);
#pragma unroll
                for (int i = 0; i < PER; ++i) {
                    const float p = ignored ? 0.f : xexp<T>(x[i] - l);
                    x[i] = g * (p - (v * PER + i == t ? 1.f : 0.f));
                }
                Io::stv(dr + v * PER, x);
            }
        } else {
            for (int64_t j = tid; j < a.V; j += kXentThreads) {
                const float p = ignored ? 0.f : xexp<T>(Io::ld(zr + j) - l);
                dr[j] = Elem<T>::from_acc(g * (p - (j == t ? 1.f : 0.f)));
            }
        }
    }
}

int xent_grid(int64_t rows) { return (int)(rows < 148 * 8 ? rows : 148 * 8); }

template <template <typename, bool> class K>
int xent_dispatch(int dtype, bool vect, const XentArgs& a, cudaStream_t s) {
    const int grid = xent_grid(a.rows);
    switch (dtype) {
        case ESA_DTYPE_F16:
            vect ? K<__half, true>::go(a, grid, s) : K<__half, false>::go(a, grid, s);
            break;
        case ESA_DTYPE_BF16:
            vect ? K<__nv_bfloat16, true>::go(a, grid, s) : K<__nv_bfloat16, false>::go(a, grid, s);
            break;
        case ESA_DTYPE_F32:
            vect ? K<float, true>::go(a, grid, s) : K<float, false>::go(a, grid, s);
            break;
        default: return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "cross entropy: logits must be f16, bf16 or f32");
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("cross entropy launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

template <typename T, bool V>
struct FwdK {
    static void go(const XentArgs& a, int grid, cudaStream_t s) {
        xent_fwd_kernel<T, V><<<grid, kXentThreads, 0, s>>>(a);
    }
};
template <typename T, bool V>
struct BwdK {
    static void go(const XentArgs& a, int grid, cudaStream_t s) {
        xent_bwd_kernel<T, V><<<grid, kXentThreads, 0, s>>>(a);
    }
};

bool vec_rows(const void* p, int64_t ld, int64_t V, int es) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (ld * es) % 16 == 0 && (V * es) % 16 == 0;
}

int xent_check(int64_t rows, int64_t V, int64_t ld, int dtype) {
    if (rows < 0 || V <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "cross entropy: need rows >= 0 and V > 0");
    if (ld < V) return set_error(ESA_ERR_INVALID_ARGUMENT, "cross entropy: row stride smaller than V");
    if (dtype != ESA_DTYPE_F16 && dtype != ESA_DTYPE_BF16 && dtype != ESA_DTYPE_F32)
        return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "cross entropy: logits must be f16, bf16 or f32");
    return ESA_OK;
}

}  // namespace

int cross_entropy_fwd(const void* logits, int64_t ld, int dtype, const int64_t* targets, int64_t ignore_index,
                      float* lse, float* loss, int64_t rows, int64_t V, cudaStream_t s) {
    if (int rc = xent_check(rows, V, ld, dtype)) return rc;
    if (rows == 0) return ESA_OK;
    if (!logits || !targets || !lse || !loss) return set_error(ESA_ERR_INVALID_ARGUMENT, "cross entropy: null pointer");
    XentArgs a{};
    a.z = static_cast<const char*>(logits);
    a.ld = ld;
    a.t = targets;
    a.ignore = ignore_index;
    a.lse = lse;
    a.loss = loss;
    a.rows = rows;
    a.V = V;
    return xent_dispatch<FwdK>(dtype, vec_rows(logits, ld, V, dtype_size(dtype)), a, s);
}

int cross_entropy_bwd(const void* logits, int64_t ld, int dtype, const int64_t* targets, int64_t ignore_index,
                      const float* lse, const float* grad_rows, void* dlogits, int64_t dld, int64_t rows, int64_t V,
                      cudaStream_t s) {
    if (int rc = xent_check(rows, V, ld, dtype)) return rc;
    if (dld < V) return set_error(ESA_ERR_INVALID_ARGUMENT, "cross entropy: gradient row stride smaller than V");
    if (rows == 0) return ESA_OK;
    if (!logits || !targets || !lse || !grad_rows || !dlogits)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "cross entropy: null pointer");
    XentArgs a{};
    a.z = static_cast<const char*>(logits);
    a.ld = ld;
    a.t = targets;
    a.ignore = ignore_index;
    a.lse = const_cast<float*>(lse);
    a.g = grad_rows;
    a.dz = static_cast<char*>(dlogits);
    a.dld = dld;
    a.rows = rows;
    a.V = V;
    const int es = dtype_size(dtype);
    return xent_dispatch<BwdK>(dtype, vec_rows(logits, ld, V, es) && vec_rows(dlogits, dld, V, es), a, s);
}

}  // namespace esa
