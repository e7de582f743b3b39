// esa_layernorm.cu -- LayerNorm of the ESAModel residual stream, fused with
// the dtype cast its consumer needs.
//
//   y = (x - mean) * rstd * w + b,   rstd = 1 / sqrt(var + eps)   (biased var)
//
// (the blocks' `F.layer_norm(x, (C,), w, b, 1e-5)`, esa/model.py of the
// reference).  Under fp16/bf16 autocast PyTorch computes it in fp32, writes
// an fp32 tensor, and the Linear that consumes it casts that to the autocast
// dtype in a separate copy; here the normalisation writes the autocast dtype
// directly (the same values: one rounding of the fp32 result), and the
// backward takes the Linear's 16-bit input gradient without the cast back.
//
// Forward: one warp per row of C channels, the row held in registers (one
// read; mean, then the variance about it, then the outputs; arithmetic in
// fp32); the row's mean and rstd are kept.  Optionally fused with the
// residual add before it: xsum = x + res is written (rounded to x's dtype, as
// the separate add would) and normalised; the backward then adds xsum's own
// gradient into dx and writes dx a second time in res's dtype (the gradient
// of res).
// Backward, per row: xhat = (x - mean) rstd, g = dy w,
//   dx = rstd (g - mean_C(g) - xhat mean_C(g xhat));
// the column sums dw = sum_rows dy xhat, db = sum_rows dy are accumulated per
// lane over the rows of a CTA, reduced across its warps in shared memory into
// one partial row per CTA, and the partial rows are summed by a second kernel
// in a fixed order (deterministic, no atomics).
#include <string>
#include <type_traits>

#include "../../include/esa_b200.h"
#include "esa_internal.h"
#include "esa_rowops.cuh"

namespace esa {
namespace {

using namespace rowops;

constexpr int kLnWarps = 8;
constexpr int kLnMaxChunks = 8;  // 8-channel chunks per lane: C <= 2048

struct LnArgs {
    const char* x;
    int xdt, xes;
    // fused residual add (forward): xsum = x + res in x's dtype, normalised
    const char* res;
    int rdt, res_es;
    char* xsum;
    // backward: optional gradient of xsum added to dx; optional second copy
    // of dx in res's dtype (the gradient of res)
    const char* dsum;
    int dsdt, dses;
    char* dres;
    const char* w;
    const char* b;
    int wdt, wes;
    char* y;
    int ydt, yes;
    const char* dy;
    int dydt, dyes;
    char* dx;
    float* mean;
    float* rstd;
    float* partial;  // [grid][2][C]: dw, db partial sums per CTA
    int64_t rows, C;
    float eps;
};

// MIX >= 0: the autocast training mix -- x, w, b (and xsum, dx, and the
// gradient of xsum) fp32, y / dy (and res / its gradient) of the 16-bit dtype
// code MIX -- resolved at compile time, so no load or store switches on a
// dtype code; MIX < 0: every dtype read from the arguments at run time.
template <int MIX>
struct LnTypes {
    int xdt, xes, wdt, wes, ydt, yes, rdt, res_es, dydt, dyes, dsdt, dses;
    __device__ __forceinline__ explicit LnTypes(const LnArgs& a)
        : xdt(MIX >= 0 ? ESA_DTYPE_F32 : a.xdt), xes(MIX >= 0 ? 4 : a.xes),
          wdt(MIX >= 0 ? ESA_DTYPE_F32 : a.wdt), wes(MIX >= 0 ? 4 : a.wes),
          ydt(MIX >= 0 ? MIX : a.ydt), yes(MIX >= 0 ? 2 : a.yes),
          rdt(MIX >= 0 ? MIX : a.rdt), res_es(MIX >= 0 ? 2 : a.res_es),
          dydt(MIX >= 0 ? MIX : a.dydt), dyes(MIX >= 0 ? 2 : a.dyes),
          dsdt(MIX >= 0 ? ESA_DTYPE_F32 : a.dsdt), dses(MIX >= 0 ? 4 : a.dses) {}
};

template <int NCH, int MIX>
__global__ void __launch_bounds__(32 * kLnWarps) ln_fwd_kernel(const LnArgs a) {
    const LnTypes<MIX> ty(a);
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kLnWarps;
    const float inv_c = 1.0f / float(a.C);
    for (int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5); row < a.rows; row += nw) {
        const char* xr = a.x + row * a.C * ty.xes;
        char* yr = a.y + row * a.C * ty.yes;
        // the row stays in registers: one read of x (and res), three reductions
        float v[NCH][8];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
            const int64_t c0 = lane * 8 + k * 256;
            if (c0 < a.C) {
                load8(xr + c0 * ty.xes, ty.xdt, v[k]);
                if (a.res != nullptr) {
                    // xsum = x + res, rounded to x's dtype as a separate add would be
                    float u[8];
                    load8(a.res + (row * a.C + c0) * ty.res_es, ty.rdt, u);
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[k][i] = round_dt(v[k][i] + u[i], ty.xdt);
                    store8(a.xsum + (row * a.C + c0) * ty.xes, ty.xdt, v[k]);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) s += v[k][i];
            }
        }
        const float mu = warp_sum(s) * inv_c;
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
            const int64_t c0 = lane * 8 + k * 256;
            if (c0 < a.C)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float d = v[k][i] - mu;
                    q = fmaf(d, d, q);
                }
        }
        const float r = rsqrt_acc(warp_sum(q) * inv_c + a.eps);
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
            const int64_t c0 = lane * 8 + k * 256;
            if (c0 < a.C) {
                float w[8], bb[8], o[8];
                load8(a.w + c0 * ty.wes, ty.wdt, w);
                load8(a.b + c0 * ty.wes, ty.wdt, bb);
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = fmaf((v[k][i] - mu) * r, w[i], bb[i]);
                store8(yr + c0 * ty.yes, ty.ydt, o);
            }
        }
        if (lane == 0) {
            a.mean[row] = mu;
            a.rstd[row] = r;
        }
    }
}

template <int NCH, int MIX>
__global__ void __launch_bounds__(32 * kLnWarps) ln_bwd_kernel(const LnArgs a) {
    extern __shared__ float ln_smem[];  // [kLnWarps][2][C]
    const LnTypes<MIX> ty(a);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t nw = (int64_t)gridDim.x * kLnWarps;
    const float inv_c = 1.0f / float(a.C);
    float dw[NCH][8], db[NCH][8];
#pragma unroll
    for (int k = 0; k < NCH; ++k)
#pragma unroll
        for (int i = 0; i < 8; ++i) dw[k][i] = db[k][i] = 0.f;
    for (int64_t row = (int64_t)blockIdx.x * kLnWarps + warp; row < a.rows; row += nw) {
        const char* xr = a.x + row * a.C * ty.xes;
        const char* dyr = a.dy + row * a.C * ty.dyes;
        char* dxr = a.dx + row * a.C * ty.xes;
        const float mu = a.mean[row], r = a.rstd[row];
        float sg = 0.f, sgx = 0.f;
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
            const int64_t c0 = lane * 8 + k * 256;
            if (c0 < a.C) {
                float v[8], d[8], w[8];
                load8(xr + c0 * ty.xes, ty.xdt, v);
                load8(dyr + c0 * ty.dyes, ty.dydt, d);
                load8(a.w + c0 * ty.wes, ty.wdt, w);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float xh = (v[i] - mu) * r;
                    const float g = d[i] * w[i];
                    sg += g;
                    sgx = fmaf(g, xh, sgx);
                    dw[k][i] = fmaf(d[i], xh, dw[k][i]);
                    db[k][i] += d[i];
                }
            }
        }
        const float mg = warp_sum(sg) * inv_c, mgx = warp_sum(sgx) * inv_c;
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
            const int64_t c0 = lane * 8 + k * 256;
            if (c0 < a.C) {
                float v[8], d[8], w[8], o[8];
                load8(xr + c0 * ty.xes, ty.xdt, v);
                load8(dyr + c0 * ty.dyes, ty.dydt, d);
                load8(a.w + c0 * ty.wes, ty.wdt, w);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float xh = (v[i] - mu) * r;
                    o[i] = r * (d[i] * w[i] - mg - xh * mgx);
                }
                if (a.dsum != nullptr) {
                    float ds[8];
                    load8(a.dsum + (row * a.C + c0) * ty.dses, ty.dsdt, ds);
#pragma unroll
                    for (int i = 0; i < 8; ++i) o[i] += ds[i];
                }
                store8(dxr + c0 * ty.xes, ty.xdt, o);
                if (a.dres != nullptr) store8(a.dres + (row * a.C + c0) * ty.res_es, ty.rdt, o);
            }
        }
    }
    // this CTA's column partial sums: warps through shared memory, in order
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
        const int64_t c0 = lane * 8 + k * 256;
        if (c0 < a.C)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                ln_smem[(warp * 2 + 0) * a.C + c0 + i] = dw[k][i];
                ln_smem[(warp * 2 + 1) * a.C + c0 + i] = db[k][i];
            }
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c < 2 * a.C; c += blockDim.x) {
        const int which = (int)(c / a.C);
        const int64_t ch = c - which * a.C;
        float s = 0.f;
        for (int w = 0; w < kLnWarps; ++w) s += ln_smem[(w * 2 + which) * a.C + ch];
        a.partial[((int64_t)blockIdx.x * 2 + which) * a.C + ch] = s;
    }
}

// dw, db = sums of the CTA partial rows: a block of 32 x 8 threads per 32
// columns, each of the 8 thread rows summing every 8th partial row, then a
// fixed-order sum of the 8 in shared memory (deterministic)
__global__ void __launch_bounds__(256) ln_bwd_finalize_kernel(const float* __restrict__ partial, int nblocks,
                                                              int64_t C, char* dw, char* db, int wdt, int wes) {
    __shared__ float part[8][33];
    const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;  // column of [2][C]
    float s = 0.f;
    if (c < 2 * C) {
        const int which = (int)(c / C);
        const int64_t ch = c - which * C;
        for (int k = threadIdx.y; k < nblocks; k += 8) s += partial[((int64_t)k * 2 + which) * C + ch];
    }
    part[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.y == 0 && c < 2 * C) {
        float tot = 0.f;
        for (int y = 0; y < 8; ++y) tot += part[y][threadIdx.x];
        const int which = (int)(c / C);
        const int64_t ch = c - which * C;
        store1<float>((which == 0 ? dw : db) + ch * wes, wdt, tot);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool is16(int dt) { return dt == ESA_DTYPE_F16 || dt == ESA_DTYPE_BF16; }

// Calls f(std::integral_constant<int, n>) for n = 1..kLnMaxChunks (8-channel
// chunks per lane).
template <typename F>
void with_nch(int64_t n, F&& f) {
    switch (n) {
        case 1: f(std::integral_constant<int, 1>{}); break;
        case 2: f(std::integral_constant<int, 2>{}); break;
        case 3: f(std::integral_constant<int, 3>{}); break;
        case 4: f(std::integral_constant<int, 4>{}); break;
        case 5: f(std::integral_constant<int, 5>{}); break;
        case 6: f(std::integral_constant<int, 6>{}); break;
        case 7: f(std::integral_constant<int, 7>{}); break;
        default: f(std::integral_constant<int, 8>{}); break;
    }
}

int ln_check(const void* p, int dt, int64_t C, const char* name, int* es) {
    *es = dtype_size(dt);
    if (*es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, std::string(name) + ": unsupported dtype code");
    if (p == nullptr) return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
    if (!aligned16(p) || (C * *es) % 16 != 0)
        return set_error(ESA_ERR_INVALID_ARGUMENT, std::string(name) + ": rows must be 16-byte aligned");
    return ESA_OK;
}

int ln_grid(int64_t rows) {
    const int64_t need = (rows + kLnWarps - 1) / kLnWarps;
    return (int)(need < 148 * 8 ? need : 148 * 8);
}

// backward: fewer CTAs (each reduces its rows' dw, db once, then writes one
// partial row), two per SM (measured: 126 us on [32768, 768] against 141 us
// with 8 per SM and 146 us with 4 per SM and the sums in shared memory)
int ln_bwd_grid(int64_t rows) {
    const int64_t need = (rows + kLnWarps - 1) / kLnWarps;
    return (int)(need < 148 * 2 ? need : 148 * 2);
}

}  // namespace

int layer_norm_partial_rows(int64_t rows) { return ln_bwd_grid(rows); }

int layer_norm_fwd(const void* x, int xdt, const void* res, int rdt, void* xsum, const void* w,
                   const void* b, int wdt, void* y, int ydt, float* mean, float* rstd, int64_t rows, int64_t C,
                   double eps, cudaStream_t s) {
    if (rows < 0 || C <= 0 || C % 8 != 0 || C > 256 * kLnMaxChunks)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "layer norm: C must be a positive multiple of 8, at most 2048");
    if (rows == 0) return ESA_OK;
    LnArgs a{};
    if (int rc = ln_check(x, xdt, C, "x", &a.xes)) return rc;
    if (int rc = ln_check(w, wdt, C, "w", &a.wes)) return rc;
    if (int rc = ln_check(b, wdt, C, "b", &a.wes)) return rc;
    if (int rc = ln_check(y, ydt, C, "y", &a.yes)) return rc;
    if (!mean || !rstd) return set_error(ESA_ERR_INVALID_ARGUMENT, "layer norm: null mean/rstd");
    if (res != nullptr) {
        int es = 0;
        if (int rc = ln_check(res, rdt, C, "res", &a.res_es)) return rc;
        if (int rc = ln_check(xsum, xdt, C, "xsum", &es)) return rc;
        a.res = static_cast<const char*>(res);
        a.rdt = rdt;
        a.xsum = static_cast<char*>(xsum);
    }
    a.x = static_cast<const char*>(x);
    a.xdt = xdt;
    a.w = static_cast<const char*>(w);
    a.b = static_cast<const char*>(b);
    a.wdt = wdt;
    a.y = static_cast<char*>(y);
    a.ydt = ydt;
    a.mean = mean;
    a.rstd = rstd;
    a.rows = rows;
    a.C = C;
    a.eps = (float)eps;
    const int grid = ln_grid(rows);
    // the autocast training mix (fp32 stream and weights, 16-bit output and residual)
    const int mix = (xdt == ESA_DTYPE_F32 && wdt == ESA_DTYPE_F32 && is16(ydt) && (res == nullptr || rdt == ydt))
                        ? ydt : -1;
    auto launch = [&](auto nch_tag) {
        constexpr int NCH = decltype(nch_tag)::value;
        if (mix == ESA_DTYPE_F16)
            ln_fwd_kernel<NCH, ESA_DTYPE_F16><<<grid, 32 * kLnWarps, 0, s>>>(a);
        else if (mix == ESA_DTYPE_BF16)
            ln_fwd_kernel<NCH, ESA_DTYPE_BF16><<<grid, 32 * kLnWarps, 0, s>>>(a);
        else
            ln_fwd_kernel<NCH, -1><<<grid, 32 * kLnWarps, 0, s>>>(a);
    };
    with_nch((C + 255) / 256, launch);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("layer norm launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

int layer_norm_bwd(const void* dy, int dydt, const void* dsum, int dsdt, const void* x, int xdt,
                   const void* w, int wdt, const float* mean, const float* rstd, void* dx, void* dres, int rdt,
                   void* dw, void* db, float* partial, int64_t rows, int64_t C, cudaStream_t s) {
    if (rows < 0 || C <= 0 || C % 8 != 0 || C > 256 * kLnMaxChunks)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "layer norm: C must be a positive multiple of 8, at most 2048");
    LnArgs a{};
    int es = 0;
    if (int rc = ln_check(x, xdt, C, "x", &a.xes)) return rc;
    if (int rc = ln_check(dx, xdt, C, "dx", &es)) return rc;
    if (int rc = ln_check(w, wdt, C, "w", &a.wes)) return rc;
    if (int rc = ln_check(dw, wdt, C, "dw", &es)) return rc;
    if (int rc = ln_check(db, wdt, C, "db", &es)) return rc;
    if (int rc = ln_check(dy, dydt, C, "dy", &a.dyes)) return rc;
    if (!mean || !rstd || !partial) return set_error(ESA_ERR_INVALID_ARGUMENT, "layer norm: null buffer");
    if (dsum != nullptr) {
        if (int rc = ln_check(dsum, dsdt, C, "dsum", &a.dses)) return rc;
        a.dsum = static_cast<const char*>(dsum);
        a.dsdt = dsdt;
    }
    if (dres != nullptr) {
        if (int rc = ln_check(dres, rdt, C, "dres", &a.res_es)) return rc;
        a.dres = static_cast<char*>(dres);
        a.rdt = rdt;
    }
    a.x = static_cast<const char*>(x);
    a.xdt = xdt;
    a.w = static_cast<const char*>(w);
    a.wdt = wdt;
    a.dy = static_cast<const char*>(dy);
    a.dydt = dydt;
    a.dx = static_cast<char*>(dx);
    a.mean = const_cast<float*>(mean);
    a.rstd = const_cast<float*>(rstd);
    a.partial = partial;
    a.rows = rows;
    a.C = C;
    const int grid = rows > 0 ? ln_bwd_grid(rows) : 1;
    const size_t smem = (size_t)kLnWarps * 2 * C * sizeof(float);
    const int nch = (int)((C + 255) / 256);
    cudaError_t e = cudaSuccess;
    auto launch1 = [&](auto kernel) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) kernel<<<grid, 32 * kLnWarps, smem, s>>>(a);
    };
    // the autocast training mix: fp32 stream, weights and xsum gradient,
    // 16-bit dy and residual gradient
    const int mix = (xdt == ESA_DTYPE_F32 && wdt == ESA_DTYPE_F32 && is16(dydt) &&
                     (dsum == nullptr || dsdt == ESA_DTYPE_F32) && (dres == nullptr || rdt == dydt))
                        ? dydt : -1;
    auto launch = [&](auto nch_tag) {
        constexpr int NCH = decltype(nch_tag)::value;
        if (mix == ESA_DTYPE_F16)
            launch1(ln_bwd_kernel<NCH, ESA_DTYPE_F16>);
        else if (mix == ESA_DTYPE_BF16)
            launch1(ln_bwd_kernel<NCH, ESA_DTYPE_BF16>);
        else
            launch1(ln_bwd_kernel<NCH, -1>);
    };
    with_nch(nch, launch);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess) {
        ln_bwd_finalize_kernel<<<(unsigned)((2 * C + 31) / 32), dim3(32, 8), 0, s>>>(
            partial, grid, C, static_cast<char*>(dw), static_cast<char*>(db), wdt, a.wes);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("layer norm backward: ") + cudaGetErrorString(e));
    return ESA_OK;
}

}  // namespace esa
