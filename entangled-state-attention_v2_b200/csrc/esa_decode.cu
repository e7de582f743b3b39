// esa_decode.cu -- one ESAModel block's decode step (a few rows, 16-bit data)
// in four launches instead of about eleven.
//
// A decode step at batch 1 reads every weight once and does little else, so
// what costs is the number of dependent launches: per block the residual
// adds, two LayerNorms, four Linear layers, GELU and the Lightning step, each
// a separate small kernel (esa/model.py block loop, esa/generation.py:
// 410-469).  Here each Linear is a GEMV kernel whose input vector is built by
// a prologue that every CTA computes redundantly from the (L2-resident)
// activations, and whose bias / GELU epilogue is fused:
//
//   K1  s1 = x + pending;  h1 = LN1(s1);        qgv = W_qgv h1 + b
//   K2  S' = Lightning(qgv, S);  z = readout;    y = W_out z + b
//   K3  s2 = s1 + y;  h2 = LN2(s2);              a = GELU(W_fc h2 + b)
//   K4                                           pending' = W_proj a + b
//
// and the LM head is K1's form with LN_f and the (tied) embedding matrix.
// Rounding follows the PyTorch path it replaces: the residual sums, the
// LayerNorm outputs, every Linear output (fp32 accumulation + bias, one
// rounding), GELU of the rounded fc output and the Lightning state / readout
// are rounded to the model's 16-bit dtype.
//
// GEMV: one warp per output row at a time (two rows in flight), 16-byte
// non-allocating loads of the weight row, the input vector in shared memory
// as floats, a warp-shuffle reduction.  The kernels of a decode step form a
// chain of programmatic dependent launches: a kernel loads its static data
// (its first two rows' weights, the LayerNorm parameters) before it waits
// for the previous kernel (griddepcontrol.wait) and then releases the next
// one, so its launch and part of its weight latency overlap the
// predecessor's tail.
// Roofline: HBM on the weights (N x K x 2 bytes per launch).
#include <string>

#include "esa_common.cuh"
#include "esa_internal.h"

namespace esa {

namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;

enum Pro { PRO_NORM = 0, PRO_LIGHTNING = 1, PRO_PLAIN = 2 };
enum Epi { EPI_BIAS = 0, EPI_BIAS_GELU = 1 };

struct DecArgs {
    // GEMV: out[b, n] = epi(sum_k W[n, k] xs[b, k] + bias[n]), b < nb, n < N
    const void* W;
    const void* bias;  // nullable
    void* out;
    int64_t N, K;
    int nb;
    // PRO_NORM: s = x (+ res); s_out = s (nullable; written by CTA 0); xs = LN(s)
    const void* x;
    const void* res;  // nullable
    void* s_out;      // nullable
    const void* ln_w;
    const void* ln_b;  // nullable
    float ln_eps;
    // PRO_LIGHTNING: qgv [nb, 3K] -> new_state (this CTA's channel slice), xs = z
    const void* qgv;
    const void* state;
    void* new_state;
    float gmin, gspan, eps;
};

template <typename T>
__device__ __forceinline__ float rnd(float x) {
    return Elem<T>::to_acc(Elem<T>::from_acc(x));
}

// Sum over the CTA (every thread gets the total).
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red may still hold the previous reduction's values
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) t += red[w];
    return t;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_acc(h[i]);
}

// xs[b][k] for k in [k0, k0 + 8)
template <int NB>
__device__ __forceinline__ void dot8(const float* xs, int64_t K, int nb, int64_t k0, const float (&w)[8],
                                     float (&acc)[NB]) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b < nb) {
            const float4 p = *reinterpret_cast<const float4*>(xs + b * K + k0);
            const float4 q = *reinterpret_cast<const float4*>(xs + b * K + k0 + 4);
            acc[b] = fmaf(w[0], p.x, acc[b]);
            acc[b] = fmaf(w[1], p.y, acc[b]);
            acc[b] = fmaf(w[2], p.z, acc[b]);
            acc[b] = fmaf(w[3], p.w, acc[b]);
            acc[b] = fmaf(w[4], q.x, acc[b]);
            acc[b] = fmaf(w[5], q.y, acc[b]);
            acc[b] = fmaf(w[6], q.z, acc[b]);
            acc[b] = fmaf(w[7], q.w, acc[b]);
        }
    }
}

// Number of 16-byte weight chunks a lane keeps in registers per row before
// the prologue (K = 1024: all four of them).
constexpr int kPre = 4;

// LayerNorm parameters a thread keeps in registers (K up to 256 * kLnPer)
constexpr int kLnPer = 4;

template <typename T, int NB, int PRO, int EPI>
__global__ void __launch_bounds__(kDecThreads, 2) decode_gemv_kernel(const DecArgs a) {
    extern __shared__ __align__(16) float xs[];  // [NB][K]
    __shared__ float red[kDecWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t K = a.K;
    const T* W = static_cast<const T*>(a.W);
    const int64_t gw = (int64_t)blockIdx.x * kDecWarps + warp;
    const int64_t wstride = (int64_t)gridDim.x * kDecWarps;

    // Static data first: this warp's first two rows' leading weight chunks and
    // the LayerNorm parameters.  Launched as a programmatic dependent of the
    // previous kernel, this runs while that kernel is still computing.
    uint4 pre[2][kPre];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int64_t n = gw + r * wstride;
#pragma unroll
        for (int j = 0; j < kPre; ++j) {
            const int64_t k0 = (int64_t)j * 256 + lane * 8;
            pre[r][j] = (n < a.N && k0 < K) ? ld_global_nc_v4(W + n * K + k0) : make_uint4(0, 0, 0, 0);
        }
    }
    float lnw[kLnPer], lnb[kLnPer];
    if constexpr (PRO == PRO_NORM) {
        const T* lw = static_cast<const T*>(a.ln_w);
        const T* lb = static_cast<const T*>(a.ln_b);
#pragma unroll
        for (int i = 0; i < kLnPer; ++i) {
            const int64_t k = threadIdx.x + (int64_t)i * kDecThreads;
            lnw[i] = k < K ? Elem<T>::to_acc(lw[k]) : 0.0f;
            lnb[i] = (k < K && lb != nullptr) ? Elem<T>::to_acc(lb[k]) : 0.0f;
        }
    }
    // the activations below are written by the previous kernels: wait for
    // them, then let the next kernel of the chain start its own prefetch
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // ---- prologue: the input vectors ------------------------------------------
    if constexpr (PRO == PRO_PLAIN) {
        const T* x = static_cast<const T*>(a.x);
        for (int b = 0; b < a.nb; ++b)
            for (int64_t k = threadIdx.x; k < K; k += kDecThreads) xs[b * K + k] = Elem<T>::to_acc(x[b * K + k]);
    } else if constexpr (PRO == PRO_NORM) {
        const T* x = static_cast<const T*>(a.x);
        const T* r = static_cast<const T*>(a.res);
        T* so = static_cast<T*>(a.s_out);
        const T* lw = static_cast<const T*>(a.ln_w);
        const T* lb = static_cast<const T*>(a.ln_b);
        for (int b = 0; b < a.nb; ++b) {
            float* row = xs + b * K;
            float sum = 0.0f;
            for (int64_t k = threadIdx.x; k < K; k += kDecThreads) {
                float s = Elem<T>::to_acc(x[b * K + k]);
                if (r != nullptr) s = rnd<T>(s + Elem<T>::to_acc(r[b * K + k]));
                if (so != nullptr && blockIdx.x == 0) so[b * K + k] = Elem<T>::from_acc(s);
                row[k] = s;
                sum += s;
            }
            const float mean = cta_sum(sum, red) / (float)K;
            float sq = 0.0f;
            for (int64_t k = threadIdx.x; k < K; k += kDecThreads) {
                const float d = row[k] - mean;
                sq += d * d;
            }
            const float rstd = rsqrtf(cta_sum(sq, red) / (float)K + a.ln_eps);
            if (K <= (int64_t)kLnPer * kDecThreads) {
#pragma unroll
                for (int i = 0; i < kLnPer; ++i) {
                    const int64_t k = threadIdx.x + (int64_t)i * kDecThreads;
                    if (k < K) row[k] = rnd<T>((row[k] - mean) * rstd * lnw[i] + lnb[i]);
                }
            } else {
                for (int64_t k = threadIdx.x; k < K; k += kDecThreads) {
                    float y = (row[k] - mean) * rstd * Elem<T>::to_acc(lw[k]);
                    if (lb != nullptr) y += Elem<T>::to_acc(lb[k]);
                    row[k] = rnd<T>(y);
                }
            }
        }
    } else {  // PRO_LIGHTNING: K = C channels, qgv rows of 3C
        const T* qgv = static_cast<const T*>(a.qgv);
        const T* st = static_cast<const T*>(a.state);
        T* ns = static_cast<T*>(a.new_state);
        // the channels whose new state this CTA writes
        const int64_t chunk = ((K + gridDim.x - 1) / gridDim.x + 31) / 32 * 32;
        const int64_t c0 = (int64_t)blockIdx.x * chunk, c1 = c0 + chunk < K ? c0 + chunk : K;
        for (int b = 0; b < a.nb; ++b) {
            const T* q = qgv + b * 3 * K;
            float* row = xs + b * K;
            float ss = 0.0f;
            for (int64_t c = threadIdx.x; c < K; c += kDecThreads) {
                // the hardware approximations of the 16-bit gated scans: their
                // errors sit below the 16-bit rounding of A, B and the state
                const float A = fmaf(0.5f * a.gspan, tanh_fast(0.5f * Elem<T>::to_acc(q[K + c])),
                                     a.gmin + 0.5f * a.gspan);
                const float B = (1.0f - A) * tanh_fast(Elem<T>::to_acc(q[2 * K + c]));
                // A and B cast to the state dtype before the update, as the reference does
                const float sp = rnd<T>(rnd<T>(A) * Elem<T>::to_acc(st[b * K + c]) + rnd<T>(B));
                if (c >= c0 && c < c1) ns[b * K + c] = Elem<T>::from_acc(sp);
                row[c] = sp;
                ss += sp * sp;
            }
            const float rr = 1.0f / sqrtf(cta_sum(ss, red) / (float)K + a.eps);
            for (int64_t c = threadIdx.x; c < K; c += kDecThreads)
                row[c] = rnd<T>(sigmoid_fast(Elem<T>::to_acc(q[c])) * row[c] * rr);
        }
    }
    __syncthreads();

    // ---- GEMV -------------------------------------------------------------------
    const T* bias = static_cast<const T*>(a.bias);
    T* out = static_cast<T*>(a.out);
    auto finish = [&](int64_t n, float (&acc)[NB]) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
        }
        if (lane < a.nb) {
            float v = 0.0f;
#pragma unroll
            for (int b = 0; b < NB; ++b)
                if (b == lane) v = acc[b];
            if (bias != nullptr) v += Elem<T>::to_acc(bias[n]);
            v = rnd<T>(v);
            if constexpr (EPI == EPI_BIAS_GELU) v = rnd<T>(0.5f * v * (1.0f + erff(v * 0.70710678118654752f)));
            out[(int64_t)lane * a.N + n] = Elem<T>::from_acc(v);
        }
    };
    bool first = true;
    for (int64_t n = gw; n < a.N; n += 2 * wstride) {
        const int64_t n2 = n + wstride;
        const bool has2 = n2 < a.N;
        float acc[NB], acc2[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            acc[b] = 0.0f;
            acc2[b] = 0.0f;
        }
        for (int64_t kb = 0; kb < K; kb += 256 * kPre) {
            uint4 u[kPre], u2[kPre];
#pragma unroll
            for (int j = 0; j < kPre; ++j) {
                const int64_t k0 = kb + (int64_t)j * 256 + lane * 8;
                if (first && kb == 0) {
                    u[j] = pre[0][j];
                    u2[j] = pre[1][j];
                } else {
                    u[j] = k0 < K ? ld_global_nc_v4(W + n * K + k0) : make_uint4(0, 0, 0, 0);
                    u2[j] = (has2 && k0 < K) ? ld_global_nc_v4(W + n2 * K + k0) : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int j = 0; j < kPre; ++j) {
                const int64_t k0 = kb + (int64_t)j * 256 + lane * 8;
                if (k0 < K) {
                    float w[8];
                    unpack8<T>(u[j], w);
                    dot8<NB>(xs, K, a.nb, k0, w, acc);
                    if (has2) {
                        unpack8<T>(u2[j], w);
                        dot8<NB>(xs, K, a.nb, k0, w, acc2);
                    }
                }
            }
        }
        first = false;
        finish(n, acc);
        if (has2) finish(n2, acc2);
    }
}

template <typename T, int NB, int PRO, int EPI>
int launch_one(const DecArgs& a, cudaStream_t s) {
    const size_t smem = (size_t)NB * a.K * sizeof(float);
    auto kern = decode_gemv_kernel<T, NB, PRO, EPI>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("decode smem attribute: ") + cudaGetErrorString(e));
    }
    int dev = 0;
    cudaGetDevice(&dev);
    // a row per warp while the rows are few, then two rows in flight per
    // warp, on up to two CTAs per SM.  (One CTA per SM, so that the next
    // kernel of the chain could be resident while this one runs, measured
    // slower: 0.709 against 0.600 ms per decoded token of the 24-layer,
    // 1024-wide fp16 model; without the programmatic launch 0.672.)
    int64_t grid = (a.N + kDecWarps - 1) / kDecWarps;
    const int64_t cap = 2 * (int64_t)device_sm_count(dev);
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid);
    lc.blockDim = dim3(kDecThreads);
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&lc, kern, a);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

template <typename T, int PRO, int EPI>
int launch_nb(const DecArgs& a, cudaStream_t s) {
    if (a.nb <= 1) return launch_one<T, 1, PRO, EPI>(a, s);
    if (a.nb <= 2) return launch_one<T, 2, PRO, EPI>(a, s);
    return launch_one<T, 4, PRO, EPI>(a, s);
}

template <typename T>
int launch_typed(const DecArgs& a, int pro, int epi, cudaStream_t s) {
    if (pro == PRO_NORM && epi == EPI_BIAS) return launch_nb<T, PRO_NORM, EPI_BIAS>(a, s);
    if (pro == PRO_NORM && epi == EPI_BIAS_GELU) return launch_nb<T, PRO_NORM, EPI_BIAS_GELU>(a, s);
    if (pro == PRO_LIGHTNING) return launch_nb<T, PRO_LIGHTNING, EPI_BIAS>(a, s);
    return launch_nb<T, PRO_PLAIN, EPI_BIAS>(a, s);
}

int launch(const DecArgs& a, int dtype, int pro, int epi, cudaStream_t s) {
    switch (dtype) {
        case ESA_DTYPE_F16: return launch_typed<__half>(a, pro, epi, s);
        case ESA_DTYPE_BF16: return launch_typed<__nv_bfloat16>(a, pro, epi, s);
        default: return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "decode kernels take fp16 or bf16 data");
    }
}

int check_shape(int64_t nb, int64_t C, int dtype) {
    if (nb < 1 || nb > kDecodeMaxRows)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "decode kernels take 1 to " + std::to_string(kDecodeMaxRows) + " rows");
    if (C <= 0 || C % 256 != 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "decode kernels need C a multiple of 256");
    if (dtype != ESA_DTYPE_F16 && dtype != ESA_DTYPE_BF16)
        return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "decode kernels take fp16 or bf16 data");
    return ESA_OK;
}

// The GEMVs read weight rows with 16-byte loads.
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

size_t decode_block_scratch_bytes(int64_t nb, int64_t C, int dtype) {
    if (check_shape(nb, C, dtype) != ESA_OK) return 0;
    // s1 [nb, C], qgv [nb, 3C], y [nb, C], act [nb, 4C]
    return (size_t)nb * C * 9 * 2;
}

int decode_block(const DecodeBlock& p, cudaStream_t s) {
    if (int rc = check_shape(p.nb, p.C, p.dtype)) return rc;
    const size_t need = decode_block_scratch_bytes(p.nb, p.C, p.dtype);
    if (p.scratch == nullptr || p.scratch_bytes < need || (reinterpret_cast<uintptr_t>(p.scratch) & 15u))
        return set_error(ESA_ERR_WORKSPACE, "decode scratch missing, misaligned or smaller than esa_decode_block_scratch_bytes()");
    if (!p.x || !p.x_out || !p.pending_out || !p.state || !p.new_state || !p.ln1_w || !p.qgv_w || !p.out_w ||
        !p.ln2_w || !p.fc_w || !p.proj_w)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (p.state == p.new_state) return set_error(ESA_ERR_INVALID_ARGUMENT, "new_state must not alias state");
    if (!aligned16(p.qgv_w) || !aligned16(p.out_w) || !aligned16(p.fc_w) || !aligned16(p.proj_w))
        return set_error(ESA_ERR_INVALID_ARGUMENT, "decode weight matrices must be 16-byte aligned");
    const int64_t nb = p.nb, C = p.C;
    char* sc = static_cast<char*>(p.scratch);
    void* s1 = sc;
    void* qgv = sc + nb * C * 2;
    void* y = sc + nb * C * 8;
    void* act = sc + nb * C * 10;
    // K1: s1 = x + pending, h1 = LN1(s1), qgv = W h1 + b
    DecArgs a{};
    a.nb = (int)nb;
    a.x = p.x;
    a.res = p.pending;
    a.s_out = s1;
    a.ln_w = p.ln1_w;
    a.ln_b = p.ln1_b;
    a.ln_eps = (float)p.ln_eps;
    a.W = p.qgv_w;
    a.bias = p.qgv_b;
    a.out = qgv;
    a.N = 3 * C;
    a.K = C;
    if (int rc = launch(a, p.dtype, PRO_NORM, EPI_BIAS, s)) return rc;
    // K2: Lightning step + readout, y = W_out z + b
    DecArgs b{};
    b.nb = (int)nb;
    b.qgv = qgv;
    b.state = p.state;
    b.new_state = p.new_state;
    b.gmin = (float)p.gate_min;
    b.gspan = (float)(p.gate_max - p.gate_min);
    b.eps = (float)p.eps;
    b.W = p.out_w;
    b.bias = p.out_b;
    b.out = y;
    b.N = C;
    b.K = C;
    if (int rc = launch(b, p.dtype, PRO_LIGHTNING, EPI_BIAS, s)) return rc;
    // K3: s2 = s1 + y -> x_out, h2 = LN2(s2), act = GELU(W_fc h2 + b)
    DecArgs c{};
    c.nb = (int)nb;
    c.x = s1;
    c.res = y;
    c.s_out = p.x_out;
    c.ln_w = p.ln2_w;
    c.ln_b = p.ln2_b;
    c.ln_eps = (float)p.ln_eps;
    c.W = p.fc_w;
    c.bias = p.fc_b;
    c.out = act;
    c.N = 4 * C;
    c.K = C;
    if (int rc = launch(c, p.dtype, PRO_NORM, EPI_BIAS_GELU, s)) return rc;
    // K4: pending' = W_proj act + b
    DecArgs d{};
    d.nb = (int)nb;
    d.x = act;
    d.W = p.proj_w;
    d.bias = p.proj_b;
    d.out = p.pending_out;
    d.N = C;
    d.K = 4 * C;
    return launch(d, p.dtype, PRO_PLAIN, EPI_BIAS, s);
}

int decode_head(const void* x, const void* pending, const void* ln_w, const void* ln_b, double ln_eps,
                const void* W, const void* bias, void* logits, int64_t nb, int64_t C, int64_t V, int dtype,
                cudaStream_t s) {
    if (int rc = check_shape(nb, C, dtype)) return rc;
    if (V <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "vocabulary size must be positive");
    if (!x || !ln_w || !W || !logits) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(W)) return set_error(ESA_ERR_INVALID_ARGUMENT, "decode weight matrices must be 16-byte aligned");
    DecArgs a{};
    a.nb = (int)nb;
    a.x = x;
    a.res = pending;
    a.s_out = nullptr;
    a.ln_w = ln_w;
    a.ln_b = ln_b;
    a.ln_eps = (float)ln_eps;
    a.W = W;
    a.bias = bias;
    a.out = logits;
    a.N = V;
    a.K = C;
    return launch(a, dtype, PRO_NORM, EPI_BIAS, s);
}

}  // namespace esa
