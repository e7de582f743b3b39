// esa_scan_api.cu -- host side of the scans: argument checks, path choice,
// tensor maps, and the sequential fallback kernel.
//
// Path choice for every scan kind:
//   1. strip scan (esa_strip.cuh) when every row is 16-byte aligned and there
//      are enough channels to fill the GPU with channel strips -- for the
//      plain forward of 16-bit data (and its summary pass) with at least two
//      warps' worth of channel pairs per SM, its lane-serial form
//      (esa_lane.cuh: one lane per channel pair walking the steps in order);
//   2. few channels and a long time axis: the split scan -- every batch row
//      cut into time pieces that the strip scan treats as rows: a summary
//      pass (each piece's end state from zero and its coefficient product),
//      a composition of the pieces' incoming states in time order (one
//      thread per channel), and the output pass from those exact states;
//   3. otherwise the time-parallel lookback scan (esa_scan_lookback.cu);
//   4. rows that are not 16-byte aligned (odd channel counts, offset views):
//      one thread per channel, sequential over time.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "esa_scan_common.cuh"

namespace esa {

int strip_fwd_plain(const ScanCall& c, bool* taken);
int strip_rev_plain(const ScanCall& c, bool* taken);
int strip_fwd_gated(const ScanCall& c, bool* taken);
int strip_rev_gated(const ScanCall& c, bool* taken);
int strip_fwd_summary(const ScanCall& c, bool* taken);
int strip_summary_launch(const ScanCall& c, bool* taken);

int lane_fwd_plain(const ScanCall& c, bool* taken, double min_warps);
int lane_fwd_summary(const ScanCall& c, bool* taken, double min_warps);
int lane_rev_plain(const ScanCall& c, bool* taken, double min_warps);
int lane_fwd_gated(const ScanCall& c, bool* taken, double min_warps);
int lane_rev_gated(const ScanCall& c, bool* taken, double min_warps);

namespace {
// ESA_SCAN_PATH=lane runs every scan kind on the lane-serial kernel where it
// applies (the test suite's second pass over the scan tests); unset or any
// other value: the automatic choice.
std::string scan_path_env() {
    const char* v = getenv("ESA_SCAN_PATH");
    return v != nullptr ? std::string(v) : std::string();
}
}  // namespace

// Lane-serial scan (esa_lane.cuh) when the channels give every SM at least
// kLaneMinWarps consumer warps.  Automatic only for the plain forward scan of
// 16-bit data and its summary pass; every other kind keeps the strip scan
// unless ESA_SCAN_PATH=lane (the lane form's reverse and gated steps ran
// slower on B200: one lane per channel vector cannot hide their longer
// per-step latency).
constexpr double kLaneMinWarps = 2.0;

int lane_scan_launch(const ScanCall& c, bool* taken) {
    static const std::string path = scan_path_env();
    *taken = false;
    const bool forced = path == "lane";
    const double mw = forced ? 0.0 : kLaneMinWarps;
    const bool fwd16 = (c.kind == Kind::FwdPlain || c.kind == Kind::FwdSummary) && dtype_size(c.te) == 2;
    if (!forced && !fwd16) return ESA_OK;
    if (c.summ || c.kind == Kind::FwdSummary) {
        switch (c.kind) {
            case Kind::FwdPlain:
            case Kind::FwdSummary: return lane_fwd_summary(c, taken, mw);
            case Kind::RevPlain: return lane_rev_plain(c, taken, mw);
            case Kind::FwdGated: return lane_fwd_gated(c, taken, mw);
            case Kind::RevGated: return lane_rev_gated(c, taken, mw);
        }
        return ESA_OK;
    }
    switch (c.kind) {
        case Kind::FwdPlain: return lane_fwd_plain(c, taken, mw);
        case Kind::RevPlain: return lane_rev_plain(c, taken, mw);
        case Kind::FwdGated: return lane_fwd_gated(c, taken, mw);
        case Kind::RevGated: return lane_rev_gated(c, taken, mw);
        case Kind::FwdSummary: return lane_fwd_summary(c, taken, mw);
    }
    return ESA_OK;
}

int strip_scan_launch(const ScanCall& c, bool* taken) {
    if (int rc = lane_scan_launch(c, taken)) return rc;
    if (*taken) return ESA_OK;
    if (c.summ) return strip_summary_launch(c, taken);
    switch (c.kind) {
        case Kind::FwdPlain: return strip_fwd_plain(c, taken);
        case Kind::RevPlain: return strip_rev_plain(c, taken);
        case Kind::FwdGated: return strip_fwd_gated(c, taken);
        case Kind::RevGated: return strip_rev_gated(c, taken);
        case Kind::FwdSummary: return strip_fwd_summary(c, taken);
    }
    *taken = false;
    return ESA_OK;
}

// ---------------------------------------------------------------------------
// Tensor maps (driver entry point fetched through the runtime: no -lcuda).
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool encode_strip_map(CUtensorMap* map, int dtype, const void* base, int64_t nb, int64_t T,
                      int64_t hd, int64_t rs, int ws, int lt, std::string* err, int promo_bytes) {
    auto fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    CUtensorMapDataType dt;
    switch (dtype) {
        case ESA_DTYPE_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
        case ESA_DTYPE_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
        case ESA_DTYPE_F32: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
        case ESA_DTYPE_F64: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT64; break;
        default: *err = "dtype"; return false;
    }
    const int es = dtype_size(dtype);
    const cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)T, (cuuint64_t)nb};
    const cuuint64_t strides[2] = {(cuuint64_t)(rs * es), (cuuint64_t)(T * rs * es)};
    const cuuint32_t box[3] = {(cuuint32_t)ws, (cuuint32_t)lt, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    promo_bytes >= 256   ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                    : promo_bytes >= 128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                    : promo_bytes >= 64  ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B
                                         : CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled error " + std::to_string((int)r);
        return false;
    }
    return true;
}

// ---------------------------------------------------------------------------
// Sequential fallback: one thread per channel, sequential over T.
// ---------------------------------------------------------------------------
namespace {

template <Kind K, typename Tin, typename Te>
__global__ void sequential_scan_kernel(const KArgs prm) {
    using P = Policy<K, Tin, Te>;
    using acc = typename P::acc;
    const int64_t ch = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= prm.nb * prm.hd) return;
    const int64_t b = ch / prm.hd, c = ch - b * prm.hd;
    const acc lo = acc(prm.gmin), span = acc(prm.span);
    auto ld = [&](int a, int64_t t, auto tag) -> acc {
        using T = decltype(tag);
        const T* p = reinterpret_cast<const T*>(prm.in[a].p) + (b * prm.T + t) * prm.in[a].rs + c;
        return static_cast<acc>(Elem<T>::to_acc(*p));
    };
    auto st = [&](int o, int64_t t, acc val, auto tag) {
        using T = decltype(tag);
        T* p = reinterpret_cast<T*>(prm.out[o].p) + (b * prm.T + t) * prm.out[o].rs + c;
        *p = Elem<T>::from_acc(static_cast<typename Elem<T>::acc>(val));
    };
    const acc e0v = prm.e0 ? static_cast<const acc*>(prm.e0)[ch] : acc(0);
    if constexpr (K == Kind::FwdSummary) {
        acc e = e0v, pr = acc(1);
        for (int64_t t = 0; t < prm.T; ++t) {
            const acc a = ld(0, t, Tin{});
            e = a * e + ld(1, t, Tin{});
            pr = pr * a;
        }
        if (prm.e_last) static_cast<acc*>(prm.e_last)[ch] = e;
        if (prm.prod_out) static_cast<acc*>(prm.prod_out)[ch] = pr;
    } else if constexpr (!P::REV) {
        acc e = e0v;
        for (int64_t t = 0; t < prm.T; ++t) {
            acc a, bb;
            if constexpr (K == Kind::FwdPlain) {
                a = ld(0, t, Tin{});
                bb = ld(1, t, Tin{});
            } else {
                a = lo + span * sigmoid_(ld(0, t, Tin{}));
                bb = (acc(1) - a) * tanh_(ld(1, t, Tin{}));
                if (prm.round_ab) {
                    a = round_to<Te>(a);
                    bb = round_to<Te>(bb);
                }
            }
            e = a * e + bb;
            st(0, t, e, Te{});
        }
        if (prm.e_last) static_cast<acc*>(prm.e_last)[ch] = e;
    } else {
        acc h = acc(0);
        for (int64_t t = prm.T - 1; t >= 0; --t) {
            if constexpr (K == Kind::RevPlain) {
                const acc a = ld(0, t, Te{});
                const acc d = ld(2, t, Te{});
                const acc ep = t > 0 ? ld(1, t - 1, Te{}) : e0v;
                const acc g = d + h;
                st(0, t, g * ep, Te{});
                st(1, t, g, Te{});
                h = a * g;
            } else {
                const acc sg = sigmoid_(ld(0, t, Tin{}));
                const acc A = lo + span * sg;
                const acc Ar = prm.round_ab ? round_to<Te>(A) : A;
                const acc V = tanh_(ld(1, t, Tin{}));
                const acc d = ld(3, t, Te{});
                const acc ep = t > 0 ? ld(2, t - 1, Te{}) : e0v;
                const acc g = d + h;
                st(0, t, (g * ep - g * V) * span * sg * (acc(1) - sg), Tin{});
                st(1, t, g * (acc(1) - A) * (acc(1) - V * V), Tin{});
                h = Ar * g;
            }
        }
        if (prm.e_last) static_cast<acc*>(prm.e_last)[ch] = h;
    }
}

template <Kind K, typename Tin, typename Te>
int seq_typed(const ScanCall& c) {
    const int threads = 256;
    const int64_t nch = c.a.nb * c.a.hd;
    const int64_t blocks = (nch + threads - 1) / threads;
    note_scan_path(ESA_PATH_SEQUENTIAL);
    sequential_scan_kernel<K, Tin, Te><<<(unsigned)blocks, threads, 0, c.stream>>>(c.a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("sequential scan launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

}  // namespace

int sequential_scan_launch(const ScanCall& c) {
    return dispatch_dtype(c.tin, [&](auto ti) -> int {
        using Tin = decltype(ti);
        return dispatch_dtype(c.te, [&](auto tee) -> int {
            using Te = decltype(tee);
            switch (c.kind) {
                case Kind::FwdPlain:
                    if constexpr (std::is_same<Tin, Te>::value) return seq_typed<Kind::FwdPlain, Tin, Te>(c);
                    break;
                case Kind::RevPlain:
                    if constexpr (std::is_same<Tin, Te>::value) return seq_typed<Kind::RevPlain, Tin, Te>(c);
                    break;
                case Kind::FwdSummary:
                    if constexpr (std::is_same<Tin, Te>::value) return seq_typed<Kind::FwdSummary, Tin, Te>(c);
                    break;
                case Kind::FwdGated: return seq_typed<Kind::FwdGated, Tin, Te>(c);
                case Kind::RevGated: return seq_typed<Kind::RevGated, Tin, Te>(c);
            }
            return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "plain scans need one dtype");
        });
    });
}

// ---------------------------------------------------------------------------
// Entry points behind the C ABI.
// ---------------------------------------------------------------------------
namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool rows_aligned(const void* p, int64_t rs, int64_t hd, int es) {
    return aligned16(p) && ((rs * es) % 16 == 0) && ((hd * es) % 16 == 0);
}

int check_dims(int64_t nb, int64_t T, int64_t hd, int compass) {
    if (nb < 0 || T < 0 || hd < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "negative dimension");
    if (compass <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "compass must be a positive integer");
    if (T > 0x7fffffffLL || nb > 0x7fffffffLL || hd > 0x7fffffffLL)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "dimension exceeds 2^31 - 1");
    return ESA_OK;
}

int run_split(ScanCall& c, bool* done);

int run(ScanCall& c) {
    if (c.a.nb == 0 || c.a.T == 0 || c.a.hd == 0) return ESA_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    c.a.status = status_ptr(dev);
    if (c.a.status == nullptr) return set_error(ESA_ERR_CUDA, "cannot resolve the device status word");
    if (!c.bulk_ok) return sequential_scan_launch(c);
    {
        bool chained = false;
        if (int rc = chain_scan_launch(c, &chained)) return rc;
        if (chained) return ESA_OK;
    }
    bool done = false;
    if (int rc = run_split(c, &done)) return rc;
    if (done) return ESA_OK;
    bool taken = false;
    const int rc = strip_scan_launch(c, &taken);
    if (rc != ESA_OK || taken) return rc;
    // the summary has no time-parallel form: one thread per channel
    if (c.kind == Kind::FwdSummary) return sequential_scan_launch(c);
    return lookback_scan_launch(c);
}

// ---- split scan -------------------------------------------------------------

struct SplitPlan {
    int64_t npiece = 1, plen = 0;
};

// Pieces per batch row for an [nb, T, hd] problem whose widest element has
// `wide_es` bytes: split when 128-channel-wide strips (16 lanes) number fewer
// than one per SM of a B200 and the time axis is long (>= 8192 steps; shorter
// problems measured faster unsplit: the extra summary pass does not pay).
// Aim at about 2400 strip-pieces (eight waves of 2 CTAs on 148 SMs, so the
// last wave's imbalance is small) with pieces of at least 1024 steps, a
// multiple of 64 steps (every strip tile length divides 64).

SplitPlan split_plan(int64_t nb, int64_t T, int64_t hd, int wide_es) {
    constexpr int min_t = 8192, target = 2400, min_piece = 1024;
    SplitPlan p;
    if (wide_es <= 0 || T < min_t) return p;
    const int64_t ws16 = 16 * (16 / wide_es);
    const int64_t strips16 = nb * ((hd + ws16 - 1) / ws16);
    if (strips16 <= 0 || strips16 >= 148) return p;
    int64_t n = (target + strips16 - 1) / strips16;
    // within 1/8 of that, the piece count whose strip-pieces fill whole waves
    // of 296 (2 CTAs on 148 SMs) best
    {
        int64_t best_n = n;
        double best_fill = 0.0;
        for (int64_t m = n - n / 8; m <= n + n / 8; ++m) {
            if (m < 2) continue;
            const int64_t items = strips16 * m;
            const double fill = (double)items / (double)(((items + 295) / 296) * 296);
            if (fill > best_fill + 1e-9) {
                best_fill = fill;
                best_n = m;
            }
        }
        n = best_n;
    }
    if (n > T / min_piece) n = T / min_piece;
    if (n < 2) return p;
    const int64_t plen = ((T + n - 1) / n + 63) / 64 * 64;
    p.npiece = (T + plen - 1) / plen;
    p.plen = plen;
    if (p.npiece < 2) p.npiece = 1;
    return p;
}

size_t split_plane_bytes(int64_t nb, const SplitPlan& p, int64_t hd, size_t acc_size) {
    return ((size_t)(nb * p.npiece * hd) * acc_size + 255) / 256 * 256;
}

// Incoming state of every (batch row, piece) from the pieces' summaries, in
// time order (reverse kinds: descending), one thread per channel; the state
// after the last piece goes to e_last, the product over all pieces to
// prod_total (either may be null).
template <typename acc>
__global__ void compose_pieces_kernel(const acc* __restrict__ prod, const acc* __restrict__ endst,
                                      const acc* __restrict__ e0, acc* __restrict__ cin,
                                      acc* __restrict__ e_last, acc* __restrict__ prod_total,
                                      int64_t nb, int64_t npiece, int64_t hd, int rev) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nb * hd) return;
    const int64_t b = idx / hd, ch = idx - b * hd;
    acc st = (e0 != nullptr && !rev) ? e0[idx] : acc(0);
    acc pr = acc(1);
    for (int64_t q = 0; q < npiece; ++q) {
        const int64_t p = rev ? npiece - 1 - q : q;
        const int64_t o = (b * npiece + p) * hd + ch;
        cin[o] = st;
        const acc a = prod[o];
        st = a * st + endst[o];
        pr = pr * a;
    }
    if (e_last != nullptr) e_last[idx] = st;
    if (prod_total != nullptr) prod_total[idx] = pr;
}

int wide_size(const ScanCall& c) {
    const int a = dtype_size(c.tin), b = dtype_size(c.te);
    return a > b ? a : b;
}

// The split scan for few-channel, long problems; *done = false (nothing
// launched) when the problem is not split or the workspace is too small.
int run_split(ScanCall& c, bool* done) {
    *done = false;
    const int wes = wide_size(c);
    const SplitPlan sp = split_plan(c.a.nb, c.a.T, c.a.hd, wes);
    if (sp.npiece < 2) return ESA_OK;
    const size_t acc_size = wes == 8 ? 8 : 4;
    const size_t plane = split_plane_bytes(c.a.nb, sp, c.a.hd, acc_size);
    if (c.ws == nullptr || c.ws_bytes < 3 * plane || (reinterpret_cast<uintptr_t>(c.ws) & 255u)) return ESA_OK;
    char* ws = static_cast<char*>(c.ws);
    void* prod = ws;
    void* endst = ws + plane;
    void* cin = ws + 2 * plane;
    const bool rev = c.kind == Kind::RevPlain || c.kind == Kind::RevGated;

    // pass 1: summaries of every piece from a zero state (already in the
    // workspace when resuming after a summary call on the same inputs)
    if (!c.resume) {
        ScanCall c1 = c;
        c1.npiece = sp.npiece;
        c1.plen = sp.plen;
        c1.summ = true;
        c1.a.e0 = nullptr;
        c1.a.cin = nullptr;
        c1.a.e_last = endst;
        c1.a.prod_out = prod;
        c1.ws = nullptr;
        c1.ws_bytes = 0;
        bool taken = false;
        if (int rc = strip_scan_launch(c1, &taken)) return rc;
        if (!taken) return ESA_OK;
    }
    // pass 2: incoming states in time order
    const int64_t n = c.a.nb * c.a.hd;
    const int threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    const bool summary = c.kind == Kind::FwdSummary;
    if (acc_size == 8) {
        compose_pieces_kernel<double><<<blocks, threads, 0, c.stream>>>(
            static_cast<const double*>(prod), static_cast<const double*>(endst),
            static_cast<const double*>(rev ? nullptr : c.a.e0), static_cast<double*>(cin),
            static_cast<double*>(c.a.e_last), static_cast<double*>(summary ? c.a.prod_out : nullptr),
            c.a.nb, sp.npiece, c.a.hd, rev ? 1 : 0);
    } else {
        compose_pieces_kernel<float><<<blocks, threads, 0, c.stream>>>(
            static_cast<const float*>(prod), static_cast<const float*>(endst),
            static_cast<const float*>(rev ? nullptr : c.a.e0), static_cast<float*>(cin),
            static_cast<float*>(c.a.e_last), static_cast<float*>(summary ? c.a.prod_out : nullptr),
            c.a.nb, sp.npiece, c.a.hd, rev ? 1 : 0);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("piece composition: ") + cudaGetErrorString(e));
    *done = true;
    if (summary) return ESA_OK;
    // pass 3: outputs from each piece's exact incoming state
    ScanCall c3 = c;
    c3.npiece = sp.npiece;
    c3.plen = sp.plen;
    c3.a.cin = cin;
    c3.a.e_last = nullptr;
    c3.ws = nullptr;
    c3.ws_bytes = 0;
    bool taken3 = false;
    if (int rc = strip_scan_launch(c3, &taken3)) return rc;
    if (!taken3) return set_error(ESA_ERR_CUDA, "split scan: output pass not launched");
    return ESA_OK;
}

}  // namespace

size_t scan_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass) {
    const size_t lb = lookback_workspace_bytes(nb, T, hd, wide_es, compass);
    const SplitPlan sp = split_plan(nb, T, hd, wide_es);
    const size_t split = sp.npiece > 1 ? 3 * split_plane_bytes(nb, sp, hd, wide_es == 8 ? 8 : 4) : 0;
    const size_t chain = chain_workspace_bytes(nb, T, hd, wide_es);
    const size_t m = lb > split ? lb : split;
    return m > chain ? m : chain;
}

int scan_fwd(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd, int dtype,
             int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes, cudaStream_t s,
             bool resume) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    if (nb * T * hd > 0 && (!A || !B || !E)) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    ScanCall c{};
    c.kind = Kind::FwdPlain;
    c.tin = c.te = dtype;
    c.a.in[0] = {static_cast<const char*>(A), hd};
    c.a.in[1] = {static_cast<const char*>(B), hd};
    c.a.out[0] = {static_cast<char*>(E), hd};
    c.a.nb = nb;
    c.a.T = T;
    c.a.hd = hd;
    c.a.e0 = e0;
    c.a.e_last = e_last;
    c.compass = compass;
    c.ws = ws;
    c.ws_bytes = ws_bytes;
    c.stream = s;
    c.bulk_ok = rows_aligned(A, hd, hd, es) && rows_aligned(B, hd, hd, es) && rows_aligned(E, hd, hd, es);
    c.resume = resume;
    return run(c);
}

int scan_summary(const void* A, const void* B, int64_t nb, int64_t T, int64_t hd, int dtype,
                 const void* e0, void* e_last, void* prod, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, 16)) return rc;
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    if (nb * T * hd > 0 && (!A || !B)) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (nb * hd > 0 && (!e_last || !prod)) return set_error(ESA_ERR_INVALID_ARGUMENT, "null output pointer");
    ScanCall c{};
    c.kind = Kind::FwdSummary;
    c.tin = c.te = dtype;
    c.a.in[0] = {static_cast<const char*>(A), hd};
    c.a.in[1] = {static_cast<const char*>(B), hd};
    c.a.nb = nb;
    c.a.T = T;
    c.a.hd = hd;
    c.a.e0 = e0;
    c.a.e_last = e_last;
    c.a.prod_out = prod;
    c.compass = 16;
    c.ws = ws;
    c.ws_bytes = ws_bytes;
    c.stream = s;
    c.bulk_ok = rows_aligned(A, hd, hd, es) && rows_aligned(B, hd, hd, es);
    return run(c);
}

int scan_rev(const void* A, const void* E, const void* dE, void* dA, void* dB, int64_t nb, int64_t T,
             int64_t hd, int dtype, int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
             cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    if (nb * T * hd > 0 && (!A || !E || !dE || !dA || !dB))
        return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    ScanCall c{};
    c.kind = Kind::RevPlain;
    c.tin = c.te = dtype;
    c.a.in[0] = {static_cast<const char*>(A), hd};
    c.a.in[1] = {static_cast<const char*>(E), hd};
    c.a.in[2] = {static_cast<const char*>(dE), hd};
    c.a.out[0] = {static_cast<char*>(dA), hd};
    c.a.out[1] = {static_cast<char*>(dB), hd};
    c.a.nb = nb;
    c.a.T = T;
    c.a.hd = hd;
    c.a.e0 = e0;
    c.a.e_last = de0;
    c.compass = compass;
    c.ws = ws;
    c.ws_bytes = ws_bytes;
    c.stream = s;
    c.bulk_ok = rows_aligned(A, hd, hd, es) && rows_aligned(E, hd, hd, es) && rows_aligned(dE, hd, hd, es) &&
                rows_aligned(dA, hd, hd, es) && rows_aligned(dB, hd, hd, es);
    return run(c);
}

int gated_scan_fwd(const void* g, const void* v, int64_t rrs, int raw_dtype, void* E, int e_dtype,
                   int64_t nb, int64_t T, int64_t hd, double gmin, double gmax, int round_ab,
                   int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    const int ei = dtype_size(raw_dtype), ee = dtype_size(e_dtype);
    if (ei == 0 || ee == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code");
    if (nb * T * hd > 0 && (!g || !v || !E)) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (rrs < hd) return set_error(ESA_ERR_INVALID_ARGUMENT, "raw_row_stride smaller than hd");
    ScanCall c{};
    c.kind = Kind::FwdGated;
    c.tin = raw_dtype;
    c.te = e_dtype;
    c.a.in[0] = {static_cast<const char*>(g), rrs};
    c.a.in[1] = {static_cast<const char*>(v), rrs};
    c.a.out[0] = {static_cast<char*>(E), hd};
    c.a.nb = nb;
    c.a.T = T;
    c.a.hd = hd;
    c.a.e0 = e0;
    c.a.e_last = e_last;
    c.a.gmin = gmin;
    c.a.span = gmax - gmin;
    c.a.round_ab = round_ab;
    c.compass = compass;
    c.ws = ws;
    c.ws_bytes = ws_bytes;
    c.stream = s;
    c.bulk_ok = rows_aligned(g, rrs, hd, ei) && rows_aligned(v, rrs, hd, ei) && rows_aligned(E, hd, hd, ee);
    return run(c);
}

int gated_scan_bwd(const void* g, const void* v, int64_t rrs, int raw_dtype, const void* E,
                   const void* dE, int e_dtype, void* dg, void* dv, int64_t drs, int draw_dtype,
                   int64_t nb, int64_t T, int64_t hd, double gmin, double gmax, int round_ab,
                   int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    const int ei = dtype_size(raw_dtype), ee = dtype_size(e_dtype);
    if (ei == 0 || ee == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code");
    if (nb * T * hd > 0 && (!g || !v || !E || !dE || !dg || !dv))
        return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (rrs < hd || drs < hd) return set_error(ESA_ERR_INVALID_ARGUMENT, "row stride smaller than hd");
    if (draw_dtype != raw_dtype)
        return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "d_gate_raw/d_value_raw must have the dtype of gate_raw/value_raw");
    ScanCall c{};
    c.kind = Kind::RevGated;
    c.tin = raw_dtype;
    c.te = e_dtype;
    c.a.in[0] = {static_cast<const char*>(g), rrs};
    c.a.in[1] = {static_cast<const char*>(v), rrs};
    c.a.in[2] = {static_cast<const char*>(E), hd};
    c.a.in[3] = {static_cast<const char*>(dE), hd};
    c.a.out[0] = {static_cast<char*>(dg), drs};
    c.a.out[1] = {static_cast<char*>(dv), drs};
    c.a.nb = nb;
    c.a.T = T;
    c.a.hd = hd;
    c.a.e0 = e0;
    c.a.e_last = de0;
    c.a.gmin = gmin;
    c.a.span = gmax - gmin;
    c.a.round_ab = round_ab;
    c.compass = compass;
    c.ws = ws;
    c.ws_bytes = ws_bytes;
    c.stream = s;
    c.bulk_ok = rows_aligned(g, rrs, hd, ei) && rows_aligned(v, rrs, hd, ei) && rows_aligned(E, hd, hd, ee) &&
                rows_aligned(dE, hd, hd, ee) && rows_aligned(dg, drs, hd, ei) && rows_aligned(dv, drs, hd, ei);
    return run(c);
}

}  // namespace esa
