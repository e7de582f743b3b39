// esa_strip_summ.cu -- strip scan instantiations: summary passes of the split
// (time-pieced) scans.  Per (batch row, piece): the end state from the
// piece's incoming state and the product of the step coefficients, no
// per-step outputs.  Forward plain uses the FwdSummary kind (esa_strip_fwd.cu).
#include "esa_strip.cuh"

namespace esa {

namespace {
template <typename Tin, typename Te>
int fwd_gated(const ScanCall& c, bool* taken) {
    return strip_launch_kind<Kind::FwdGated, Tin, Te, 1, 2, 2, 2, true>(c, taken);
}
template <typename Tin, typename Te>
int rev_gated(const ScanCall& c, bool* taken) {
    return strip_launch_kind<Kind::RevGated, Tin, Te, 1, 2, 2, 2, true>(c, taken);
}

// the (logit dtype, scan dtype) pairs of the fused kernels
template <template <typename, typename> class F>
int gated_pairs(const ScanCall& c, bool* taken) {
    const int ti = c.tin, te = c.te;
    if (ti == te)
        return dispatch_dtype(ti, [&](auto tag) -> int {
            using T = decltype(tag);
            return F<T, T>::run(c, taken);
        });
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_F16) return F<float, __half>::run(c, taken);
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_BF16) return F<float, __nv_bfloat16>::run(c, taken);
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_F64) return F<float, double>::run(c, taken);
    if (ti == ESA_DTYPE_F16 && te == ESA_DTYPE_F32) return F<__half, float>::run(c, taken);
    if (ti == ESA_DTYPE_BF16 && te == ESA_DTYPE_F32) return F<__nv_bfloat16, float>::run(c, taken);
    *taken = false;
    return ESA_OK;
}
template <typename Tin, typename Te>
struct FwdGatedSumm {
    static int run(const ScanCall& c, bool* taken) { return fwd_gated<Tin, Te>(c, taken); }
};
template <typename Tin, typename Te>
struct RevGatedSumm {
    static int run(const ScanCall& c, bool* taken) { return rev_gated<Tin, Te>(c, taken); }
};
}  // namespace

int strip_fwd_summary(const ScanCall& c, bool* taken);

int strip_summary_launch(const ScanCall& c, bool* taken) {
    *taken = false;
    switch (c.kind) {
        case Kind::FwdPlain:
        case Kind::FwdSummary:
            return strip_fwd_summary(c, taken);
        case Kind::RevPlain:
            return dispatch_dtype(c.te, [&](auto tag) -> int {
                using T = decltype(tag);
                return strip_launch_kind<Kind::RevPlain, T, T, 1, 2, 4, 4, true>(c, taken);
            });
        case Kind::FwdGated: return gated_pairs<FwdGatedSumm>(c, taken);
        case Kind::RevGated: return gated_pairs<RevGatedSumm>(c, taken);
    }
    return ESA_OK;
}

}  // namespace esa
