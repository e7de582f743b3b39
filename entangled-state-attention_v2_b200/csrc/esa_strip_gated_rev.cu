// esa_strip_gated_rev.cu -- strip scan instantiations: reverse scan with the
// gate chain rule fused (d gate_raw, d value_raw out).  Same dtype pairs as
// the fused forward; other pairs use the lookback kernel.
#include "esa_strip.cuh"

namespace esa {

namespace {
// steps a thread in the narrow form: 64-step tiles (four staged arrays, 32 KB
// a 16-bit stage)
constexpr int kNarrowSteps = 8;

template <typename Tin, typename Te>
int go(const ScanCall& c, bool* taken) {
    return strip_launch_kind<Kind::RevGated, Tin, Te, 1, 2, 2, 2, false, kNarrowSteps>(c, taken);
}
}  // namespace

int strip_rev_gated(const ScanCall& c, bool* taken) {
    *taken = false;
    const int ti = c.tin, te = c.te;
    if (ti == te) {
        return dispatch_dtype(ti, [&](auto tag) -> int {
            using T = decltype(tag);
            return go<T, T>(c, taken);
        });
    }
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_F16) return go<float, __half>(c, taken);
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_BF16) return go<float, __nv_bfloat16>(c, taken);
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_F64) return go<float, double>(c, taken);
    if (ti == ESA_DTYPE_F16 && te == ESA_DTYPE_F32) return go<__half, float>(c, taken);
    if (ti == ESA_DTYPE_BF16 && te == ESA_DTYPE_F32) return go<__nv_bfloat16, float>(c, taken);
    return ESA_OK;
}

}  // namespace esa
