// esa_strip_gated.cu -- strip scan instantiations: forward scan with the gate
// prologue fused (logits in, E out).  The (logit dtype, scan dtype) pairs a
// layer produces: same dtype, fp32 logits with a 16-bit or fp64 scan, 16-bit
// logits (autocast) with an fp32 scan.  Other pairs use the lookback kernel.
#include "esa_strip.cuh"

namespace esa {

namespace {
// steps a thread in the narrow form: 128-step tiles; its A, B register cache
// holds 16 x 2 x 2 values
constexpr int kNarrowSteps = 16;

template <typename Tin, typename Te>
int go(const ScanCall& c, bool* taken) {
    // wide form: two steps per row group keep the A/B register cache at
    // 2*VEC*2 values
    return strip_launch_kind<Kind::FwdGated, Tin, Te, 1, 2, 2, 2, false, kNarrowSteps>(c, taken);
}
}  // namespace

int strip_fwd_gated(const ScanCall& c, bool* taken) {
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
