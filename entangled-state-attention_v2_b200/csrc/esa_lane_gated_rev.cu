// esa_lane_gated_rev.cu -- lane-serial scan instantiations: reverse scan with
// the gate chain rule fused (d gate_raw, d value_raw out), and its summary
// pass.
// The (logit dtype, scan dtype) pairs of the strip scan's fused kernels;
// other pairs are not taken.
#include "esa_lane.cuh"

namespace esa {

namespace {
template <typename Tin, typename Te>
int go(const ScanCall& c, bool* taken, double min_warps) {
    if (c.summ) return lane_launch_kind<Kind::RevGated, Tin, Te, true>(c, taken, min_warps);
    return lane_launch_kind<Kind::RevGated, Tin, Te>(c, taken, min_warps);
}
}  // namespace

int lane_rev_gated(const ScanCall& c, bool* taken, double min_warps) {
    *taken = false;
    const int ti = c.tin, te = c.te;
    if (ti == te) {
        return dispatch_dtype(ti, [&](auto tag) -> int {
            using T = decltype(tag);
            return go<T, T>(c, taken, min_warps);
        });
    }
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_F16) return go<float, __half>(c, taken, min_warps);
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_BF16) return go<float, __nv_bfloat16>(c, taken, min_warps);
    if (ti == ESA_DTYPE_F32 && te == ESA_DTYPE_F64) return go<float, double>(c, taken, min_warps);
    if (ti == ESA_DTYPE_F16 && te == ESA_DTYPE_F32) return go<__half, float>(c, taken, min_warps);
    if (ti == ESA_DTYPE_BF16 && te == ESA_DTYPE_F32) return go<__nv_bfloat16, float>(c, taken, min_warps);
    return ESA_OK;
}

}  // namespace esa
