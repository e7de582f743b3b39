// esa_lane_plain.cu -- lane-serial scan instantiations: forward scan of
// materialised A, B, its summary pass, and the reverse scan (gradient of A, B).
#include "esa_lane.cuh"

namespace esa {

int lane_fwd_plain(const ScanCall& c, bool* taken, double min_warps) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return lane_launch_kind<Kind::FwdPlain, T, T>(c, taken, min_warps);
    });
}

int lane_fwd_summary(const ScanCall& c, bool* taken, double min_warps) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return lane_launch_kind<Kind::FwdSummary, T, T>(c, taken, min_warps);
    });
}

int lane_rev_plain(const ScanCall& c, bool* taken, double min_warps) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        if (c.summ) return lane_launch_kind<Kind::RevPlain, T, T, true>(c, taken, min_warps);
        return lane_launch_kind<Kind::RevPlain, T, T>(c, taken, min_warps);
    });
}

}  // namespace esa
