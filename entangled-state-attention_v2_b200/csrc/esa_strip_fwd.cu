// esa_strip_fwd.cu -- strip scan instantiations: forward scan of materialised A, B.
#include "esa_strip.cuh"

namespace esa {

int strip_fwd_plain(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        // steps per row group for strips of 4/8/16/32 lanes: 64-step tiles (32 at 512 B rows)
        return strip_launch_kind<Kind::FwdPlain, T, T, 1, 2, 4, 4>(c, taken);
    });
}

int strip_fwd_summary(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return strip_launch_kind<Kind::FwdSummary, T, T, 1, 2, 4, 4>(c, taken);
    });
}

}  // namespace esa
