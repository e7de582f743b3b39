// esa_strip_fwd.cu -- strip scan instantiations: forward scan of materialised A, B.
#include "esa_strip.cuh"

// steps per row group for strips of 4/8/16/32 lanes (build-time overrides
// for tuning sweeps)
#ifndef ESA_FWD_SR4
#define ESA_FWD_SR4 1
#define ESA_FWD_SR8 2
#define ESA_FWD_SR16 4
#define ESA_FWD_SR32 4
#endif

namespace esa {

int strip_fwd_plain(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        // steps per row group for strips of 4/8/16/32 lanes: 64-step tiles (32 at 512 B rows)
        return strip_launch_kind<Kind::FwdPlain, T, T, ESA_FWD_SR4, ESA_FWD_SR8, ESA_FWD_SR16,
                                 ESA_FWD_SR32>(c, taken);
    });
}

int strip_fwd_summary(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return strip_launch_kind<Kind::FwdSummary, T, T, 1, 2, 4, 4>(c, taken);
    });
}

}  // namespace esa
