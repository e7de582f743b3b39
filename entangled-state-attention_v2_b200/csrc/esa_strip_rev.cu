// esa_strip_rev.cu -- strip scan instantiations: reverse scan (gradient of A, B).
#include "esa_strip.cuh"

// steps per row group for strips of 4/8/16/32 lanes (build-time overrides
// for tuning sweeps)
#ifndef ESA_REV_SR4
#define ESA_REV_SR4 1
#define ESA_REV_SR8 2
#define ESA_REV_SR16 2  // measured: 5.54 vs 5.45 TB/s on the [32,4096,16,64] fp16 reverse, no spill
#define ESA_REV_SR32 2  // measured: 6.2 vs 5.8 TB/s on the [32,4096,16,64] fp32 reverse
#endif

namespace esa {

int strip_rev_plain(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return strip_launch_kind<Kind::RevPlain, T, T, ESA_REV_SR4, ESA_REV_SR8, ESA_REV_SR16,
                                 ESA_REV_SR32>(c, taken);
    });
}

}  // namespace esa
