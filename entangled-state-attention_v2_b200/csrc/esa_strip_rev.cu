// esa_strip_rev.cu -- strip scan instantiations: reverse scan (gradient of A, B).
#include "esa_strip.cuh"

namespace esa {

// steps per row group for strips of 4/8/16/32 lanes
constexpr int kRevSr4 = 1;
constexpr int kRevSr8 = 2;
constexpr int kRevSr16 = 2;  // measured: 5.54 vs 5.45 TB/s on the [32,4096,16,64] fp16 reverse, no spill
constexpr int kRevSr32 = 2;  // measured: 6.2 vs 5.8 TB/s on the [32,4096,16,64] fp32 reverse

int strip_rev_plain(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return strip_launch_kind<Kind::RevPlain, T, T, kRevSr4, kRevSr8, kRevSr16, kRevSr32>(c, taken);
    });
}

}  // namespace esa
