// esa_strip_rev.cu -- strip scan instantiations: reverse scan (gradient of A, B).
#include "esa_strip.cuh"

namespace esa {

// steps per row group for strips of 4/8/16/32 lanes
constexpr int kRevSr4 = 1;
constexpr int kRevSr8 = 2;
constexpr int kRevSr16 = 2;  // measured: 5.54 vs 5.45 TB/s on the [32,4096,16,64] fp16 reverse, no spill
constexpr int kRevSr32 = 2;  // measured: 6.2 vs 5.8 TB/s on the [32,4096,16,64] fp32 reverse

// 16-bit data: the narrow form, 128-channel strips of 32 four-channel lanes
// with four steps a thread (32-step tiles); measured 6.07 vs 5.59 TB/s on the
// [32,4096,16,64] fp16 reverse against 8-channel lanes in row-group pairs.
// fp32 keeps the wide form (6.21 vs 5.87 TB/s).
constexpr int kRevNarrowSteps = 4;
constexpr int kRevNarrowVec = 4;

int strip_rev_plain(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        if constexpr (sizeof(T) == 2)
            return strip_launch_kind<Kind::RevPlain, T, T, kRevSr4, kRevSr8, kRevSr16, kRevSr32, false,
                                     kRevNarrowSteps, kRevNarrowVec>(c, taken);
        else
            return strip_launch_kind<Kind::RevPlain, T, T, kRevSr4, kRevSr8, kRevSr16, kRevSr32>(c, taken);
    });
}

}  // namespace esa
