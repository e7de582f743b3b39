// esa_strip_rev.cu -- strip scan instantiations: reverse scan (gradient of A, B).
#include "esa_strip.cuh"

namespace esa {

int strip_rev_plain(const ScanCall& c, bool* taken) {
    return dispatch_dtype(c.te, [&](auto tag) -> int {
        using T = decltype(tag);
        return strip_launch_kind<Kind::RevPlain, T, T, 1, 2, 4, 4>(c, taken);
    });
}

}  // namespace esa
