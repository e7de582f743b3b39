// esa_tile_fwd_plain.cu -- instantiations of the row-tile layer kernel, forward
// without the readout (the bare gated scan), for the dtype mixes the ESA layer runs in:
// 16-bit throughout (the autocast layer), fp32 throughout, and fp32
// activations with a 16-bit scan (precision "fp16" / "bf16" with fp32
// inputs).  One unit per kind, so that nvcc compiles them in parallel.
#include "esa_tile_launch.cuh"

namespace esa {

#define ESA_TILE_VL(TR, TE, TY)                                                          \
    if (v == 2 && lt == 16) return tile_launch_typed<false, false, TR, TE, TY, 2, 16>(L); \
    if (v == 2 && lt == 8) return tile_launch_typed<false, false, TR, TE, TY, 2, 8>(L);   \
    if (v == 4 && lt == 8) return tile_launch_typed<false, false, TR, TE, TY, 4, 8>(L);   \
    return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "row-tile kernel: lane width / tile length not built");

int tile_launch_fwd_plain(int tr, int te, int ty, int v, int lt, const TileLaunch& L) {
    (void)ty;
    if (tr == ESA_DTYPE_F16 && te == ESA_DTYPE_F16) { ESA_TILE_VL(__half, __half, __half) }
    if (tr == ESA_DTYPE_BF16 && te == ESA_DTYPE_BF16) { ESA_TILE_VL(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16) }
    if (tr == ESA_DTYPE_F32 && te == ESA_DTYPE_F32) { ESA_TILE_VL(float, float, float) }
    if (tr == ESA_DTYPE_F32 && te == ESA_DTYPE_F16) { ESA_TILE_VL(float, __half, __half) }
    if (tr == ESA_DTYPE_F32 && te == ESA_DTYPE_BF16) { ESA_TILE_VL(float, __nv_bfloat16, __nv_bfloat16) }
    return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "row-tile kernel: dtype mix not built");
}

}  // namespace esa
