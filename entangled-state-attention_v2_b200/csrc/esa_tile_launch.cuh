// esa_tile_launch.cuh -- host side of the row-tile layer kernels: the launch
// description and the typed launcher (tensor maps, shared-memory opt-in,
// grid) that the esa_tile_*.cu units instantiate.
#pragma once

#include <cstring>
#include <string>

#include "esa_tile.cuh"

namespace esa {

// One launch: kernel arguments plus the staged inputs (base pointer, row
// stride in elements, dtype code) in the kernel's array order.
struct TileLaunch {
    TileArgs a;
    const void* in[5];
    int64_t in_rs[5];
    int in_dt[5];
    cudaStream_t stream;
};

template <bool REV, bool RO, typename Tr, typename Te, typename Ty, int V, int LT>
int tile_occupancy(size_t smem, int threads) {
    auto kern = tile_layer_kernel<REV, RO, Tr, Te, Ty, V, LT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess) return 0;
    return per_sm;
}

template <bool REV, bool RO, typename Tr, typename Te, typename Ty, int V, int LT>
int tile_launch_typed(const TileLaunch& L) {
    using Cfg = TileCfg<REV, RO, Tr, Te, Ty, V, LT>;
    const TileArgs& a = L.a;
    CUtensorMap maps[5];
    memset(maps, 0, sizeof(maps));
    for (int i = 0; i < Cfg::NARR; ++i) {
        if (!Cfg::HAS(i)) continue;
        std::string err;
        const int row_bytes = a.wb * dtype_size(L.in_dt[i]);
        if (!encode_strip_map(&maps[i], L.in_dt[i], L.in[i], a.nb, a.T, a.C, L.in_rs[i], a.wb, Cfg::rows(i), &err,
                              row_bytes >= 256 ? 256 : row_bytes))
            return set_error(ESA_ERR_CUDA, "tile tensor map: " + err);
    }
    const size_t smem = (size_t)a.nstage * a.stage_bytes + Cfg::tail_bytes();
    const int threads = 32 * (a.nwc + 1);
    int dev = 0;
    cudaGetDevice(&dev);
    const int occ = tile_occupancy<REV, RO, Tr, Te, Ty, V, LT>(smem, threads);
    if (occ <= 0) return set_error(ESA_ERR_CUDA, "row-tile kernel: no residency for this configuration");
    int64_t grid = (int64_t)occ * device_sm_count(dev);
    if (grid > a.ntiles) grid = a.ntiles;
    tile_layer_kernel<REV, RO, Tr, Te, Ty, V, LT><<<(unsigned)grid, threads, smem, L.stream>>>(
        a, maps[0], maps[1], maps[2], maps[3], maps[4]);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("row-tile launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

// Launch of one kind (forward / backward, with or without the readout) for
// element types (tr, te, ty) and lane width / tile length (v, lt);
// ESA_ERR_UNSUPPORTED_DTYPE when not instantiated (esa_tile_*.cu).
int tile_launch_fwd_ro(int tr, int te, int ty, int v, int lt, const TileLaunch& L);
int tile_launch_fwd_plain(int tr, int te, int ty, int v, int lt, const TileLaunch& L);
int tile_launch_rev_ro(int tr, int te, int ty, int v, int lt, const TileLaunch& L);
int tile_launch_rev_plain(int tr, int te, int ty, int v, int lt, const TileLaunch& L);

}  // namespace esa
