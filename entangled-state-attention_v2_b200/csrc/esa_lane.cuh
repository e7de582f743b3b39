// esa_lane.cuh -- lane-serial strip scan: every lane runs the recurrence of
// its own channels step by step over the whole time axis.
//
// The strip scan (esa_strip.cuh) spreads a tile's steps over the threads of a
// CTA and stitches them together with shuffles, shared-memory exchanges and
// two CTA barriers per tile: about 17 instructions per element on the
// [32, 4096, 16, 64] fp16 forward.  When the problem has enough channels
// (32768 there), the time axis needs no parallel split at all: a lane that
// owns V channels and walks the steps in order does one FMA per element per
// step, and the work per element drops to its loads, conversions, FMA and
// store (about 5 instructions).  A warp of such lanes covers 32*V channels
// (128-byte rows: V = 2 for 16-bit data, 1 for 32- and 64-bit data).
//
// CTA = NW consumer warps (a strip of WS = 32*V*NW channels of one batch
// row) + one producer warp.  The producer's lane 0 walks the CTA's items and
// tiles in the consumers' order and issues 3-D tiled TMA loads (box
// [1, LT, WS], L2 evict-first) into an NSTAGE-deep ring of shared-memory
// stages: a "full" mbarrier per stage completes on the copy bytes, an
// "empty" mbarrier per stage on one arrival per consumer warp.  The ring
// runs on across the CTA's items without draining.  Consumers wait on full,
// run the tile's LT steps from registers (forward: ascending time; reverse:
// descending), store outputs with coalesced 4-byte (8 for fp64) stores, and
// release the stage.  There are no CTA-wide barriers after the setup.
//
// Items, pieces, incoming states (KArgs::cin), summaries (SUMM) and the
// final state follow the strip scan's contract exactly (StripParams), so the
// two are interchangeable behind strip_scan_launch.
#pragma once

#include <atomic>

#include "esa_strip.cuh"

namespace esa {

// Policy with a lane vector of V channels (the per-step helpers step_coef /
// step_apply take their vector width and register cache from it).
template <Kind K, typename Tin, typename Te, int V>
struct LanePolicy : Policy<K, Tin, Te> {
    using acc = typename Policy<K, Tin, Te>::acc;
    static constexpr int VEC = V;
    template <int S>
    struct Cache {
        acc c0[S][V];
        acc c1[S][V];
    };
};

template <Kind K, typename Tin, typename Te, int NW_>
struct LaneCfg {
    using Base = Policy<K, Tin, Te>;
    // 4-byte lane vectors for 16-bit data (128-byte warp rows), one channel
    // per lane otherwise
    static constexpr int V = Base::WIDE == 2 ? 2 : 1;
    using P = LanePolicy<K, Tin, Te, V>;
    static constexpr int NW = NW_;            // consumer warps
    static constexpr int NT = 32 * (NW + 1);  // + the producer warp
    static constexpr int LT = 32;             // steps per tile
    static constexpr int WS = 32 * V * NW;    // channels per strip
    static __host__ __device__ constexpr int row_bytes(int a) { return WS * P::es(a); }
    static __host__ __device__ constexpr int array_off(int a) {
        int o = 0;
        for (int i = 0; i < a; ++i) o += LT * row_bytes(i);
        return o;
    }
    static __host__ __device__ constexpr int stage_bytes() { return array_off(P::NIN); }
    static size_t smem_bytes(int nstage) { return (size_t)nstage * (stage_bytes() + 2 * sizeof(uint64_t)) + 128; }
};

template <Kind K, typename Tin, typename Te, int NW, bool SUMM_>
__global__ void __launch_bounds__(32 * (NW + 1)) lane_scan_kernel(const StripParams prm,
                                                                  const __grid_constant__ CUtensorMap m0,
                                                                  const __grid_constant__ CUtensorMap m1,
                                                                  const __grid_constant__ CUtensorMap m2,
                                                                  const __grid_constant__ CUtensorMap m3) {
    using Cfg = LaneCfg<K, Tin, Te, NW>;
    using P = typename Cfg::P;
    using acc = typename P::acc;
    constexpr int V = Cfg::V;
    constexpr int WS = Cfg::WS;
    constexpr int LT = Cfg::LT;
    constexpr bool SUMM = SUMM_ || K == Kind::FwdSummary;
    const KArgs& ka = prm.a;
    const int nstage = prm.nstage;

    extern __shared__ __align__(128) char smem_raw[];
    char* smem = smem_raw + ((128u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 127u)) & 127u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nstage * Cfg::stage_bytes());
    uint64_t* empty = full + nstage;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbarrier_init();
    }
    __syncthreads();

    struct ItemGeom {
        int64_t row, strip, b, pbeg, pend, ntt;
    };
    auto geom = [&](int64_t it) {
        ItemGeom g;
        g.row = it / prm.spr;
        g.strip = it - g.row * prm.spr;
        g.b = g.row / prm.npiece;
        g.pbeg = (g.row - g.b * prm.npiece) * prm.plen;
        g.pend = g.pbeg + prm.plen < ka.T ? g.pbeg + prm.plen : ka.T;
        g.ntt = (g.pend - g.pbeg + LT - 1) / LT;
        return g;
    };
    auto tile_t0 = [&](const ItemGeom& g, int64_t j) -> int64_t {
        return g.pbeg + (P::REV ? (g.ntt - 1 - j) : j) * (int64_t)LT;
    };

    if (warp == NW) {
        // ---- producer: lane 0 fills the ring in consumption order ----------
        if (lane != 0) return;
        const CUtensorMap* maps[4] = {&m0, &m1, &m2, &m3};
        const uint64_t policy = policy_evict_first();
        uint64_t fills = 0;
        int slot = 0;
        unsigned rnd = 0;  // fills of `slot` before this one
        bool ok = true;
        for (int64_t item = blockIdx.x; item < prm.nitems && ok; item += gridDim.x) {
            const ItemGeom g = geom(item);
            for (int64_t j = 0; j < g.ntt; ++j) {
                // the stage's previous tile released by every consumer warp
                if (rnd > 0 && !mbar_wait_bounded(&empty[slot], (rnd - 1) & 1u, ka.status)) {
                    ok = false;
                    break;
                }
                char* stage = smem + (size_t)slot * Cfg::stage_bytes();
                mbar_arrive_expect_tx(&full[slot], (unsigned)Cfg::stage_bytes());
#pragma unroll
                for (int a = 0; a < P::NIN; ++a)
                    tma_load_3d(stage + Cfg::array_off(a), maps[a], (int)(g.strip * WS),
                                (int)(tile_t0(g, j) + P::shift(a)), (int)g.b, &full[slot], policy);
                ++fills;
                if (++slot == nstage) {
                    slot = 0;
                    ++rnd;
                }
            }
        }
        if (!ok) {
            // consumers gone: let every copy still in flight land before exit
            const uint64_t first = fills > (uint64_t)nstage ? fills - nstage : 0;
            for (uint64_t u = first; u < fills; ++u)
                mbar_wait_bounded(&full[u % nstage], (unsigned)((u / nstage) & 1), ka.status);
        }
        return;
    }

    // ---- consumers ----------------------------------------------------------
    const int c = (warp * 32 + lane) * V;  // first channel of this lane within the strip
    int slot = 0;
    unsigned parity = 0;
    for (int64_t item = blockIdx.x; item < prm.nitems; item += gridDim.x) {
        const ItemGeom g = geom(item);
        const int64_t gc = g.strip * WS + c;
        const bool valid = gc < ka.hd;  // hd is a multiple of V (16-byte rows)
        acc e[V], prod[V];
        {
            const acc* src = ka.cin != nullptr ? static_cast<const acc*>(ka.cin) + g.row * ka.hd + gc
                             : (!P::REV && ka.e0 != nullptr) ? static_cast<const acc*>(ka.e0) + g.b * ka.hd + gc
                                                             : nullptr;
#pragma unroll
            for (int i = 0; i < V; ++i) {
                e[i] = (src != nullptr && valid) ? src[i] : acc(0);
                prod[i] = acc(1);
            }
        }
        bool ok = true;
        for (int64_t j = 0; j < g.ntt; ++j) {
            const int64_t t0 = tile_t0(g, j);
            // every lane observes the copy (acquire); the warp stops together
            // if any lane's wait ran out
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], parity, ka.status))) {
                ok = false;
                break;
            }
            const char* sbase = smem + (size_t)slot * Cfg::stage_bytes();
            const int nrows = (int)(g.pend - t0 < LT ? g.pend - t0 : LT);
            char* ob0 = nullptr;
            char* ob1 = nullptr;
            int64_t os0 = 0, os1 = 0;
            if constexpr (!SUMM) {
                const int64_t orow0 = g.b * ka.T + t0;
                ob0 = ka.out[0].p + (orow0 * ka.out[0].rs + gc) * (int64_t)P::OES;
                ob1 = ka.out[1].p + (orow0 * ka.out[1].rs + gc) * (int64_t)P::OES;
                os0 = ka.out[0].rs * (int64_t)P::OES;
                os1 = ka.out[1].rs * (int64_t)P::OES;
            }
            // full tiles that do not hold step 0 run without per-step branches
            auto steps = [&](auto full_tag) {
                constexpr bool FULLT = decltype(full_tag)::value;
#pragma unroll
                for (int rr = 0; rr < LT; ++rr) {
                    const int r = P::REV ? (LT - 1 - rr) : rr;
                    if (FULLT || r < nrows) {
                        const char* rows[4];
#pragma unroll
                        for (int a = 0; a < 4; ++a)
                            rows[a] = a < P::NIN ? sbase + Cfg::array_off(a) + r * Cfg::row_bytes(a) + c * P::es(a)
                                                 : nullptr;
                        typename P::template Cache<1> cache;
                        acc a[V], bb[V];
                        step_coef<K, Tin, Te, 1, P>(rows, ka, a, bb, cache, 0);
                        if constexpr (SUMM) {
                            vfma(e, a, e, bb);
                            vmul(prod, prod, a);
                        } else {
                            step_apply<K, Tin, Te, 1, P, !FULLT>(rows, ka, g.b, t0 + r, gc, valid, e, cache, 0,
                                                                 ob0 + r * os0, ob1 + r * os1);
                        }
                    }
                }
            };
            if (nrows == LT && t0 > 0)
                steps(std::true_type{});
            else
                steps(std::false_type{});
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == nstage) {
                slot = 0;
                parity ^= 1u;
            }
        }
        if (!ok) break;
        if (valid) {
            if constexpr (SUMM) {
#pragma unroll
                for (int i = 0; i < V; ++i) static_cast<acc*>(ka.prod_out)[g.row * ka.hd + gc + i] = prod[i];
            }
            // final state: E at the piece end (forward) or the gradient
            // w.r.t. the incoming state (reverse)
            if (ka.e_last != nullptr) {
#pragma unroll
                for (int i = 0; i < V; ++i) static_cast<acc*>(ka.e_last)[g.row * ka.hd + gc + i] = e[i];
            }
        }
    }
}

template <Kind K, typename Tin, typename Te, int NW, bool SUMM>
int lane_launch_typed(const ScanCall& call, int nstage, int grid) {
    using Cfg = LaneCfg<K, Tin, Te, NW>;
    using P = typename Cfg::P;
    StripParams prm{};
    prm.a = call.a;
    prm.spr = (call.a.hd + Cfg::WS - 1) / Cfg::WS;
    prm.npiece = call.npiece > 1 ? call.npiece : 1;
    prm.plen = prm.npiece > 1 ? call.plen : ((call.a.T + Cfg::LT - 1) / Cfg::LT) * Cfg::LT;
    if (prm.plen % Cfg::LT != 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "piece length not a multiple of the tile");
    prm.nitems = call.a.nb * prm.npiece * prm.spr;
    prm.nstage = nstage;
    CUtensorMap maps[4];
    memset(maps, 0, sizeof(maps));
    const int dts[4] = {
        (K == Kind::RevPlain) ? call.te : call.tin,
        (K == Kind::RevPlain) ? call.te : call.tin,
        call.te,
        call.te,
    };
    for (int a = 0; a < P::NIN; ++a) {
        std::string err;
        const int rb = Cfg::row_bytes(a);
        if (!encode_strip_map(&maps[a], dts[a], call.a.in[a].p, call.a.nb, call.a.T, call.a.hd, call.a.in[a].rs,
                              Cfg::WS, Cfg::LT, &err, rb >= 256 ? 256 : rb))
            return set_error(ESA_ERR_CUDA, "tensor map: " + err);
    }
    const size_t smem = Cfg::smem_bytes(nstage);
    cudaError_t e = cudaFuncSetAttribute(lane_scan_kernel<K, Tin, Te, NW, SUMM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("lane smem attribute: ") + cudaGetErrorString(e));
    if (grid > prm.nitems) grid = (int)prm.nitems;
    note_scan_path(ESA_PATH_LANE);
    lane_scan_kernel<K, Tin, Te, NW, SUMM><<<grid, Cfg::NT, smem, call.stream>>>(prm, maps[0], maps[1], maps[2],
                                                                                 maps[3]);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("lane scan launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

template <Kind K, typename Tin, typename Te, int NW, bool SUMM>
int lane_occupancy(int dev, int nstage) {
    using Cfg = LaneCfg<K, Tin, Te, NW>;
    // [device][nstage]: 0 unknown, -1 none, else occupancy (atomic: see
    // strip_occupancy)
    static std::atomic<int> cache[16][17];
    if (dev < 0 || dev >= 16 || nstage < 1 || nstage > 16) return 0;
    std::atomic<int>& slot = cache[dev][nstage];
    const int known = slot.load(std::memory_order_relaxed);
    if (known != 0) return known < 0 ? 0 : known;
    const size_t smem = Cfg::smem_bytes(nstage);
    int per_sm = 0;
    if (smem <= 232448 &&
        cudaFuncSetAttribute(lane_scan_kernel<K, Tin, Te, NW, SUMM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lane_scan_kernel<K, Tin, Te, NW, SUMM>, Cfg::NT,
                                                      smem) == cudaSuccess &&
        per_sm > 0) {
        slot.store(per_sm, std::memory_order_relaxed);
    } else {
        slot.store(-1, std::memory_order_relaxed);
        per_sm = 0;
    }
    return per_sm;
}

// Picks the consumer warps per CTA and the ring depth, or declines
// (*taken = false) when the lanes cannot fill the GPU: fewer than
// `min_warps_per_sm` consumer warps per SM.  The ring holds at least
// `inflight` bytes of tiles ahead of the one being consumed.
template <Kind K, typename Tin, typename Te, bool SUMM = false>
int lane_launch_kind(const ScanCall& call, bool* taken, double min_warps_per_sm) {
    *taken = false;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sm_count(dev);
    const int64_t nb = call.a.nb * (call.npiece > 1 ? call.npiece : 1), hd = call.a.hd;
    if (call.a.T < 16) return ESA_OK;
    using C1 = LaneCfg<K, Tin, Te, 1>;
    const int64_t warps = nb * ((hd + C1::WS - 1) / C1::WS);
    if ((double)warps < min_warps_per_sm * sms) return ESA_OK;
    // two consumer warps (256-byte rows) when every SM still gets a CTA
    // (fp16 forward, us: [32,4096,16,64] 132.8 vs 134.3 with one warp;
    // [74,2048,16,64] 158.2 vs 180.0; [128,1024,16,64] 138.0 vs 154.1)
    int nw = 1;
    {
        using C2 = LaneCfg<K, Tin, Te, 2>;
        const int64_t ctas2 = nb * ((hd + C2::WS - 1) / C2::WS);
        nw = ctas2 >= (int64_t)sms ? 2 : 1;
    }
    const int stage = nw == 2 ? LaneCfg<K, Tin, Te, 2>::stage_bytes() : C1::stage_bytes();
    int ns = 0;
    {
        // about 16 KB of tiles in flight per consumer warp (the
        // [32,4096,16,64] fp16 forward with one consumer warp: 134.9 us at
        // three 8 KB stages against 150.7 at two and 147.5 / 161.6 / 217.2 at
        // four / six / eight; with two, 132.8 at three 16 KB stages against
        // 147.2 at two)
        ns = 1 + (16 * 1024 * nw + stage - 1) / stage;
        ns = ns < 2 ? 2 : (ns > 16 ? 16 : ns);
    }
    int occ = nw == 2 ? lane_occupancy<K, Tin, Te, 2, SUMM>(dev, ns) : lane_occupancy<K, Tin, Te, 1, SUMM>(dev, ns);
    while (occ <= 0 && ns > 2) {
        --ns;
        occ = nw == 2 ? lane_occupancy<K, Tin, Te, 2, SUMM>(dev, ns) : lane_occupancy<K, Tin, Te, 1, SUMM>(dev, ns);
    }
    if (occ <= 0) return ESA_OK;
    *taken = true;
    const int64_t cap = (int64_t)occ * sms;
    const int64_t items = nw == 2 ? nb * ((hd + LaneCfg<K, Tin, Te, 2>::WS - 1) / LaneCfg<K, Tin, Te, 2>::WS) : warps;
    const int grid = (int)(items < cap ? items : cap);
    return nw == 2 ? lane_launch_typed<K, Tin, Te, 2, SUMM>(call, ns, grid)
                   : lane_launch_typed<K, Tin, Te, 1, SUMM>(call, ns, grid);
}

}  // namespace esa
