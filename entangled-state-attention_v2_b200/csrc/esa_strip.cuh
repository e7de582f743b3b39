// esa_strip.cuh -- channel-strip scan: the main path of every scan kind.
//
// A CTA owns a strip of WS = LPR*VEC consecutive channels of one batch row and
// sweeps the whole time axis through it, tile by tile (LT steps per tile).
// The recurrence state never leaves the chip between tiles, so there is no
// inter-CTA communication and no waiting on other CTAs at all; the only waits
// are on this CTA's own TMA copies.  Parallelism comes from the channel
// count: nb*hd channels give nb*ceil(hd/WS) strips (e.g. 256 for the
// [32, 4096, 16, 64] fp16 microbenchmark with 128-channel strips).  For the
// split scan (few channels, long T) every batch row is cut into time pieces
// that are processed as rows of their own (StripParams::npiece/plen), from an
// incoming state per piece (KArgs::cin); the SUMM instantiations write only
// each piece's end state and coefficient product.
//
// Data movement.  One thread issues 3-D tiled TMA loads
// (cp.async.bulk.tensor.3d, tensor map [nb, T, hd], box [1, LT, WS], L2
// evict-first) of every staged array into an NSTAGE-deep ring of shared-memory
// stages (two by default), completing on one mbarrier per stage; the CTA
// consumes stage j while the next NSTAGE-1 tiles are in flight, and at the end
// of a strip the freed stages already take the first tiles of the CTA's next
// strip.  Outputs are stored from registers
// with 16-byte coalesced stores.  Each input byte crosses HBM once, each
// output byte once: the kernel's DRAM traffic is exactly the algorithmic one.
//
// Work inside a tile (8 warps).  Lane l of warp w owns channel vector
// cl = l % LPR (VEC channels, one 16-byte vector of the widest type) of row
// group rg = w*(32/LPR) + l/LPR, i.e. SR consecutive steps:
//   phase 1: compose the row group's SR steps into an affine pair (a, b);
//   warp:    inclusive Kogge-Stone scan of the pairs across the warp's row
//            groups with warp shuffles (lanes LPR apart share channels);
//   CTA:     warp totals through shared memory -> exclusive prefix per warp;
//   phase 3: re-run the SR steps from the exact incoming state
//            (carry o warp prefix o row-group prefix) and write the outputs;
//            the last row group leaves the tile's final state as the carry of
//            the next tile.
// Reverse kinds run the tiles and steps in descending time.
#pragma once

#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>
#include <type_traits>

#include "esa_scan_common.cuh"


namespace esa {

struct StripParams {
    KArgs a;
    int64_t spr;     // strips per (batch row, piece) = ceil(hd / WS)
    int64_t nitems;  // nb * npiece * spr
    int64_t npiece;  // time pieces per batch row (1: the whole axis)
    int64_t plen;    // steps per piece (a multiple of LT; >= T when npiece == 1)
    int nstage;
};

template <Kind K, typename Tin, typename Te, int LPR_, int SR_, int VN = 0>
struct StripCfg {
    using P = Policy<K, Tin, Te, VN>;
    static constexpr int LPR = LPR_;
    static constexpr int SR = SR_;
    static constexpr int NW = 8;
    static constexpr int NT = 32 * NW;
    static constexpr int VEC = P::VEC;
    static constexpr int RGW = 32 / LPR;  // row groups per warp
    static constexpr int RG = NW * RGW;   // row groups per CTA
    static constexpr int LT = RG * SR;    // steps per tile
    static constexpr int WS = LPR * VEC;  // channels per strip
    static __host__ __device__ constexpr int row_bytes(int a) { return WS * P::es(a); }
    static __host__ __device__ constexpr int array_off(int a) {
        int o = 0;
        for (int i = 0; i < a; ++i) o += LT * row_bytes(i);
        return o;
    }
    static __host__ __device__ constexpr int stage_bytes() { return array_off(P::NIN); }
    static size_t smem_bytes(int nstage) {
        return (size_t)nstage * stage_bytes() + (2 * NW * WS + 2 * WS) * sizeof(typename P::acc) +
               (size_t)nstage * sizeof(uint64_t) + 128;
    }
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar, uint64_t policy) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        :: "r"(d), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(b), "l"(policy)
        : "memory");
}

template <class Cfg>
__device__ __forceinline__ void strip_issue(const StripParams& prm, const CUtensorMap* const (&maps)[4],
                                            char* stage, uint64_t* bar, int64_t b, int64_t strip,
                                            int64_t t0, uint64_t policy) {
    using P = typename Cfg::P;
    mbar_arrive_expect_tx(bar, (unsigned)Cfg::stage_bytes());
#pragma unroll
    for (int a = 0; a < P::NIN; ++a)
        tma_load_3d(stage + Cfg::array_off(a), maps[a], (int)(strip * Cfg::WS),
                    (int)(t0 + P::shift(a)), (int)b, bar, policy);
}

// A shared-memory row of one accumulator vector per lane (LPR lanes x N
// accumulators), stored planar: plane p holds every lane's p-th 16-byte chunk,
// so a warp-wide access to one plane is a contiguous span (no bank conflicts
// beyond its width, whatever N is).
template <typename A, int N, int LPR>
__device__ __forceinline__ void lds_planar(const A* row, int cl, A (&out)[N]) {
    constexpr int PER = 16 / (int)sizeof(A);
    if constexpr (N < PER) {  // under 16 bytes a lane: one plane
        lds_vec<A, N>(row + cl * N, out);
        return;
    }
#pragma unroll
    for (int p = 0; p < N / PER; ++p) {
        const VecN<A, PER> v = *reinterpret_cast<const VecN<A, PER>*>(row + (p * LPR + cl) * PER);
#pragma unroll
        for (int i = 0; i < PER; ++i) out[p * PER + i] = v.v[i];
    }
}
template <typename A, int N, int LPR>
__device__ __forceinline__ void sts_planar(A* row, int cl, const A (&in)[N]) {
    constexpr int PER = 16 / (int)sizeof(A);
    if constexpr (N < PER) {
        sts_vec<A, N>(row + cl * N, in);
        return;
    }
#pragma unroll
    for (int p = 0; p < N / PER; ++p) {
        VecN<A, PER> v;
#pragma unroll
        for (int i = 0; i < PER; ++i) v.v[i] = in[p * PER + i];
        *reinterpret_cast<VecN<A, PER>*>(row + (p * LPR + cl) * PER) = v;
    }
}

template <Kind K, typename Tin, typename Te, int LPR, int SR, bool SUMM_, int VN = 0>
__global__ void __launch_bounds__(256, 2) strip_scan_kernel(const StripParams prm,
                                                         const __grid_constant__ CUtensorMap m0,
                                                         const __grid_constant__ CUtensorMap m1,
                                                         const __grid_constant__ CUtensorMap m2,
                                                         const __grid_constant__ CUtensorMap m3) {
    using Cfg = StripCfg<K, Tin, Te, LPR, SR, VN>;
    using P = typename Cfg::P;
    using acc = typename P::acc;
    constexpr int VEC = P::VEC;
    constexpr int WS = Cfg::WS;
    constexpr int NW = Cfg::NW;
    constexpr int RGW = Cfg::RGW;
    constexpr int LT = Cfg::LT;
    constexpr unsigned FULL = 0xffffffffu;
    // summary pass: no per-step outputs; the end state of each (row, piece)
    // from its incoming state and the product of its step coefficients
    constexpr bool SUMM = SUMM_ || K == Kind::FwdSummary;
    const KArgs& ka = prm.a;
    const int nstage = prm.nstage;

    extern __shared__ __align__(128) char smem_raw[];
    // 128-byte aligned base, derived from the shared array itself so that the
    // compiler keeps every pointer below in the shared window (LDS/STS, not
    // generic loads)
    char* smem = smem_raw + ((128u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 127u)) & 127u);
    // per-warp tile aggregates [NW][WS]
    acc* wagg_a = reinterpret_cast<acc*>(smem + (size_t)nstage * Cfg::stage_bytes());
    acc* wagg_b = wagg_a + NW * WS;
    acc* carry = wagg_b + NW * WS;  // [2][WS], double-buffered by tile parity
    uint64_t* bars = reinterpret_cast<uint64_t*>(carry + 2 * WS);

    const CUtensorMap* maps[4] = {&m0, &m1, &m2, &m3};
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rgl = lane / LPR;         // row group within the warp
    const int cl = lane - rgl * LPR;    // channel vector within the strip
    const int rg = warp * RGW + rgl;    // row group within the tile
    const int c = cl * VEC;             // first channel of this thread within the strip
    // the row group that processes a tile's last steps (carries the state on)
    const bool last_rg = P::REV ? (rg == 0) : (rg == Cfg::RG - 1);
    const bool last_rgl = P::REV ? (rgl == 0) : (rgl == RGW - 1);

    const uint64_t policy = policy_evict_first();
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstage; ++s) mbar_init(&bars[s], 1);
        fence_mbarrier_init();
    }
    __syncthreads();

    uint64_t used = 0;    // tiles consumed by this CTA so far (stage = used % nstage)
    uint64_t issued = 0;  // tiles whose copies this CTA has issued
    int slot = 0;         // ring stage of the next tile to consume (= used % nstage)
    unsigned parity = 0;  // its mbarrier phase parity (= (used / nstage) & 1)
    bool aborted = false;
    // tiles of the current item already issued by the previous item's tail
    // (the ring runs on into the next item of this CTA without draining)
    int pre = 0;
    // geometry of an item: (batch row, piece) row, strip, piece start, tiles
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
    auto geom_t0 = [&](const ItemGeom& g, int64_t j) -> int64_t {
        return g.pbeg + (P::REV ? (g.ntt - 1 - j) : j) * (int64_t)LT;
    };
    for (int64_t item = blockIdx.x; item < prm.nitems && !aborted; item += gridDim.x) {
        const ItemGeom ig = geom(item);
        const int64_t row = ig.row;  // (batch row, piece)
        const int64_t strip = ig.strip;
        const int64_t b = ig.b;
        const int64_t pend = ig.pend;
        const int64_t ntt = ig.ntt;  // tiles of the piece
        const int64_t gc = strip * WS + c;  // first global channel of this thread
        const bool valid = gc < ka.hd;
        auto tile_t0 = [&](int64_t j) -> int64_t { return geom_t0(ig, j); };
        // the next item of this CTA, whose first tiles this item's tail issues
        const int64_t next = item + gridDim.x;
        const bool has_next = next < prm.nitems && ntt >= nstage;
        const ItemGeom ng = geom(has_next ? next : item);
        const int next_pre = has_next ? (int)(ng.ntt < nstage ? ng.ntt : nstage) : 0;
        acc prod_run[VEC];  // FwdSummary: product of A so far (last row group's lanes)
#pragma unroll
        for (int i = 0; i < VEC; ++i) prod_run[i] = acc(1);
        // initial carry: the piece's incoming state (split passes), else e0
        // (forward) or zero (reverse: nothing after T)
        if (rgl == 0 && warp == 0) {
            acc x[VEC];
            const acc* src = ka.cin != nullptr ? static_cast<const acc*>(ka.cin) + row * ka.hd + gc
                             : (!P::REV && ka.e0 != nullptr) ? static_cast<const acc*>(ka.e0) + b * ka.hd + gc
                                                             : nullptr;
#pragma unroll
            for (int i = 0; i < VEC; ++i) x[i] = (src != nullptr && valid) ? src[i] : acc(0);
            sts_planar<acc, VEC, LPR>(carry, cl, x);  // slot 0
        }
        // prologue: fill the ring
        const int npro = (int)(ntt < nstage ? ntt : nstage);
        if (threadIdx.x == 0) {
            int sl = slot + pre;
            if (sl >= nstage) sl -= nstage;
            for (int s = pre; s < npro; ++s) {
                strip_issue<Cfg>(prm, maps, smem + (size_t)sl * Cfg::stage_bytes(), &bars[sl], b,
                                 strip, tile_t0(s), policy);
                if (++sl == nstage) sl = 0;
            }
        }
        issued += npro > pre ? npro - pre : 0;
        __syncthreads();

        for (int64_t j = 0; j < ntt; ++j, ++used) {
            const int cur = (int)(j & 1);
            const int64_t t0 = tile_t0(j);
            const bool ok = mbar_wait_bounded(&bars[slot], parity, ka.status);
            const char* sbase = smem + (size_t)slot * Cfg::stage_bytes();
            auto rows_at = [&](int r, const char* (&rows)[4]) {
#pragma unroll
                for (int a = 0; a < 4; ++a)
                    rows[a] = a < P::NIN ? sbase + Cfg::array_off(a) + r * Cfg::row_bytes(a) + c * P::es(a)
                                         : nullptr;
            };

            // ---- phase 1: this row group's SR steps ------------------------
            typename P::template Cache<SR> cache;
            acc pa[VEC], pb[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                pa[i] = acc(1);
                pb[i] = acc(0);
            }
            // every step of this row group inside [0, T) (all but the last tile):
            // the step loops run without per-step bounds checks
            const bool rg_full = t0 + (rg + 1) * SR <= pend;
            auto phase1 = [&](auto full_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
                for (int ss = 0; ss < SR; ++ss) {
                    const int s = P::REV ? (SR - 1 - ss) : ss;
                    const int r = rg * SR + s;
                    if (FULL || t0 + r < pend) {
                        const char* rows[4];
                        rows_at(r, rows);
                        acc a[VEC], bb[VEC];
                        step_coef<K, Tin, Te, SR, P>(rows, ka, a, bb, cache, s);
                        vfma(pb, a, pb, bb);
                        vmul(pa, a, pa);
                    }
                }
            };
            if (rg_full)
                phase1(std::true_type{});
            else
                phase1(std::false_type{});
            // ---- warp: inclusive scan over row groups (shuffles) -----------
            acc ex_a[VEC], ex_b[VEC];  // first round's neighbour (RGW == 2: the exclusive prefix)
#pragma unroll
            for (int d = 1; d < RGW; d <<= 1) {
                acc qa[VEC], qb[VEC];
                const bool take = P::REV ? (rgl + d < RGW) : (rgl >= d);
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    if constexpr (P::REV) {
                        qa[i] = __shfl_down_sync(FULL, pa[i], d * LPR);
                        qb[i] = __shfl_down_sync(FULL, pb[i], d * LPR);
                    } else {
                        qa[i] = __shfl_up_sync(FULL, pa[i], d * LPR);
                        qb[i] = __shfl_up_sync(FULL, pb[i], d * LPR);
                    }
                    if (d == 1) {
                        ex_a[i] = qa[i];
                        ex_b[i] = qb[i];
                    }
                    // lanes without an earlier row group compose with identity
                    qa[i] = take ? qa[i] : acc(1);
                    qb[i] = take ? qb[i] : acc(0);
                }
                vcompose(pa, pb, qa, qb);
            }
            // exclusive prefix of this row group within the warp (with two row
            // groups it is the first round's shuffled value)
            acc xa[VEC], xb[VEC];
            {
                const bool first = P::REV ? (rgl == RGW - 1) : (rgl == 0);
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    acc qa = acc(1), qb = acc(0);
                    if constexpr (RGW == 2) {
                        qa = ex_a[i];
                        qb = ex_b[i];
                    } else if constexpr (RGW > 1) {
                        if constexpr (P::REV) {
                            qa = __shfl_down_sync(FULL, pa[i], LPR);
                            qb = __shfl_down_sync(FULL, pb[i], LPR);
                        } else {
                            qa = __shfl_up_sync(FULL, pa[i], LPR);
                            qb = __shfl_up_sync(FULL, pb[i], LPR);
                        }
                    }
                    xa[i] = first ? acc(1) : qa;
                    xb[i] = first ? acc(0) : qb;
                }
            }
            acc* const wa = wagg_a;
            acc* const wb = wagg_b;
            if (last_rgl) {
                sts_planar<acc, VEC, LPR>(wa + warp * WS, cl, pa);
                sts_planar<acc, VEC, LPR>(wb + warp * WS, cl, pb);
            }
            __syncthreads();  // warp totals of this tile visible

            // ---- CTA: exclusive prefix over the warps before this one -------
            acc ea[VEC], eb[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                ea[i] = acc(1);
                eb[i] = acc(0);
            }
#pragma unroll
            for (int n = 0; n < NW; ++n) {
                const int w = P::REV ? (NW - 1 - n) : n;
                if (w == warp) break;
                acc aw[VEC], bw[VEC];
                lds_planar<acc, VEC, LPR>(wa + w * WS, cl, aw);
                lds_planar<acc, VEC, LPR>(wb + w * WS, cl, bw);
                vfma(eb, aw, eb, bw);
                vmul(ea, aw, ea);
            }
            acc e[VEC];
            lds_planar<acc, VEC, LPR>(carry + cur * WS, cl, e);
            vfma(e, ea, e, eb);  // through the warps before this one
            if constexpr (SUMM) {
                // no per-step outputs: the last row group's warp-inclusive pair
                // carries the state to the tile end; the product of A follows
                if (last_rg) {
                    vfma(e, pa, e, pb);
                    vmul(prod_run, prod_run, ea);
                    vmul(prod_run, prod_run, pa);
                }
            } else {
            // ---- phase 3: incoming state, re-run, outputs ------------------
            vfma(e, xa, e, xb);  // through the row groups before this one
            // output addresses of this row group's first step; one row stride per step
            const int64_t orow0 = b * ka.T + t0 + rg * SR;
            char* const ob0 = ka.out[0].p + (orow0 * ka.out[0].rs + gc) * (int64_t)P::OES;
            char* const ob1 = ka.out[1].p + (orow0 * ka.out[1].rs + gc) * (int64_t)P::OES;
            const int64_t os0 = ka.out[0].rs * (int64_t)P::OES, os1 = ka.out[1].rs * (int64_t)P::OES;
            // MAY_T0: the tile holds step 0, whose E_{-1} is e0 (reverse kinds);
            // every other tile reads E_{t-1} from the stage with no test on t
            auto phase3 = [&](auto full_tag, auto t0_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
                constexpr bool MAY_T0 = decltype(t0_tag)::value;
#pragma unroll
                for (int ss = 0; ss < SR; ++ss) {
                    const int s = P::REV ? (SR - 1 - ss) : ss;
                    const int r = rg * SR + s;
                    const int64_t t = t0 + r;
                    if (FULL || t < pend) {
                        const char* rows[4];
                        rows_at(r, rows);
                        step_apply<K, Tin, Te, SR, P, MAY_T0>(rows, ka, b, t, gc, valid, e, cache, s,
                                                              ob0 + s * os0, ob1 + s * os1);
                    }
                }
            };
            if (P::REV && t0 == 0) {
                if (rg_full)
                    phase3(std::true_type{}, std::true_type{});
                else
                    phase3(std::false_type{}, std::true_type{});
            } else {
                if (rg_full)
                    phase3(std::true_type{}, std::false_type{});
                else
                    phase3(std::false_type{}, std::false_type{});
            }
            }
            if (last_rg) sts_planar<acc, VEC, LPR>(carry + (cur ^ 1) * WS, cl, e);
            // stage `slot` consumed, next carry visible; the whole CTA stops if
            // any thread's copy wait ran out
            if (__syncthreads_or(!ok)) {
                aborted = true;
                break;
            }
            if (j + nstage < ntt) {
                if (threadIdx.x == 0)
                    strip_issue<Cfg>(prm, maps, smem + (size_t)slot * Cfg::stage_bytes(), &bars[slot],
                                     b, strip, tile_t0(j + nstage), policy);
                ++issued;
            } else if (j + nstage - ntt < next_pre) {
                // the freed stage takes the next item's tile j + nstage - ntt
                if (threadIdx.x == 0)
                    strip_issue<Cfg>(prm, maps, smem + (size_t)slot * Cfg::stage_bytes(), &bars[slot],
                                     ng.b, ng.strip, geom_t0(ng, j + nstage - ntt), policy);
                ++issued;
            }
            if (++slot == nstage) {
                slot = 0;
                parity ^= 1u;
            }
        }
        if (aborted) break;
        if constexpr (SUMM) {
            if (last_rg && valid) {
#pragma unroll
                for (int i = 0; i < VEC; ++i) static_cast<acc*>(ka.prod_out)[row * ka.hd + gc + i] = prod_run[i];
            }
        }
        // final state: E_{T-1} (forward) or the gradient w.r.t. e0 (reverse)
        if (ka.e_last != nullptr && rgl == 0 && warp == 0 && valid) {
            const int fin = (int)(ntt & 1);
            acc x[VEC];
            lds_planar<acc, VEC, LPR>(carry + fin * WS, cl, x);
#pragma unroll
            for (int i = 0; i < VEC; ++i) static_cast<acc*>(ka.e_last)[row * ka.hd + gc + i] = x[i];
        }
        pre = next_pre;
        __syncthreads();
    }
    // after a failed wait, give every copy still in flight one more bounded
    // wait, so that no TMA copy targets this CTA's shared memory after exit
    for (uint64_t u = used; u < issued; ++u)
        mbar_wait_bounded(&bars[u % nstage], (unsigned)((u / nstage) & 1), ka.status);
}

// Build a 3-D tensor map [nb][T][hd] (row stride rs elements) with box
// [1][LT][WS] for dtype code `dtype`; L2 promotion of `promo_bytes` (256,
// 128, 64 or 0 = none).
bool encode_strip_map(CUtensorMap* map, int dtype, const void* base, int64_t nb, int64_t T,
                      int64_t hd, int64_t rs, int ws, int lt, std::string* err, int promo_bytes = 256);

template <Kind K, typename Tin, typename Te, int LPR, int SR, bool SUMM, int VN = 0>
int strip_launch_typed(const ScanCall& call, int nstage, int grid) {
    using Cfg = StripCfg<K, Tin, Te, LPR, SR, VN>;
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
        const int64_t rs = call.a.in[a].rs;
        if (!encode_strip_map(&maps[a], dts[a], call.a.in[a].p, call.a.nb, call.a.T, call.a.hd, rs,
                              Cfg::WS, Cfg::LT, &err))
            return set_error(ESA_ERR_CUDA, "tensor map: " + err);
    }
    const size_t smem = Cfg::smem_bytes(nstage);
    auto kern = strip_scan_kernel<K, Tin, Te, LPR, SR, SUMM, VN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("strip smem attribute: ") + cudaGetErrorString(e));
    if (grid > prm.nitems) grid = (int)prm.nitems;
    note_scan_path(ESA_PATH_STRIP);
    kern<<<grid, Cfg::NT, smem, call.stream>>>(prm, maps[0], maps[1], maps[2], maps[3]);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("strip scan launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

// Occupancy (CTAs per SM) of a strip configuration with `nstage` stages
// (cached per device and stage count; 0 if it cannot be resident).
template <Kind K, typename Tin, typename Te, int LPR, int SR, bool SUMM, int VN = 0>
int strip_occupancy(int dev, int nstage) {
    using Cfg = StripCfg<K, Tin, Te, LPR, SR, VN>;
    // [device][nstage]: 0 unknown, -1 none, else occupancy; atomic so that
    // concurrent first calls from several host threads are well defined (they
    // compute the same value)
    static std::atomic<int> cache[16][9];
    if (dev < 0 || dev >= 16 || nstage < 1 || nstage > 8) return 0;
    std::atomic<int>& slot = cache[dev][nstage];
    const int known = slot.load(std::memory_order_relaxed);
    if (known != 0) return known < 0 ? 0 : known;
    const size_t smem = Cfg::smem_bytes(nstage);
    int per_sm = 0;
    if (smem <= 232448 &&
        cudaFuncSetAttribute(strip_scan_kernel<K, Tin, Te, LPR, SR, SUMM, VN>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, strip_scan_kernel<K, Tin, Te, LPR, SR, SUMM, VN>,
                                                      Cfg::NT, smem) == cudaSuccess &&
        per_sm > 0) {
        slot.store(per_sm, std::memory_order_relaxed);
    } else {
        slot.store(-1, std::memory_order_relaxed);
        per_sm = 0;
    }
    return per_sm;
}


// Picks the strip width (LPR) and pipeline depth for the call, or declines
// (*taken = false) when the strips cannot fill the GPU (then the caller uses
// the time-parallel lookback scan).  Each width is scored by load balance
// (strips over SMs in one wave, or waves over the resident CTAs) x 0.6 when
// SMs would hold a single CTA x a short-row penalty (0.97 for 128-byte rows,
// 0.9 for 64-byte rows); ties go to the wider strip.  Stages: two (see below).
template <Kind K, typename Tin, typename Te, int SR4, int SR8, int SR16, int SR32, bool SUMM = false, int NSR = 0,
          int NVN = 2>
int strip_launch_kind(const ScanCall& call, bool* taken) {
    *taken = false;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sm_count(dev);
    // rows of the strip scan: batch rows x time pieces
    const int64_t T = call.a.T, nb = call.a.nb * (call.npiece > 1 ? call.npiece : 1), hd = call.a.hd;
    using P = Policy<K, Tin, Te>;
    if (T < 16) return ESA_OK;
    // narrow form (NSR > 0, float accumulators): strips of 32 lanes of NVN
    // channels, one row group a warp and NSR steps a thread -- no shuffle
    // scan across row groups, the CTA prefix amortised over NSR steps (the
    // [16, 2048, 768] fp16 gated forward: 2.03 -> 2.76 TB/s against 8-channel
    // lanes; the [32, 4096, 16, 64] fp16 plain reverse with 4-channel lanes:
    // 5.59 -> 6.07 TB/s); taken whenever its strips fill the GPU
    if constexpr (NSR > 0 && std::is_same<typename Policy<K, Tin, Te, NVN>::acc, float>::value) {
        const int64_t n = nb * ((hd + 32 * NVN - 1) / (32 * NVN));
        if (n >= (sms * 3) / 4) {
            int ns = 0, o = 0;
            for (int s = 2; s <= 6; ++s) {
                const int os = strip_occupancy<K, Tin, Te, 32, NSR, SUMM, NVN>(dev, s);
                if (os > o) {
                    o = os;
                    ns = s;
                }
                if (o >= 2) break;
            }
            if (o > 0) {
                *taken = true;
                const int64_t cap = (int64_t)o * sms;
                return strip_launch_typed<K, Tin, Te, 32, NSR, SUMM, NVN>(call, ns, (int)(n < cap ? n : cap));
            }
        }
    }
    auto strips = [&](int lpr) { return nb * ((hd + lpr * P::VEC - 1) / (lpr * P::VEC)); };
    auto occ = [&](int lpr, int ns) -> int {
        switch (lpr) {
            case 32: return strip_occupancy<K, Tin, Te, 32, SR32, SUMM>(dev, ns);
            case 16: return strip_occupancy<K, Tin, Te, 16, SR16, SUMM>(dev, ns);
            case 8: return strip_occupancy<K, Tin, Te, 8, SR8, SUMM>(dev, ns);
            default: return strip_occupancy<K, Tin, Te, 4, SR4, SUMM>(dev, ns);
        }
    };
    int pick_lpr = 0, pick_ns = 0, pick_occ = 0;
    double best = 0.0;
    for (int lpr : {32, 16, 8, 4}) {
        const int64_t n = strips(lpr);
        if (n < (sms * 3) / 4) continue;  // too few strips to fill the GPU
        // two stages (measured: never slower than 3-6, and 8 % faster on the
        // [32,4096,16,64] fp16 forward -- 5.84 vs 5.38 TB/s -- with the same
        // occupancy); more only if two do not fit.  The 16-bit reverse takes
        // three when they keep the occupancy of two (237.8 vs 243.9 us on
        // [32,4096,16,64] fp16: its stages hold 32 steps, not 64).
        int ns = 0, o = 0;
        if (K == Kind::RevPlain && sizeof(Te) == 2 && occ(lpr, 3) >= occ(lpr, 2) && occ(lpr, 3) > 0) {
            ns = 3;
            o = occ(lpr, 3);
        }
        for (int s = 2; s <= 6 && ns == 0; ++s) {
            const int os = occ(lpr, s);
            if (os > o) {
                o = os;
                ns = s;
            }
            if (o >= 2) break;
        }
        if (o <= 0) continue;
        const int64_t slots = (int64_t)o * sms;
        // load balance: one wave spread over the SMs, or waves over the slots
        double balance;
        int64_t per_sm;
        if (n <= slots) {
            per_sm = (n + sms - 1) / sms;
            balance = (double)n / (double)(per_sm * sms);
        } else {
            per_sm = o;
            const int64_t waves = (n + slots - 1) / slots;
            balance = (double)n / (double)(waves * slots);
        }
        // a lone 8-warp CTA per SM cannot hide the per-tile barriers and
        // shared-memory round trips; 64-byte rows make short DRAM bursts
        const double conc = per_sm >= 2 ? 1.0 : 0.6;
        const double width = lpr >= 16 ? 1.0 : (lpr == 8 ? 0.97 : 0.9);
        const double score = balance * conc * width;
        if (score > best + 1e-9) {
            best = score;
            pick_lpr = lpr;
            pick_ns = ns;
            pick_occ = o;
        }
    }
    if (pick_lpr == 0) return ESA_OK;  // too few channels for strips: not taken
    *taken = true;
    const int64_t n = strips(pick_lpr);
    const int64_t cap = (int64_t)pick_occ * sms;
    const int grid = (int)(n < cap ? n : cap);
    switch (pick_lpr) {
        case 32: return strip_launch_typed<K, Tin, Te, 32, SR32, SUMM>(call, pick_ns, grid);
        case 16: return strip_launch_typed<K, Tin, Te, 16, SR16, SUMM>(call, pick_ns, grid);
        case 8: return strip_launch_typed<K, Tin, Te, 8, SR8, SUMM>(call, pick_ns, grid);
        default: return strip_launch_typed<K, Tin, Te, 4, SR4, SUMM>(call, pick_ns, grid);
    }
}

}  // namespace esa
