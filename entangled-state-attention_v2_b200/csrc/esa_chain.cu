// esa_chain.cu -- single-pass chained scan for few channels and long time
// axes (the [4, 262144, 32, 64] long-sequence forward scan).
//
// With few channels the lane-serial kernel (esa_lane.cuh) has too few lanes
// to fill 148 SMs, so the time axis has to be cut into pieces that run in
// parallel.  The split scan (esa_scan_api.cu: run_split) does that in three
// launches: a summary pass reading A and B, a composition of the piece
// summaries, and an output pass reading A and B again from HBM (10 bytes per
// 16-bit element moved for 6 algorithmic).  This kernel does it in one.
//
// item = (piece p, strip of WS channels of one batch row), claimed from an
// atomic ticket in (piece, strip) order; its predecessors are the items of
// the same strip and earlier pieces (k - nstrips, k - 2 nstrips, ...).
// A CTA is NW consumer warps, one producer warp and one look-back warp:
//   producer: claims items, streams each item's tiles twice into the ring
//           (3-D TMA): pass 0 with L2 evict-normal, pass 1 (the same tiles,
//           now served by L2: the pieces in flight on the whole GPU are
//           sized to stay resident) with L2 evict-first;
//   consumers, pass 0: each lane composes its channels' steps from a zero
//           state (end state and product of A), publishes that aggregate
//           and, once the look-back warp hands over the item's incoming
//           state, the inclusive prefix (per item a flag word that
//           counts the consumer warps' published parts of each);
//   look-back warp: as soon as an item is claimed -- while the consumers
//           still run its pass 0 -- resolves its incoming state from the
//           predecessors' flags (single-pass decoupled look-back, Merrill &
//           Garland 2016: compose aggregates back to the nearest inclusive
//           prefix), so the consumers rarely wait for it;
//   consumers, pass 1: re-run the steps from the exact incoming state and
//           write E with streaming stores.
//
// HBM traffic is the algorithmic A, B read once and E written once (an ncu
// capture of [4, 65536, 32, 64] bf16 reads 2.149 GB for 2.147 algorithmic).
// Items are claimed in order by running CTAs and an item only waits on items
// claimed before it, so every wait ends; each wait is still bounded (device
// status word + per-launch abort flag).
#include <atomic>
#include <string>

#include "esa_lane.cuh"
#include "esa_lookback.cuh"

namespace esa {

namespace {

constexpr int kChainNW = 2;        // consumer warps per CTA
constexpr int kChainItemRing = 4;  // item indices in flight between the producer and its readers

struct ChainParams {
    KArgs a;
    int64_t spr;      // strips per batch row
    int64_t nstrips;  // nb * spr: items per piece index
    int64_t npiece;   // pieces per batch row
    int64_t plen;     // steps per piece (a multiple of the tile)
    int64_t nitems;   // npiece * nstrips
    int nstage;
    Workspace ws;     // ticket, abort flag, per-item flags, aggregates and prefixes (WS floats each)
};

__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Streaming (evict-first) store of one lane vector of E.
template <typename T, int V>
__device__ __forceinline__ void store_cs(char* p, const float (&e)[V]) {
    if constexpr (std::is_same<T, __half>::value && V == 2) {
        const __half2 h = __floats2half2_rn(e[0], e[1]);
        __stcs(reinterpret_cast<unsigned*>(p), *reinterpret_cast<const unsigned*>(&h));
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value && V == 2) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(e[0], e[1]);
        __stcs(reinterpret_cast<unsigned*>(p), *reinterpret_cast<const unsigned*>(&h));
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) __stcs(reinterpret_cast<float*>(p) + i, e[i]);
    }
}

// Release-ordered add to an item's flag word: every consumer warp adds
// kFlagAgg once its part of the aggregate is written and kFlagPfx once its
// part of the inclusive prefix is (a first piece publishes no aggregate), so
// the low byte counts aggregate parts and the next byte prefix parts: NW
// parts make that value complete, and no consumer warp waits for another.
constexpr unsigned kFlagAgg = 1u, kFlagPfx = 256u;
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Vector load / store of N floats of a workspace array (L2, bypassing L1).
template <int N>
__device__ __forceinline__ void ldcg_vec(const float* p, float (&v)[N]) {
    if constexpr (N == 4) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(p));
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (N == 2) {
        const float2 x = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = x.x; v[1] = x.y;
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = __ldcg(p + i);
    }
}

template <typename T, int NW>
struct ChainCfg {
    static constexpr int V = sizeof(T) == 2 ? 2 : 1;
    static constexpr int LT = 32;            // steps per tile
    static constexpr int WS = 32 * V * NW;   // channels per strip
    static constexpr int CPL = WS / 32;      // channels per look-back lane
    static constexpr int ROW = WS * (int)sizeof(T);
    static constexpr int NT = 32 * (NW + 2);
    static constexpr int stage_bytes() { return 2 * LT * ROW; }  // A and B
    static size_t smem_bytes(int nstage) {
        return (size_t)nstage * (stage_bytes() + 2 * sizeof(uint64_t)) +
               kChainItemRing * (2 * sizeof(uint64_t) + sizeof(int64_t)) + 2 * (WS * sizeof(float) + 2 * sizeof(uint64_t)) +
               128;
    }
};

// Incoming state of item k (piece p > 0) for this lane's CPL channels,
// composed from the predecessors' aggregates back to the nearest inclusive
// prefix.  Returns false if the wait ran out (x is then zero).
template <int WS, int CPL, int NW>
__device__ __forceinline__ bool resolve_incoming(const Workspace& ws, unsigned* status, int64_t k,
                                                 int64_t nstrips, int64_t p, int lane, float (&x)[CPL]) {
    const float* agg_a = static_cast<const float*>(ws.agg_a);
    const float* agg_b = static_cast<const float*>(ws.agg_b);
    const float* pref = static_cast<const float*>(ws.pref);
    float ca[CPL], cb[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        ca[i] = 1.0f;
        cb[i] = 0.0f;
    }
    int64_t consumed = 0;
    unsigned long long t_start = 0;
    unsigned spins = 0;
    while (true) {
        const int64_t i = consumed + lane;
        unsigned f = 0;
        if (i < p) f = ld_acquire_gpu(ws.flags + (k - (i + 1) * nstrips));
        const bool pfx_done = (f / kFlagPfx) >= (unsigned)NW;
        const bool agg_done = (f % kFlagPfx) >= (unsigned)NW;
        const unsigned nz = __ballot_sync(0xffffffffu, agg_done || pfx_done);
        const unsigned ip = __ballot_sync(0xffffffffu, pfx_done);
        const int m = (nz == 0xffffffffu) ? 32 : (__ffs(~nz) - 1);
        const unsigned mm = (m >= 32) ? 0xffffffffu : ((1u << m) - 1u);
        const unsigned pm = ip & mm;
        const int pf = pm ? (__ffs(pm) - 1) : -1;
        const int nagg = (pf >= 0) ? pf : m;
        // aggregates of the run before the prefix, four predecessors' loads
        // in flight at a time
        for (int q0 = 0; q0 < nagg; q0 += 4) {
            float ra[4][CPL], rb[4][CPL];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (q0 + u < nagg) {
                    const int64_t jo = (k - (consumed + q0 + u + 1) * nstrips) * WS + lane * CPL;
                    ldcg_vec<CPL>(agg_a + jo, ra[u]);
                    ldcg_vec<CPL>(agg_b + jo, rb[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (q0 + u < nagg) {
#pragma unroll
                    for (int c = 0; c < CPL; ++c) {
                        cb[c] = fmaf(ca[c], rb[u][c], cb[c]);
                        ca[c] = ca[c] * ra[u][c];
                    }
                }
            }
        }
        if (pf >= 0) {
            float pv[CPL];
            ldcg_vec<CPL>(pref + (k - (consumed + pf + 1) * nstrips) * WS + lane * CPL, pv);
#pragma unroll
            for (int c = 0; c < CPL; ++c) x[c] = fmaf(ca[c], pv[c], cb[c]);
            return true;
        }
        consumed += m;
        if (m == 0) {
            // the nearest pending predecessor has published nothing yet: one
            // lane polls its flag alone, backing off from 128 ns to 2 us
            // between reads (hundreds of warps polling at full rate would
            // load the L2 the scans stream through), then the window is read
            // again
            const unsigned* fp = ws.flags + (k - (consumed + 1) * nstrips);
            bool ready = false, expired = false;
            unsigned ns = 128;
            if (spins == 0) t_start = globaltimer_ns();
            while (!ready && !expired) {
                if (lane == 0) {
                    const unsigned f0 = ld_acquire_gpu(fp);
                    ready = (f0 / kFlagPfx) >= (unsigned)NW || (f0 % kFlagPfx) >= (unsigned)NW;
                    if (!ready) {
                        __nanosleep(ns);
                        ns = ns < 2048 ? 2 * ns : 2048;
                        // give up after the wait budget, or at once if another
                        // wait of this launch already gave up
                        expired = (++spins > kWaitMaxIters) || (globaltimer_ns() - t_start > kWaitBudgetNs) ||
                                  (*(volatile unsigned*)ws.abort_flag != 0u);
                    }
                }
                ready = __shfl_sync(0xffffffffu, ready, 0);
                expired = __shfl_sync(0xffffffffu, expired, 0);
            }
            if (expired) {
                if (lane == 0) {
                    atomicOr(status, ESA_STATUS_LOOKBACK_TIMEOUT);
                    atomicExch(ws.abort_flag, 1u);
                }
#pragma unroll
                for (int c = 0; c < CPL; ++c) x[c] = 0.0f;
                return false;
            }
        }
    }
}

template <typename T, int NW>
__global__ void __launch_bounds__(32 * (NW + 2)) chain_scan_kernel(const ChainParams prm,
                                                                   const __grid_constant__ CUtensorMap mA,
                                                                   const __grid_constant__ CUtensorMap mB) {
    using Cfg = ChainCfg<T, NW>;
    constexpr int V = Cfg::V;
    constexpr int LT = Cfg::LT;
    constexpr int WS = Cfg::WS;
    constexpr int CPL = Cfg::CPL;
    constexpr int R = kChainItemRing;
    const KArgs& ka = prm.a;
    const int nstage = prm.nstage;

    extern __shared__ __align__(128) char smem_raw[];
    char* smem = smem_raw + ((128u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 127u)) & 127u);
    float* s_x = reinterpret_cast<float*>(smem + (size_t)nstage * Cfg::stage_bytes());  // [2][WS]
    uint64_t* full = reinterpret_cast<uint64_t*>(s_x + 2 * WS);
    uint64_t* empty = full + nstage;
    uint64_t* item_full = empty + nstage;    // [R]: s_item[q] written (producer)
    uint64_t* item_empty = item_full + R;    // [R]: s_item[q] read (look-back warp + consumer warps)
    uint64_t* x_full = item_empty + R;       // [2]: s_x[h] written (look-back warp)
    uint64_t* x_empty = x_full + 2;          // [2]: s_x[h] read (consumer warps)
    int64_t* s_item = reinterpret_cast<int64_t*>(x_empty + 2);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        for (int q = 0; q < R; ++q) {
            mbar_init(&item_full[q], 1);
            mbar_init(&item_empty[q], NW + 1);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&x_full[h], 1);
            mbar_init(&x_empty[h], NW);
        }
        fence_mbarrier_init();
    }
    __syncthreads();

    if (warp == NW) {
        // ---- producer: lane 0 claims items and fills the ring --------------
        if (lane != 0) return;
        const uint64_t pol_keep = policy_evict_normal();
        const uint64_t pol_last = policy_evict_first();
        uint64_t fills = 0;
        int slot = 0;
        unsigned rnd = 0;  // completed trips of the ring before `slot`'s next fill
        bool ok = true;
        auto acquire_slot = [&]() -> bool {
            return rnd == 0 || mbar_wait_bounded(&empty[slot], (rnd - 1) & 1u, ka.status);
        };
        auto advance = [&]() {
            ++fills;
            if (++slot == nstage) {
                slot = 0;
                ++rnd;
            }
        };
        // one pass of an item's tiles into the ring
        auto issue_pass = [&](int64_t k, int pass, bool first_acquired) {
            const int64_t p = k / prm.nstrips;
            const int64_t rs = k - p * prm.nstrips;
            const int64_t b = rs / prm.spr;
            const int64_t strip = rs - b * prm.spr;
            const int64_t pbeg = p * prm.plen;
            const int64_t pend = pbeg + prm.plen < ka.T ? pbeg + prm.plen : ka.T;
            const int64_t ntt = (pend - pbeg + LT - 1) / LT;
            const uint64_t pol = pass == 0 ? pol_keep : pol_last;
            for (int64_t j = 0; j < ntt; ++j) {
                if ((j > 0 || !first_acquired) && !acquire_slot()) {
                    ok = false;
                    return;
                }
                char* stage = smem + (size_t)slot * Cfg::stage_bytes();
                const int t0 = (int)(pbeg + j * LT);
                mbar_arrive_expect_tx(&full[slot], (unsigned)Cfg::stage_bytes());
                tma_load_3d(stage, &mA, (int)(strip * WS), t0, (int)b, &full[slot], pol);
                tma_load_3d(stage + LT * Cfg::ROW, &mB, (int)(strip * WS), t0, (int)b, &full[slot], pol);
                advance();
            }
        };
        // per claim: pass 0 of the item, then its pass 1
        for (int64_t n = 0; ok; ++n) {
            const int q = (int)(n % R);
            // the item slot's previous index read by all its readers, and the
            // first stage free; only then claim, so that a claimed item is
            // never held back behind this CTA's current one
            if ((n >= R && !mbar_wait_bounded(&item_empty[q], (unsigned)((n / R - 1) & 1), ka.status)) ||
                !acquire_slot()) {
                ok = false;
                break;
            }
            const int64_t k = (int64_t)atomicAdd(prm.ws.ticket, 1u);
            s_item[q] = k < prm.nitems ? k : -1;
            mbar_arrive(&item_full[q]);
            if (k >= prm.nitems) {
                // no more work: complete the stage's phase without data so
                // the consumers read the end marker
                mbar_arrive(&full[slot]);
                advance();
                break;
            }
            issue_pass(k, 0, true);
            if (ok) issue_pass(k, 1, false);
        }
        if (!ok) {
            atomicExch(prm.ws.abort_flag, 1u);
            // consumers gone: let every copy still in flight land before exit
            const uint64_t first = fills > (uint64_t)nstage ? fills - nstage : 0;
            for (uint64_t u = first; u < fills; ++u)
                mbar_wait_bounded(&full[u % nstage], (unsigned)((u / nstage) & 1), ka.status);
        }
        return;
    }

    if (warp == NW + 1) {
        // ---- look-back warp: each item's incoming state, ahead of pass 0's end
        for (int64_t n = 0;; ++n) {
            const int q = (int)(n % R);
            const int h = (int)(n & 1);
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&item_full[q], (unsigned)((n / R) & 1), ka.status))) break;
            const int64_t k = s_item[q];
            __syncwarp();
            if (lane == 0) mbar_arrive(&item_empty[q]);
            if (k < 0) break;
            const int64_t p = k / prm.nstrips;
            const int64_t rs = k - p * prm.nstrips;
            const int64_t b = rs / prm.spr;
            const int64_t strip = rs - b * prm.spr;
            float x[CPL];
            if (p == 0) {
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    const int64_t gc = strip * WS + lane * CPL + c;
                    x[c] = (ka.e0 != nullptr && gc < ka.hd) ? static_cast<const float*>(ka.e0)[b * ka.hd + gc] : 0.0f;
                }
            } else {
                resolve_incoming<WS, CPL, NW>(prm.ws, ka.status, k, prm.nstrips, p, lane, x);
            }
            // hand the state over once the consumers have read the previous
            // item's from this buffer
            if (n >= 2 &&
                !__all_sync(0xffffffffu, mbar_wait_bounded(&x_empty[h], (unsigned)((n / 2 - 1) & 1), ka.status)))
                break;
#pragma unroll
            for (int c = 0; c < CPL; ++c) s_x[h * WS + lane * CPL + c] = x[c];
            __syncwarp();
            if (lane == 0) mbar_arrive(&x_full[h]);
        }
        return;
    }

    // ---- consumers ----------------------------------------------------------
    const int cw = (warp * 32 + lane) * V;  // first channel of this lane within the strip
    float* const agg_a = static_cast<float*>(prm.ws.agg_a);
    float* const agg_b = static_cast<float*>(prm.ws.agg_b);
    float* const pref = static_cast<float*>(prm.ws.pref);
    int slot = 0;
    unsigned parity = 0;
    auto wait_full = [&]() -> bool {
        return __all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], parity, ka.status));
    };
    auto release = [&]() {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == nstage) {
            slot = 0;
            parity ^= 1u;
        }
    };
    // geometry of an item for this lane
    struct Item {
        int64_t k, p, b, gc, pbeg, pend, ntt;
        bool valid;
    };
    auto item_of = [&](int64_t k) {
        Item it;
        it.k = k;
        it.p = k / prm.nstrips;
        const int64_t rs = k - it.p * prm.nstrips;
        it.b = rs / prm.spr;
        it.gc = (rs - it.b * prm.spr) * WS + cw;
        it.valid = it.gc < ka.hd;  // hd is a multiple of V (16-byte rows)
        it.pbeg = it.p * prm.plen;
        it.pend = it.pbeg + prm.plen < ka.T ? it.pbeg + prm.plen : ka.T;
        it.ntt = (it.pend - it.pbeg + LT - 1) / LT;
        return it;
    };
    bool ok = true;
    // pass 0 of `it` (its first tile already waited for): the aggregate from
    // a zero state, published for this warp's channels
    auto pass0 = [&](const Item& it, float (&ea)[V], float (&pa)[V]) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
            ea[i] = 0.0f;
            pa[i] = 1.0f;
        }
        for (int64_t j = 0; j < it.ntt; ++j) {
            if (j > 0 && !wait_full()) {
                ok = false;
                return;
            }
            const char* sA = smem + (size_t)slot * Cfg::stage_bytes() + cw * (int)sizeof(T);
            const char* sB = sA + LT * Cfg::ROW;
            const int64_t t0 = it.pbeg + j * LT;
            const int nrows = (int)(it.pend - t0 < LT ? it.pend - t0 : LT);
            if (nrows == LT) {
#pragma unroll
                for (int r = 0; r < LT; ++r) {
                    float a[V], bb[V];
                    load_smem<T, V>(sA + r * Cfg::ROW, a);
                    load_smem<T, V>(sB + r * Cfg::ROW, bb);
                    vfma(ea, a, ea, bb);
                    vmul(pa, pa, a);
                }
            } else {
                for (int r = 0; r < nrows; ++r) {
                    float a[V], bb[V];
                    load_smem<T, V>(sA + r * Cfg::ROW, a);
                    load_smem<T, V>(sB + r * Cfg::ROW, bb);
                    vfma(ea, a, ea, bb);
                    vmul(pa, pa, a);
                }
            }
            release();
        }
        if (it.p > 0) {
#pragma unroll
            for (int i = 0; i < V; ++i) {
                agg_a[it.k * WS + cw + i] = pa[i];
                agg_b[it.k * WS + cw + i] = ea[i];
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) red_release_add(prm.ws.flags + it.k, kFlagAgg);
        }
    };
    // the incoming state of `it` (the CTA's item number `np`) from the
    // look-back warp, its inclusive prefix published, then pass 1
    auto pass1 = [&](const Item& it, int64_t np, const float (&ea)[V], const float (&pa)[V]) {
        const int h = (int)(np & 1);
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&x_full[h], (unsigned)((np / 2) & 1), ka.status))) {
            ok = false;
            return;
        }
        float e[V];
#pragma unroll
        for (int i = 0; i < V; ++i) e[i] = s_x[h * WS + cw + i];
        __syncwarp();
        if (lane == 0) mbar_arrive(&x_empty[h]);
#pragma unroll
        for (int i = 0; i < V; ++i) pref[it.k * WS + cw + i] = fmaf(pa[i], e[i], ea[i]);
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_add(prm.ws.flags + it.k, kFlagPfx);
        const int64_t ors = ka.out[0].rs * (int64_t)sizeof(T);
        for (int64_t j = 0; j < it.ntt; ++j) {
            if (!wait_full()) {
                ok = false;
                return;
            }
            const char* sA = smem + (size_t)slot * Cfg::stage_bytes() + cw * (int)sizeof(T);
            const char* sB = sA + LT * Cfg::ROW;
            const int64_t t0 = it.pbeg + j * LT;
            const int nrows = (int)(it.pend - t0 < LT ? it.pend - t0 : LT);
            char* ob = ka.out[0].p + ((it.b * ka.T + t0) * ka.out[0].rs + it.gc) * (int64_t)sizeof(T);
            if (nrows == LT) {
#pragma unroll
                for (int r = 0; r < LT; ++r) {
                    float a[V], bb[V];
                    load_smem<T, V>(sA + r * Cfg::ROW, a);
                    load_smem<T, V>(sB + r * Cfg::ROW, bb);
                    vfma(e, a, e, bb);
                    if (it.valid) store_cs<T, V>(ob + r * ors, e);
                }
            } else {
                for (int r = 0; r < nrows; ++r) {
                    float a[V], bb[V];
                    load_smem<T, V>(sA + r * Cfg::ROW, a);
                    load_smem<T, V>(sB + r * Cfg::ROW, bb);
                    vfma(e, a, e, bb);
                    if (it.valid) store_cs<T, V>(ob + r * ors, e);
                }
            }
            release();
        }
        if (it.p == prm.npiece - 1 && ka.e_last != nullptr && it.valid) {
#pragma unroll
            for (int i = 0; i < V; ++i) static_cast<float*>(ka.e_last)[it.b * ka.hd + it.gc + i] = e[i];
        }
    };
    for (int64_t n = 0; ok; ++n) {
        const int q = (int)(n % R);
        // the first tile of the next item carries its index (or the end marker)
        if (!wait_full()) {
            ok = false;
            break;
        }
        const int64_t k = s_item[q];
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[q]);
        if (k < 0) break;
        const Item it = item_of(k);
        float ea[V], pa[V];
        pass0(it, ea, pa);
        if (!ok) break;
        pass1(it, n, ea, pa);
    }
    if (!ok && lane == 0) atomicExch(prm.ws.abort_flag, 1u);
}

struct ChainLayout {
    size_t flags_off, agg_a_off, agg_b_off, pref_off, total;
};

size_t chain_round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// flags [items], then aggregates (a, b) and inclusive prefixes [items][WS] floats
ChainLayout chain_layout(int64_t nunits, int wch) {
    ChainLayout L;
    L.flags_off = 256;
    L.agg_a_off = chain_round_up(L.flags_off + 4 * (size_t)nunits, 256);
    const size_t d = chain_round_up((size_t)nunits * wch * sizeof(float), 256);
    L.agg_b_off = L.agg_a_off + d;
    L.pref_off = L.agg_b_off + d;
    L.total = L.pref_off + d;
    return L;
}

// Steps per piece: the pieces that all resident CTAs hold between their two
// passes (grid x piece x row bytes of A and B) stay within 80 MB of the
// 126 MB L2, and a piece is at least four tiles.  (On [4, 262144, 32, 64]
// bf16 with the look-back inside the consumer warps: 2 CTAs an SM at 40 MB,
// 2.93 TB/s; 4 at 40 MB, 3.40; 4 at 80 MB, 3.91; 4 at 100 MB, 3.96.)
int64_t chain_piece_len(int64_t row_bytes_ab, int grid) {
    constexpr int64_t kL2Budget = 80ll << 20;
    int64_t plen = kL2Budget / ((int64_t)grid * row_bytes_ab);
    plen = plen / 32 * 32;
    return plen < 128 ? 128 : (plen > 1024 ? 1024 : plen);
}

template <typename T>
int chain_occupancy(int dev, int nstage) {
    using Cfg = ChainCfg<T, kChainNW>;
    static std::atomic<int> cache[16][9];
    if (dev < 0 || dev >= 16 || nstage < 2 || nstage > 8) return 0;
    std::atomic<int>& slot = cache[dev][nstage];
    const int known = slot.load(std::memory_order_relaxed);
    if (known != 0) return known < 0 ? 0 : known;
    int per_sm = 0;
    const size_t smem = Cfg::smem_bytes(nstage);
    if (cudaFuncSetAttribute(chain_scan_kernel<T, kChainNW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_scan_kernel<T, kChainNW>, Cfg::NT,
                                                      smem) == cudaSuccess &&
        per_sm > 0) {
        slot.store(per_sm, std::memory_order_relaxed);
    } else {
        slot.store(-1, std::memory_order_relaxed);
        per_sm = 0;
    }
    return per_sm;
}

constexpr int kChainStages = 3;
constexpr int kChainCtasPerSm = 4;

// The plan of a chained scan: grid, piece length, piece count, units.
struct ChainPlan {
    int grid = 0;
    int64_t plen = 0, npiece = 0, nstrips = 0, spr = 0;
    ChainLayout L{};
};

template <typename T>
ChainPlan chain_plan(int64_t nb, int64_t T_, int64_t hd, int sms) {
    using Cfg = ChainCfg<T, kChainNW>;
    ChainPlan c;
    c.grid = kChainCtasPerSm * sms;
    c.spr = (hd + Cfg::WS - 1) / Cfg::WS;
    c.nstrips = nb * c.spr;
    c.plen = chain_piece_len(2 * Cfg::ROW, c.grid);
    c.npiece = (T_ + c.plen - 1) / c.plen;
    c.L = chain_layout(c.npiece * c.nstrips, Cfg::WS);
    return c;
}

template <typename T>
int chain_launch_typed(const ScanCall& call, bool* taken) {
    using Cfg = ChainCfg<T, kChainNW>;
    *taken = false;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sm_count(dev);
    const ChainPlan pl = chain_plan<T>(call.a.nb, call.a.T, call.a.hd, sms);
    if (call.ws == nullptr || call.ws_bytes < pl.L.total || (reinterpret_cast<uintptr_t>(call.ws) & 255u))
        return ESA_OK;  // not taken: the caller's other paths need less scratch
    if (chain_occupancy<T>(dev, kChainStages) < kChainCtasPerSm) return ESA_OK;
    ChainParams prm{};
    prm.a = call.a;
    prm.spr = pl.spr;
    prm.nstrips = pl.nstrips;
    prm.npiece = pl.npiece;
    prm.plen = pl.plen;
    prm.nitems = pl.npiece * pl.nstrips;
    prm.nstage = kChainStages;
    char* ws = static_cast<char*>(call.ws);
    prm.ws.ticket = reinterpret_cast<unsigned*>(ws);
    prm.ws.abort_flag = reinterpret_cast<unsigned*>(ws) + 1;
    prm.ws.flags = reinterpret_cast<unsigned*>(ws + pl.L.flags_off);
    prm.ws.agg_a = ws + pl.L.agg_a_off;
    prm.ws.agg_b = ws + pl.L.agg_b_off;
    prm.ws.pref = ws + pl.L.pref_off;
    CUtensorMap maps[2];
    memset(maps, 0, sizeof(maps));
    for (int a = 0; a < 2; ++a) {
        std::string err;
        if (!encode_strip_map(&maps[a], call.te, call.a.in[a].p, call.a.nb, call.a.T, call.a.hd, call.a.in[a].rs,
                              Cfg::WS, Cfg::LT, &err, 256))
            return set_error(ESA_ERR_CUDA, "tensor map: " + err);
    }
    cudaError_t e = cudaMemsetAsync(ws, 0, pl.L.agg_a_off, call.stream);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("workspace reset: ") + cudaGetErrorString(e));
    const size_t smem = Cfg::smem_bytes(kChainStages);
    e = cudaFuncSetAttribute(chain_scan_kernel<T, kChainNW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("chain smem attribute: ") + cudaGetErrorString(e));
    int grid = pl.grid;
    if ((int64_t)grid > prm.nitems) grid = (int)prm.nitems;
    *taken = true;
    note_scan_path(ESA_PATH_CHAIN);
    chain_scan_kernel<T, kChainNW><<<grid, Cfg::NT, smem, call.stream>>>(prm, maps[0], maps[1]);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("chain scan launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

}  // namespace

// Shapes the chained scan serves: 16- or 32-bit data whose lane-serial
// strips would give fewer than one consumer warp per SM, over a time axis of
// at least 8192 steps (the shapes the split scan serves otherwise).
bool chain_applies_dims(int64_t nb, int64_t T, int64_t hd, int es) {
    if (es != 2 && es != 4) return false;
    const int64_t lane_ws = 32 * (es == 2 ? 2 : 1);  // channels per consumer warp
    const int64_t warps = nb * ((hd + lane_ws - 1) / lane_ws);
    return warps < 148 && T >= 8192;
}

// Taken for the plain forward scan (not a summary, not a resumed scan).
bool chain_applies(const ScanCall& c) {
    if (c.kind != Kind::FwdPlain || c.summ || c.resume || c.tin != c.te) return false;
    return chain_applies_dims(c.a.nb, c.a.T, c.a.hd, dtype_size(c.te));
}

size_t chain_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int es) {
    if (!chain_applies_dims(nb, T, hd, es)) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sm_count(dev) > 0 ? device_sm_count(dev) : 148;
    return es == 2 ? chain_plan<__half>(nb, T, hd, sms).L.total : chain_plan<float>(nb, T, hd, sms).L.total;
}

int chain_scan_launch(const ScanCall& c, bool* taken) {
    *taken = false;
    if (!chain_applies(c)) return ESA_OK;
    switch (c.te) {
        case ESA_DTYPE_F16: return chain_launch_typed<__half>(c, taken);
        case ESA_DTYPE_BF16: return chain_launch_typed<__nv_bfloat16>(c, taken);
        case ESA_DTYPE_F32: return chain_launch_typed<float>(c, taken);
        default: return ESA_OK;
    }
}

}  // namespace esa
