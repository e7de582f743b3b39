// esa_lookback.cuh -- single-pass decoupled look-back (Merrill & Garland
// 2016) over tiles of VEC-channel lanes, shared by the time-parallel scans.
//
// Tile k publishes its aggregate (flag AGG), composes the aggregates of its
// predecessors k - nct, k - 2 nct, ... back to the nearest inclusive prefix
// (flag PFX), and publishes its own inclusive prefix.  Tiles are claimed from
// an atomic ticket in processing order, so every predecessor is owned by a
// running or finished CTA and every wait ends; each wait is still bounded.
#pragma once

#include "esa_scan_common.cuh"

namespace esa {

constexpr unsigned FLAG_AGG = 1, FLAG_PFX = 2;

struct Workspace {
    unsigned* ticket;
    unsigned* abort_flag;  // set by the first wait of this launch that runs out
    unsigned* flags;
    void* agg_a;
    void* agg_b;
    void* pref;
};

// Decoupled lookback, run by one warp.  Publishes the tile aggregate (ta, tb),
// resolves the incoming carry x, publishes the inclusive prefix ta*x + tb.
template <typename acc, int VEC>
__device__ __forceinline__ void lookback(const Workspace& ws, unsigned* status, int64_t k,
                                         int64_t nct, int64_t gproc, int wch, int lane,
                                         const acc (&ta)[VEC], const acc (&tb)[VEC],
                                         const acc (&x0)[VEC], acc (&x)[VEC], acc (&pfx)[VEC]) {
    acc* agg_a = static_cast<acc*>(ws.agg_a);
    acc* agg_b = static_cast<acc*>(ws.agg_b);
    acc* pref = static_cast<acc*>(ws.pref);
    const int64_t off = k * wch + lane * VEC;
    if (gproc == 0) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) x[i] = x0[i];
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            agg_a[off + i] = ta[i];
            agg_b[off + i] = tb[i];
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu(ws.flags + k, FLAG_AGG);

        acc ca[VEC], cb[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            ca[i] = acc(1);
            cb[i] = acc(0);
        }
        int64_t consumed = 0;
        unsigned long long t_start = 0;
        unsigned spins = 0;
        while (true) {
            const int64_t i = consumed + lane;
            unsigned f = 0;
            if (i < gproc) f = ld_acquire_gpu(ws.flags + (k - (i + 1) * nct));
            const unsigned nz = __ballot_sync(0xffffffffu, f != 0);
            const unsigned ip = __ballot_sync(0xffffffffu, f == FLAG_PFX);
            __syncwarp();
            const int m = (nz == 0xffffffffu) ? 32 : (__ffs(~nz) - 1);
            const unsigned mm = (m >= 32) ? 0xffffffffu : ((1u << m) - 1u);
            const unsigned pm = ip & mm;
            const int p = pm ? (__ffs(pm) - 1) : -1;
            const int nagg = (p >= 0) ? p : m;
            // the prefix's load and the aggregates' loads go out together,
            // the aggregates a few predecessors at a time (independent loads
            // in flight instead of one L2 round trip per predecessor); the
            // composition order is unchanged
            acc pv[VEC];
            if (p >= 0) {
                const int64_t jo = (k - (consumed + p + 1) * nct) * wch + lane * VEC;
#pragma unroll
                for (int v = 0; v < VEC; ++v) pv[v] = __ldcg(pref + jo + v);
            }
            // (two at a time for 32-byte lane vectors, which keep more in registers)
            constexpr int PB = VEC * (int)sizeof(acc) >= 32 ? 2 : 4;
            for (int q0 = 0; q0 < nagg; q0 += PB) {
                acc ra[PB][VEC], rb[PB][VEC];
#pragma unroll
                for (int u = 0; u < PB; ++u) {
                    if (q0 + u < nagg) {
                        const int64_t jo = (k - (consumed + q0 + u + 1) * nct) * wch + lane * VEC;
#pragma unroll
                        for (int v = 0; v < VEC; ++v) {
                            ra[u][v] = __ldcg(agg_a + jo + v);
                            rb[u][v] = __ldcg(agg_b + jo + v);
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < PB; ++u) {
                    if (q0 + u < nagg) {
#pragma unroll
                        for (int v = 0; v < VEC; ++v) {
                            cb[v] = ca[v] * rb[u][v] + cb[v];
                            ca[v] = ca[v] * ra[u][v];
                        }
                    }
                }
            }
            if (p >= 0) {
#pragma unroll
                for (int v = 0; v < VEC; ++v) x[v] = ca[v] * pv[v] + cb[v];
                break;
            }
            consumed += m;
            if (m == 0) {
                if (spins == 0) t_start = globaltimer_ns();
                ++spins;
                __nanosleep(64);
                // give up after the wait budget, or at once if another wait of
                // this launch already gave up (no cascade of full budgets)
                bool expired = (spins > kWaitMaxIters) ||
                               (globaltimer_ns() - t_start > kWaitBudgetNs) ||
                               (*(volatile unsigned*)ws.abort_flag != 0u);
                expired = __shfl_sync(0xffffffffu, expired, 0);
                if (expired) {
                    if (lane == 0) {
                        atomicOr(status, ESA_STATUS_LOOKBACK_TIMEOUT);
                        atomicExch(ws.abort_flag, 1u);
                    }
#pragma unroll
                    for (int v = 0; v < VEC; ++v) x[v] = acc(0);
                    break;
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        pfx[i] = ta[i] * x[i] + tb[i];
        pref[off + i] = pfx[i];
    }
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_gpu(ws.flags + k, FLAG_PFX);
}

}  // namespace esa
