// esa_scan_lookback.cu -- time-parallel chunked scan with decoupled lookback.
//
// Used when the problem has too few channels to fill the GPU with channel
// strips (esa_scan_strip.cu), e.g. short prompts, small batches or one long
// sequence: parallelism then has to come from the time axis.
//
// A tile is (time chunk g, channel tile): LT = S * nwarp steps by WCH = 32*VEC
// channels of one batch row.  Lane l of every warp owns VEC consecutive
// channels (one 16-byte vector of the widest element type); warp w owns steps
// [w*S, (w+1)*S).  One warp stages the NEXT tile into shared memory with bulk
// asynchronous copies (cp.async.bulk, L2 evict-first) completing on an
// mbarrier while the CTA works on the current tile (2 stages).
//
// Carries (Merrill & Garland 2016, single-pass decoupled lookback):
//   phase 1: each warp composes its S steps into an affine aggregate;
//   cross-warp: aggregates through shared memory -> per-warp exclusive prefix
//            and the tile aggregate;
//   lookback: warp 0 publishes the tile aggregate (flag AGG), reads the flags
//            of up to 32 predecessor tiles at once (one per lane), composes
//            aggregates back to the nearest inclusive prefix (flag PFX) and
//            publishes its own inclusive prefix;
//   phase 3: every warp re-runs its S steps from its exact incoming state.
// Tiles come from an atomic ticket in (time chunk, channel tile) order, so
// every predecessor of a tile is owned by a CTA that is already running, and a
// tile publishes its aggregate before it waits: the waits always end.  Each
// wait is still bounded (one second of %globaltimer plus an iteration cap); on
// expiry the kernel raises the device status word, marks the launch aborted
// (later waits of the launch give up at once) and finishes with an undefined
// but finite result.
#include <string>

#include "esa_lookback.cuh"

namespace esa {

namespace {

constexpr int S = 4;  // time steps per warp per tile

struct Geometry {
    int64_t ncpr;    // channel tiles per batch row
    int64_t nct;     // channel tiles in total
    int64_t G;       // time chunks
    int64_t ntiles;  // G * nct
    int nwarp;       // warps per CTA; LT = S * nwarp
};


struct LbParams {
    KArgs a;
    Geometry geo;
    Workspace ws;
};

template <Kind K, typename Tin, typename Te>
struct LbCfg {
    using P = Policy<K, Tin, Te>;
    static constexpr int WCH = 32 * P::VEC;
    static __host__ __device__ constexpr int row_bytes(int i) { return WCH * P::es(i); }
    static __host__ __device__ constexpr int stage_row_bytes() {
        int s = 0;
        for (int i = 0; i < P::NIN; ++i) s += row_bytes(i);
        return s;
    }
};


struct TileCoord {
    int64_t gproc;  // processing index of the time chunk (lookback order)
    int64_t g;      // time chunk
    int64_t b;      // batch row
    int64_t cb;     // first channel
    int width;      // valid channels
    int64_t t0;     // first step
};

template <bool REV>
__device__ __forceinline__ TileCoord tile_coord(const Geometry& geo, int64_t hd, int64_t k, int wch,
                                                int lt) {
    TileCoord tc;
    tc.gproc = k / geo.nct;
    const int64_t ct = k - tc.gproc * geo.nct;
    tc.g = REV ? (geo.G - 1 - tc.gproc) : tc.gproc;
    tc.b = ct / geo.ncpr;
    tc.cb = (ct - tc.b * geo.ncpr) * wch;
    const int64_t w = hd - tc.cb;
    tc.width = (int)(w < wch ? w : wch);
    tc.t0 = tc.g * lt;
    return tc;
}

// Issue the bulk copies of tile k into stage buffer `stage` (one warp).
template <Kind K, typename Tin, typename Te>
__device__ __forceinline__ void issue_tile(const LbParams& prm, int64_t k, char* stage,
                                           uint64_t* bar, int lane, uint64_t policy) {
    using P = Policy<K, Tin, Te>;
    using C = LbCfg<K, Tin, Te>;
    const int lt = S * prm.geo.nwarp;
    const int64_t T = prm.a.T;
    const TileCoord tc = tile_coord<P::REV>(prm.geo, prm.a.hd, k, C::WCH, lt);
    // rows r with step t = t0 + r < T whose source row t + shift is >= 0
    const int64_t rem = T - tc.t0;
    const int nvalid = (int)(rem < lt ? rem : lt);
    unsigned total = 0;
#pragma unroll
    for (int a = 0; a < P::NIN; ++a) {
        const int n = (P::shift(a) < 0 && tc.t0 == 0) ? nvalid - 1 : nvalid;
        total += (unsigned)n * (unsigned)(tc.width * P::es(a));
    }
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
    __syncwarp();
    int abase = 0;
#pragma unroll
    for (int a = 0; a < P::NIN; ++a) {
        const int rb = C::row_bytes(a);
        const int bytes = tc.width * P::es(a);
        for (int r = lane; r < lt; r += 32) {
            const int64_t t = tc.t0 + r;
            const int64_t tr = t + P::shift(a);
            if (t < T && tr >= 0) {
                const char* src = prm.a.in[a].p +
                                  ((tc.b * T + tr) * prm.a.in[a].rs + tc.cb) * (int64_t)P::es(a);
                bulk_g2s(stage + abase + r * rb, src, (unsigned)bytes, bar, policy);
            }
        }
        abase += lt * rb;
    }
}

template <Kind K, typename Tin, typename Te>
__global__ void __launch_bounds__(512) lookback_scan_kernel(const LbParams prm) {
    using P = Policy<K, Tin, Te>;
    using C = LbCfg<K, Tin, Te>;
    using acc = typename P::acc;
    constexpr int VEC = P::VEC;
    constexpr int WCH = C::WCH;
    const Geometry& geo = prm.geo;
    const KArgs& ka = prm.a;
    const int nwarp = geo.nwarp;
    const int lt = S * nwarp;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    extern __shared__ __align__(128) char smem[];
    const int stage_bytes = lt * C::stage_row_bytes();
    acc* sagg_a = reinterpret_cast<acc*>(smem + 2 * stage_bytes);
    acc* sagg_b = sagg_a + nwarp * WCH;
    acc* scarry = sagg_b + nwarp * WCH;
    uint64_t* bars = reinterpret_cast<uint64_t*>(scarry + WCH);
    // s_tile[0]: first ticket; s_tile[1 + (it & 1)]: ticket of the tile after
    // the one processed in iteration `it` (double-buffered: the write of
    // iteration `it` never races the read of iteration `it`)
    int64_t* s_tile = reinterpret_cast<int64_t*>(bars + 2);

    const uint64_t policy = policy_evict_first();
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbarrier_init();
        s_tile[0] = atomicAdd(prm.ws.ticket, 1u);
    }
    __syncthreads();
    int64_t k = s_tile[0];
    unsigned outstanding = 0;  // stages with copies issued and not yet waited for
    if (k < geo.ntiles) {
        if (warp == 0) issue_tile<K, Tin, Te>(prm, k, smem, &bars[0], lane, policy);
        outstanding |= 1u;
    }
    if (threadIdx.x == 0) s_tile[1] = atomicAdd(prm.ws.ticket, 1u);
    __syncthreads();

    unsigned phase_bits = 0;
    int it = 0;
    bool healthy = true;
    const int c = lane * VEC;
    while (k < geo.ntiles) {
        const int st = it & 1;
        const int64_t kn = s_tile[1 + (it & 1)];
        if (kn < geo.ntiles) {
            if (warp == nwarp - 1)
                issue_tile<K, Tin, Te>(prm, kn, smem + (st ^ 1) * stage_bytes, &bars[st ^ 1], lane, policy);
            outstanding |= 1u << (st ^ 1);
        }
        unsigned knn = 0;
        if (threadIdx.x == 0) knn = atomicAdd(prm.ws.ticket, 1u);

        const TileCoord tc = tile_coord<P::REV>(geo, ka.hd, k, WCH, lt);
        if (mbar_wait_bounded(&bars[st], (phase_bits >> st) & 1u, ka.status)) {
            phase_bits ^= (1u << st);
            outstanding &= ~(1u << st);
        } else {
            healthy = false;
            atomicExch(prm.ws.abort_flag, 1u);
        }

        const char* sbase = smem + st * stage_bytes;
        auto row_ptrs = [&](int r, const char* (&rows)[4]) {
            int abase = 0;
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                if (a < P::NIN) {
                    rows[a] = sbase + abase + r * C::row_bytes(a) + c * P::es(a);
                    abase += lt * C::row_bytes(a);
                } else {
                    rows[a] = nullptr;
                }
            }
        };

        // ---- phase 1 ------------------------------------------------------
        typename P::template Cache<S> cache;
        acc pa[VEC], pb[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            pa[i] = acc(1);
            pb[i] = acc(0);
        }
#pragma unroll
        for (int ss = 0; ss < S; ++ss) {
            const int s = P::REV ? (S - 1 - ss) : ss;
            const int r = warp * S + s;
            if (tc.t0 + r < ka.T) {
                const char* rows[4];
                row_ptrs(r, rows);
                acc a[VEC], b[VEC];
                step_coef<K, Tin, Te, S>(rows, ka, a, b, cache, s);
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    pb[i] = a[i] * pb[i] + b[i];
                    pa[i] = a[i] * pa[i];
                }
            }
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            sagg_a[warp * WCH + c + i] = pa[i];
            sagg_b[warp * WCH + c + i] = pb[i];
        }
        if (threadIdx.x == 0) s_tile[1 + ((it + 1) & 1)] = (int64_t)knn;
        __syncthreads();

        // ---- cross-warp exclusive prefix ------------------------------------
        acc ea[VEC], eb[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            ea[i] = acc(1);
            eb[i] = acc(0);
        }
        for (int n = 0; n < nwarp; ++n) {
            const int w = P::REV ? (nwarp - 1 - n) : n;
            if (w == warp) break;
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                const acc aw = sagg_a[w * WCH + c + i];
                const acc bw = sagg_b[w * WCH + c + i];
                eb[i] = aw * eb[i] + bw;
                ea[i] = aw * ea[i];
            }
        }

        // ---- lookback (warp 0) ----------------------------------------------
        if (warp == 0) {
            acc ta[VEC], tb[VEC], x0[VEC], x[VEC], pfx[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                ta[i] = acc(1);
                tb[i] = acc(0);
            }
            for (int n = 0; n < nwarp; ++n) {
                const int w = P::REV ? (nwarp - 1 - n) : n;
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const acc aw = sagg_a[w * WCH + c + i];
                    const acc bw = sagg_b[w * WCH + c + i];
                    tb[i] = aw * tb[i] + bw;
                    ta[i] = aw * ta[i];
                }
            }
#pragma unroll
            for (int i = 0; i < VEC; ++i) x0[i] = acc(0);
            if (!P::REV && ka.e0 != nullptr && c < tc.width) {
                const acc* e0 = static_cast<const acc*>(ka.e0) + tc.b * ka.hd + tc.cb + c;
#pragma unroll
                for (int i = 0; i < VEC; ++i) x0[i] = e0[i];
            }
            lookback<acc, VEC>(prm.ws, ka.status, k, geo.nct, tc.gproc, WCH, lane, ta, tb, x0, x, pfx);
#pragma unroll
            for (int i = 0; i < VEC; ++i) scarry[c + i] = x[i];
            // forward: the last chunk's inclusive prefix is E_{T-1}
            if (!P::REV && ka.e_last != nullptr && tc.g == geo.G - 1 && c < tc.width) {
                acc* el = static_cast<acc*>(ka.e_last) + tc.b * ka.hd + tc.cb + c;
#pragma unroll
                for (int i = 0; i < VEC; ++i) el[i] = pfx[i];
            }
        }
        __syncthreads();

        // ---- phase 3 ------------------------------------------------------
        {
            const bool valid = c < tc.width;
            acc e[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) e[i] = ea[i] * scarry[c + i] + eb[i];
#pragma unroll
            for (int ss = 0; ss < S; ++ss) {
                const int s = P::REV ? (S - 1 - ss) : ss;
                const int r = warp * S + s;
                const int64_t t = tc.t0 + r;
                if (t < ka.T) {
                    const char* rows[4];
                    row_ptrs(r, rows);
                    const int64_t orow = tc.b * ka.T + t;
                    step_apply<K, Tin, Te, S>(
                        rows, ka, tc.b, t, tc.cb + c, valid, e, cache, s,
                        ka.out[0].p + (orow * ka.out[0].rs + tc.cb + c) * (int64_t)P::OES,
                        ka.out[1].p + (orow * ka.out[1].rs + tc.cb + c) * (int64_t)P::OES);
                }
            }
            // reverse: H_0 = A_0 G_0 is the gradient w.r.t. the initial state
            if (P::REV && ka.e_last != nullptr && tc.t0 == 0 && warp == 0 && valid) {
                acc* de0 = static_cast<acc*>(ka.e_last) + tc.b * ka.hd + tc.cb + c;
#pragma unroll
                for (int i = 0; i < VEC; ++i) de0[i] = e[i];
            }
        }
        // stage st and the shared scratch are free again; stop the whole CTA
        // if any thread's copy wait ran out
        if (!__syncthreads_and(healthy)) break;
        k = kn;
        ++it;
    }
    // after a failed wait, give every copy still in flight one more bounded
    // wait, so that no bulk copy targets this CTA's shared memory after exit
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
        if (outstanding & (1u << s2)) mbar_wait_bounded(&bars[s2], (phase_bits >> s2) & 1u, ka.status);
}

// Steps per tile for a given compass: 16, 32 or 64 (nearest).  Kernels that
// stage four arrays (the fused reverse scan) cap it at 32 so that two stages
// fit in shared memory; the workspace is sized for the capped value (the
// larger tile count).
// Steps per tile: compass rounded up to 32 or 64.  (16-step tiles made the
// look-back chains twice as long for nothing: a gated fp16 scan of
// [1, 512, 1024] took 24.1 us per call against 20.6 us with 32-step tiles,
// [1, 2048, 768] 39.0 against 32.0, [1, 256, 1024] 18.5 against 18.6.)
int lt_for(int compass, int nin) {
    int lt = compass <= 32 ? 32 : 64;
    if (nin >= 4 && lt > 32) lt = 32;
    return lt;
}

Geometry make_geometry(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass, int nin) {
    Geometry g;
    const int wch = 32 * (16 / wide_es);
    const int lt = lt_for(compass, nin);
    g.ncpr = (hd + wch - 1) / wch;
    g.nct = nb * g.ncpr;
    g.G = (T + lt - 1) / lt;
    g.ntiles = g.G * g.nct;
    g.nwarp = lt / S;
    return g;
}

struct WsLayout {
    size_t flags_off, agg_a_off, agg_b_off, pref_off, total;
};

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

WsLayout ws_layout(int64_t ntiles, int wch, size_t acc_size) {
    WsLayout L;
    L.flags_off = 256;
    L.agg_a_off = round_up(L.flags_off + 4 * (size_t)ntiles, 256);
    const size_t d = round_up((size_t)ntiles * wch * acc_size, 256);
    L.agg_b_off = L.agg_a_off + d;
    L.pref_off = L.agg_b_off + d;
    L.total = L.pref_off + d;
    return L;
}

template <Kind K, typename Tin, typename Te>
size_t smem_bytes_for(int nwarp) {
    using P = Policy<K, Tin, Te>;
    using C = LbCfg<K, Tin, Te>;
    const int lt = S * nwarp;
    size_t b = 2ull * lt * C::stage_row_bytes();
    b += (2ull * nwarp * C::WCH + C::WCH) * sizeof(typename P::acc);
    b += 2 * sizeof(uint64_t) + 3 * sizeof(int64_t);
    return b;
}

template <Kind K, typename Tin, typename Te>
int launch_typed(const ScanCall& call) {
    using P = Policy<K, Tin, Te>;
    using C = LbCfg<K, Tin, Te>;
    using acc = typename P::acc;
    LbParams prm{};
    prm.a = call.a;
    prm.geo = make_geometry(call.a.nb, call.a.T, call.a.hd, P::WIDE, call.compass, P::NIN);
    const Geometry& geo = prm.geo;
    const WsLayout L = ws_layout(geo.ntiles, C::WCH, sizeof(acc));
    if (call.ws == nullptr || call.ws_bytes < L.total || (reinterpret_cast<uintptr_t>(call.ws) & 15u))
        return set_error(ESA_ERR_WORKSPACE, "workspace missing, misaligned or smaller than esa_scan_workspace_bytes()");
    char* ws = static_cast<char*>(call.ws);
    prm.ws.ticket = reinterpret_cast<unsigned*>(ws);
    prm.ws.abort_flag = reinterpret_cast<unsigned*>(ws) + 1;
    prm.ws.flags = reinterpret_cast<unsigned*>(ws + L.flags_off);
    prm.ws.agg_a = ws + L.agg_a_off;
    prm.ws.agg_b = ws + L.agg_b_off;
    prm.ws.pref = ws + L.pref_off;
    cudaError_t e = cudaMemsetAsync(ws, 0, L.agg_a_off, call.stream);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("workspace reset: ") + cudaGetErrorString(e));

    const size_t smem = smem_bytes_for<K, Tin, Te>(geo.nwarp);
    if (smem > 232448) return set_error(ESA_ERR_INVALID_ARGUMENT, "tile configuration exceeds shared memory");
    int dev = 0;
    cudaGetDevice(&dev);
    e = cudaFuncSetAttribute(lookback_scan_kernel<K, Tin, Te>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("smem attribute: ") + cudaGetErrorString(e));
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lookback_scan_kernel<K, Tin, Te>, 32 * geo.nwarp, smem);
    if (e != cudaSuccess || per_sm <= 0) return set_error(ESA_ERR_CUDA, "lookback scan kernel cannot be resident");
    int64_t grid = (int64_t)per_sm * device_sm_count(dev);
    if (grid > geo.ntiles) grid = geo.ntiles;
    note_scan_path(ESA_PATH_LOOKBACK);
    lookback_scan_kernel<K, Tin, Te><<<(unsigned)grid, 32 * geo.nwarp, smem, call.stream>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("lookback scan launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

}  // namespace

size_t lookback_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass) {
    // sized for the smallest tile any kernel uses at this compass (most tiles)
    const Geometry g = make_geometry(nb, T, hd, wide_es, compass, 4);
    const size_t acc_size = wide_es == 8 ? 8 : 4;
    return ws_layout(g.ntiles, 32 * (16 / wide_es), acc_size).total;
}

int lookback_scan_launch(const ScanCall& c) {
    return dispatch_dtype(c.tin, [&](auto ti) -> int {
        using Tin = decltype(ti);
        return dispatch_dtype(c.te, [&](auto tee) -> int {
            using Te = decltype(tee);
            switch (c.kind) {
                case Kind::FwdPlain:
                    if constexpr (std::is_same<Tin, Te>::value) return launch_typed<Kind::FwdPlain, Tin, Te>(c);
                    break;
                case Kind::RevPlain:
                    if constexpr (std::is_same<Tin, Te>::value) return launch_typed<Kind::RevPlain, Tin, Te>(c);
                    break;
                case Kind::FwdGated: return launch_typed<Kind::FwdGated, Tin, Te>(c);
                case Kind::RevGated: return launch_typed<Kind::RevGated, Tin, Te>(c);
                case Kind::FwdSummary: break;
            }
            return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "plain scans need one dtype");
        });
    });
}

}  // namespace esa
