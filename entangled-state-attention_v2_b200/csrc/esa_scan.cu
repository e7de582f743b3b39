// esa_scan.cu -- single-pass chunked scans of E_t = A_t * E_{t-1} + B_t on sm_100a.
//
// Problem: independent channels (b, c), c < hd, each a length-T affine
// recurrence; data [nb, T, hd] with hd contiguous (the reference's [B,T,H,D]).
//
// Tiling.  A tile is (time chunk g, channel tile ct): LT = S * nwarp steps by
// WCH = 32 * VEC channels of one batch row.  Lane l of every warp owns VEC
// consecutive channels (one 16-byte vector of the widest element type); warp w
// owns steps [w*S, (w+1)*S) of the chunk.  So every warp-row access is a
// contiguous 32*VEC*es-byte segment (fully coalesced) and the sequential work
// per thread is S steps x VEC independent chains.
//
// Data movement.  One warp of the CTA stages the NEXT tile's rows into shared
// memory with bulk asynchronous copies (cp.async.bulk, the TMA engine, L2
// evict-first) completing on an mbarrier, while the CTA works on the current
// tile from the other stage (2 stages).  Each input byte crosses HBM once and
// each output byte is stored once from registers (16-byte coalesced stores),
// so the kernel moves exactly the algorithmic bytes plus the small lookback
// descriptors.
//
// Carries.  Single pass with decoupled lookback (Merrill & Garland 2016):
//   phase 1: each warp composes its S steps into an affine aggregate (a, b);
//   cross-warp: aggregates through shared memory -> per-warp exclusive prefix
//            and the tile aggregate;
//   lookback: warp 0 publishes the tile aggregate (flag AGG), then reads the
//            flags of up to 32 predecessor tiles at once (one per lane) and
//            composes aggregates back to the nearest inclusive prefix (flag
//            PFX); publishes its own inclusive prefix;
//   phase 3: every warp re-runs its S steps from its exact incoming state and
//            writes the outputs.
// Tiles are taken from an atomic ticket in (time chunk, channel tile) order, so
// every predecessor of a tile is owned by a CTA that is already running, and a
// tile publishes its aggregate before it waits on anything: the waits always
// end.  Each wait is still bounded (one second of %globaltimer, plus an
// iteration cap); on expiry the kernel raises the device status word and
// finishes with an undefined but finite result rather than hanging.
//
// Accumulation is in fp32 (fp64 for fp64 data); inputs are read exactly and
// only the outputs are rounded to the storage type.
//
// Reverse direction (gradients).  With H_t = A_t * G_t the backward recurrence
// G_t = dE_t + A_{t+1} G_{t+1} becomes H_t = A_t H_{t+1} + A_t dE_t, an affine
// scan over t descending with per-step coefficients (A_t, A_t dE_t) -- the same
// machinery run on time chunks in descending order.
#include <algorithm>
#include <cstdio>
#include <string>

#include "esa_common.cuh"
#include "esa_internal.h"

namespace esa {

// ---------------------------------------------------------------------------
// Device status word.  Kernels OR ESA_STATUS_* bits into it when a bounded wait
// runs out; esa_device_status() reads (and optionally clears) it.  One copy per
// device: a __device__ variable lives in each context's module.
// ---------------------------------------------------------------------------
__device__ unsigned int g_device_status = 0;

__device__ __forceinline__ void raise_status(unsigned int bits) { atomicOr(&g_device_status, bits); }

// Bounded wait on an mbarrier phase.  Returns false (and raises the device
// error word) if the phase did not complete within the wait budget.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = globaltimer_ns();
    for (unsigned it = 0; it < kWaitMaxIters; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitBudgetNs) break;
    }
    raise_status(ESA_STATUS_COPY_TIMEOUT);
    return false;
}


constexpr int S = 4;  // time steps per warp per tile
constexpr unsigned FLAG_AGG = 1, FLAG_PFX = 2;
constexpr unsigned FULL = 0xffffffffu;

// A row-strided view: element (row, c) at p + (row * rs + c) * sizeof(T),
// row = b * T + t.
struct View {
    const char* p;
    int64_t rs;
};
struct MutView {
    char* p;
    int64_t rs;
};

struct Geometry {
    int64_t nb, T, hd;
    int64_t ncpr;    // channel tiles per batch row
    int64_t nct;     // channel tiles in total
    int64_t G;       // time chunks
    int64_t ntiles;  // G * nct
    int nwarp;       // warps per CTA; LT = S * nwarp
};

struct Workspace {
    unsigned* ticket;
    unsigned* abort_flag;  // set by the first wait of this launch that runs out
    unsigned* flags;
    void* agg_a;
    void* agg_b;
    void* pref;
};

template <typename T, int N>
struct alignas(sizeof(T) * N) VecN {
    T v[N];
};

// ---------------------------------------------------------------------------
// Kernel argument block.  Kind selects the per-step math.
// ---------------------------------------------------------------------------
enum class Kind { FwdPlain, FwdGated, RevPlain, RevGated };

template <Kind K, typename Tin, typename Te>
struct Params {
    View in[4];        // staged inputs (see Policy)
    MutView out[2];    // outputs
    Geometry geo;
    Workspace ws;
    const void* e0;    // acc [nb*hd] or null
    void* e_last;      // fwd: acc [nb*hd] or null;  rev: de0
    float gmin, gmax;
    int round_ab;
};

template <typename T>
__device__ __forceinline__ float round_to(float x) {
    return Elem<T>::to_acc(Elem<T>::from_acc(x));
}
template <typename T>
__device__ __forceinline__ double round_to(double x) {
    return static_cast<double>(Elem<T>::from_acc(static_cast<typename Elem<T>::acc>(x)));
}

// ---------------------------------------------------------------------------
// Per-kind policy: which arrays are staged, the per-step coefficients, and the
// phase-3 update with its outputs.
// ---------------------------------------------------------------------------
template <Kind K, typename Tin, typename Te>
struct Policy {
    static constexpr bool REV = (K == Kind::RevPlain || K == Kind::RevGated);
    static constexpr bool GATED = (K == Kind::FwdGated || K == Kind::RevGated);
    // staged arrays: fwd {in0, in1}; rev plain {A, Eprev, dE}; rev gated {g, v, Eprev, dE}
    static constexpr int NIN = (K == Kind::RevGated) ? 4 : (K == Kind::RevPlain ? 3 : 2);
    using acc = typename std::conditional<(sizeof(Tin) == 8 || sizeof(Te) == 8), double, float>::type;
    static constexpr int WIDE = (sizeof(Tin) > sizeof(Te)) ? sizeof(Tin) : sizeof(Te);
    static constexpr int VEC = 16 / WIDE;
    static constexpr int WCH = 32 * VEC;
    // element size of staged array i
    static __host__ __device__ constexpr int es(int i) {
        return (K == Kind::RevGated) ? (i < 2 ? (int)sizeof(Tin) : (int)sizeof(Te))
               : (K == Kind::RevPlain) ? (int)sizeof(Te)
                                       : (int)sizeof(Tin);
    }
    // row shift of staged array i: Eprev rows are one step behind.
    static __host__ __device__ constexpr int shift(int i) {
        return (K == Kind::RevPlain && i == 1) || (K == Kind::RevGated && i == 2) ? -1 : 0;
    }
    // shared-memory bytes of one staged row of array i
    static __host__ __device__ constexpr int row_bytes(int i) { return WCH * es(i); }
    static __host__ __device__ constexpr int stage_row_bytes() {
        int s = 0;
        for (int i = 0; i < NIN; ++i) s += row_bytes(i);
        return s;
    }
    // register cache carried from phase 1 to phase 3
    struct Cache {
        acc c0[S][GATED ? VEC : 1];
        acc c1[S][(K == Kind::FwdGated) ? VEC : 1];
    };
};

template <typename T, int N, typename A>
__device__ __forceinline__ void load_smem(const char* p, A (&out)[N]) {
    VecN<T, N> v = *reinterpret_cast<const VecN<T, N>*>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = static_cast<A>(Elem<T>::to_acc(v.v[i]));
}

template <typename T, int N, typename A>
__device__ __forceinline__ void store_global(char* p, const A (&in)[N]) {
    VecN<T, N> v;
#pragma unroll
    for (int i = 0; i < N; ++i) v.v[i] = Elem<T>::from_acc(static_cast<typename Elem<T>::acc>(in[i]));
    *reinterpret_cast<VecN<T, N>*>(p) = v;
}

// Per-step coefficients (a, b) of the affine map for step row r (phase 1).
template <Kind K, typename Tin, typename Te, typename P = Policy<K, Tin, Te>>
__device__ __forceinline__ void step_coef(const char* const (&srow)[4], int lane, float gmin,
                                          float gmax, int round_ab, typename P::acc (&a)[P::VEC],
                                          typename P::acc (&b)[P::VEC], typename P::Cache& cache,
                                          int s) {
    using acc = typename P::acc;
    constexpr int VEC = P::VEC;
    if constexpr (K == Kind::FwdPlain) {
        load_smem<Tin, VEC>(srow[0] + lane * VEC * sizeof(Tin), a);
        load_smem<Tin, VEC>(srow[1] + lane * VEC * sizeof(Tin), b);
    } else if constexpr (K == Kind::FwdGated) {
        acc g[VEC], v[VEC];
        load_smem<Tin, VEC>(srow[0] + lane * VEC * sizeof(Tin), g);
        load_smem<Tin, VEC>(srow[1] + lane * VEC * sizeof(Tin), v);
        const acc lo = gmin, span = acc(gmax) - acc(gmin);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            acc A = lo + span * sigmoid_(g[i]);
            acc B = (acc(1) - A) * tanh_(v[i]);
            if (round_ab) {
                A = round_to<Te>(A);
                B = round_to<Te>(B);
            }
            a[i] = A;
            b[i] = B;
            cache.c0[s][i] = A;
            cache.c1[s][i] = B;
        }
    } else if constexpr (K == Kind::RevPlain) {
        acc d[VEC];
        load_smem<Te, VEC>(srow[0] + lane * VEC * sizeof(Te), a);
        load_smem<Te, VEC>(srow[2] + lane * VEC * sizeof(Te), d);
#pragma unroll
        for (int i = 0; i < VEC; ++i) b[i] = a[i] * d[i];
    } else {  // RevGated
        acc g[VEC], d[VEC];
        load_smem<Tin, VEC>(srow[0] + lane * VEC * sizeof(Tin), g);
        load_smem<Te, VEC>(srow[3] + lane * VEC * sizeof(Te), d);
        const acc lo = gmin, span = acc(gmax) - acc(gmin);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            acc sg = sigmoid_(g[i]);
            acc A = lo + span * sg;
            if (round_ab) A = round_to<Te>(A);
            cache.c0[s][i] = sg;
            a[i] = A;
            b[i] = A * d[i];
        }
    }
}

// ---------------------------------------------------------------------------
// Decoupled lookback, run by one warp.  Publishes the tile aggregate (ta, tb),
// resolves the incoming carry x from predecessors, publishes the inclusive
// prefix ta*x + tb, and returns x and the prefix.
// ---------------------------------------------------------------------------
template <typename acc, int VEC>
__device__ __forceinline__ void lookback(const Workspace& ws, int64_t k, int64_t nct,
                                         int64_t gproc, int wch, int lane,
                                         const acc (&ta)[VEC], const acc (&tb)[VEC],
                                         const acc (&x0)[VEC], acc (&x)[VEC],
                                         acc (&pfx)[VEC]) {
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
            const unsigned nz = __ballot_sync(FULL, f != 0);
            const unsigned ip = __ballot_sync(FULL, f == FLAG_PFX);
            __syncwarp();
            const int m = (nz == FULL) ? 32 : (__ffs(~nz) - 1);
            const unsigned mm = (m >= 32) ? FULL : ((1u << m) - 1u);
            const unsigned pm = ip & mm;
            const int p = pm ? (__ffs(pm) - 1) : -1;
            const int nagg = (p >= 0) ? p : m;
            for (int q = 0; q < nagg; ++q) {
                const int64_t jo = (k - (consumed + q + 1) * nct) * wch + lane * VEC;
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    const acc aj = __ldcg(agg_a + jo + v);
                    const acc bj = __ldcg(agg_b + jo + v);
                    cb[v] = ca[v] * bj + cb[v];
                    ca[v] = ca[v] * aj;
                }
            }
            if (p >= 0) {
                const int64_t jo = (k - (consumed + p + 1) * nct) * wch + lane * VEC;
#pragma unroll
                for (int v = 0; v < VEC; ++v) x[v] = ca[v] * __ldcg(pref + jo + v) + cb[v];
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
                expired = __shfl_sync(FULL, expired, 0);
                if (expired) {
                    if (lane == 0) {
                        raise_status(ESA_STATUS_LOOKBACK_TIMEOUT);
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

// ---------------------------------------------------------------------------
// Tile coordinates.
// ---------------------------------------------------------------------------
struct TileCoord {
    int64_t gproc;  // processing index of the time chunk (lookback order)
    int64_t g;      // time chunk
    int64_t b;      // batch row
    int64_t cb;     // first channel
    int width;      // valid channels
    int64_t t0;     // first step
};

template <bool REV>
__device__ __forceinline__ TileCoord tile_coord(const Geometry& geo, int64_t k, int wch, int lt) {
    TileCoord tc;
    tc.gproc = k / geo.nct;
    const int64_t ct = k - tc.gproc * geo.nct;
    tc.g = REV ? (geo.G - 1 - tc.gproc) : tc.gproc;
    tc.b = ct / geo.ncpr;
    tc.cb = (ct - tc.b * geo.ncpr) * wch;
    const int64_t w = geo.hd - tc.cb;
    tc.width = (int)(w < wch ? w : wch);
    tc.t0 = tc.g * lt;
    return tc;
}

// Issue the bulk copies of tile k into stage buffer `stage` (one warp).
template <Kind K, typename Tin, typename Te, typename P = Policy<K, Tin, Te>>
__device__ __forceinline__ void issue_tile(const Params<K, Tin, Te>& prm, int64_t k, char* stage,
                                           uint64_t* bar, int lane, uint64_t policy) {
    const Geometry& geo = prm.geo;
    const int lt = S * geo.nwarp;
    const TileCoord tc = tile_coord<P::REV>(geo, k, P::WCH, lt);
    // bytes this tile will deliver
    // rows r with step t = t0 + r < T whose source row t + shift is >= 0
    const int64_t rem = geo.T - tc.t0;
    const int nvalid = (int)(rem < lt ? rem : lt);
    unsigned total = 0;
#pragma unroll
    for (int a = 0; a < P::NIN; ++a) {
        const int n = (P::shift(a) < 0 && tc.t0 == 0) ? nvalid - 1 : nvalid;
        total += (unsigned)n * (unsigned)(tc.width * P::es(a));
    }
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
    __syncwarp();
    // stage layout: array a occupies rows [0, lt) of row_bytes(a) each
    int abase = 0;
#pragma unroll
    for (int a = 0; a < P::NIN; ++a) {
        const int rb = P::row_bytes(a);
        const int bytes = tc.width * P::es(a);
        for (int r = lane; r < lt; r += 32) {
            const int64_t t = tc.t0 + r;
            const int64_t tr = t + P::shift(a);
            if (t < geo.T && tr >= 0) {
                const char* src = prm.in[a].p +
                                  ((tc.b * geo.T + tr) * prm.in[a].rs + tc.cb) * (int64_t)P::es(a);
                bulk_g2s(stage + abase + r * rb, src, (unsigned)bytes, bar, policy);
            }
        }
        abase += lt * rb;
    }
}

// ---------------------------------------------------------------------------
// The persistent tiled scan kernel.
// ---------------------------------------------------------------------------
template <Kind K, typename Tin, typename Te>
__global__ void __launch_bounds__(512) tiled_scan_kernel(const Params<K, Tin, Te> prm) {
    using P = Policy<K, Tin, Te>;
    using acc = typename P::acc;
    constexpr int VEC = P::VEC;
    constexpr int WCH = P::WCH;
    const Geometry& geo = prm.geo;
    const int nwarp = geo.nwarp;
    const int lt = S * nwarp;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    extern __shared__ __align__(128) char smem[];
    const int stage_bytes = lt * P::stage_row_bytes();
    acc* sagg_a = reinterpret_cast<acc*>(smem + 2 * stage_bytes);
    acc* sagg_b = sagg_a + nwarp * WCH;
    acc* scarry = sagg_b + nwarp * WCH;
    uint64_t* bars = reinterpret_cast<uint64_t*>(scarry + WCH);
    // s_tile[0]: first ticket; s_tile[1 + (it & 1)]: ticket of the tile after
    // the one processed in iteration `it` (double-buffered so that the write of
    // iteration `it` never races the read of iteration `it`).
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

    unsigned phase_bits = 0;  // parity of each stage's mbarrier
    int it = 0;
    bool healthy = true;
    while (k < geo.ntiles) {
        const int st = it & 1;
        const int64_t kn = s_tile[1 + (it & 1)];
        // prefetch the next tile into the other stage (freed at the end of the
        // previous iteration)
        if (kn < geo.ntiles) {
            if (warp == nwarp - 1)
                issue_tile<K, Tin, Te>(prm, kn, smem + (st ^ 1) * stage_bytes, &bars[st ^ 1], lane, policy);
            outstanding |= 1u << (st ^ 1);
        }
        unsigned knn = 0;
        if (threadIdx.x == 0) knn = atomicAdd(prm.ws.ticket, 1u);

        const TileCoord tc = tile_coord<P::REV>(geo, k, WCH, lt);
        if (mbar_wait_bounded(&bars[st], (phase_bits >> st) & 1u)) {
            phase_bits ^= (1u << st);
            outstanding &= ~(1u << st);
        } else {
            healthy = false;
            atomicExch(prm.ws.abort_flag, 1u);
        }

        // row pointers of this warp's S rows
        const char* sbase = smem + st * stage_bytes;
        auto row_ptrs = [&](int r, const char* (&rows)[4]) {
            int abase = 0;
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                if (a < P::NIN) {
                    rows[a] = sbase + abase + r * P::row_bytes(a);
                    abase += lt * P::row_bytes(a);
                } else {
                    rows[a] = nullptr;
                }
            }
        };

        // ---- phase 1: warp aggregate over its S steps --------------------
        typename P::Cache cache;
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
            if (tc.t0 + r < geo.T) {
                const char* rows[4];
                row_ptrs(r, rows);
                acc a[VEC], b[VEC];
                step_coef<K, Tin, Te>(rows, lane, prm.gmin, prm.gmax, prm.round_ab, a, b, cache, s);
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    pb[i] = a[i] * pb[i] + b[i];
                    pa[i] = a[i] * pa[i];
                }
            }
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            sagg_a[warp * WCH + lane * VEC + i] = pa[i];
            sagg_b[warp * WCH + lane * VEC + i] = pb[i];
        }
        if (threadIdx.x == 0) s_tile[1 + ((it + 1) & 1)] = (int64_t)knn;
        __syncthreads();

        // ---- cross-warp: exclusive prefix of this warp ----------------------
        acc ea[VEC], eb[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            ea[i] = acc(1);
            eb[i] = acc(0);
        }
        if constexpr (!P::REV) {
            for (int w = 0; w < warp; ++w) {
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const acc aw = sagg_a[w * WCH + lane * VEC + i];
                    const acc bw = sagg_b[w * WCH + lane * VEC + i];
                    eb[i] = aw * eb[i] + bw;
                    ea[i] = aw * ea[i];
                }
            }
        } else {
            for (int w = nwarp - 1; w > warp; --w) {
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const acc aw = sagg_a[w * WCH + lane * VEC + i];
                    const acc bw = sagg_b[w * WCH + lane * VEC + i];
                    eb[i] = aw * eb[i] + bw;
                    ea[i] = aw * ea[i];
                }
            }
        }

        // ---- lookback (warp 0) --------------------------------------------
        if (warp == 0) {
            acc ta[VEC], tb[VEC], x0[VEC], x[VEC], pfx[VEC];
            const int last = P::REV ? 0 : (nwarp - 1);
            // tile aggregate = exclusive prefix of the last warp (in processing
            // order) composed with that warp's own aggregate
            {
                acc qa[VEC], qb[VEC];
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    qa[i] = acc(1);
                    qb[i] = acc(0);
                }
                for (int n = 0; n < nwarp; ++n) {
                    const int w = P::REV ? (nwarp - 1 - n) : n;
#pragma unroll
                    for (int i = 0; i < VEC; ++i) {
                        const acc aw = sagg_a[w * WCH + lane * VEC + i];
                        const acc bw = sagg_b[w * WCH + lane * VEC + i];
                        qb[i] = aw * qb[i] + bw;
                        qa[i] = aw * qa[i];
                    }
                }
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    ta[i] = qa[i];
                    tb[i] = qb[i];
                }
            }
            (void)last;
            const int c = lane * VEC;
#pragma unroll
            for (int i = 0; i < VEC; ++i) x0[i] = acc(0);
            if (!P::REV && prm.e0 != nullptr && c < tc.width) {
                const acc* e0 = static_cast<const acc*>(prm.e0) + tc.b * geo.hd + tc.cb + c;
#pragma unroll
                for (int i = 0; i < VEC; ++i) x0[i] = e0[i];
            }
            lookback<acc, VEC>(prm.ws, k, geo.nct, tc.gproc, WCH, lane, ta, tb, x0, x, pfx);
#pragma unroll
            for (int i = 0; i < VEC; ++i) scarry[c + i] = x[i];
            // forward: the last chunk's inclusive prefix is E_{T-1}
            if (!P::REV && prm.e_last != nullptr && tc.g == geo.G - 1 && c < tc.width) {
                acc* el = static_cast<acc*>(prm.e_last) + tc.b * geo.hd + tc.cb + c;
#pragma unroll
                for (int i = 0; i < VEC; ++i) el[i] = pfx[i];
            }
        }
        __syncthreads();

        // ---- phase 3: exact re-run from the incoming state, write outputs ---
        {
            const int c = lane * VEC;
            const bool valid = c < tc.width;
            acc e[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) e[i] = ea[i] * scarry[c + i] + eb[i];
#pragma unroll
            for (int ss = 0; ss < S; ++ss) {
                const int s = P::REV ? (S - 1 - ss) : ss;
                const int r = warp * S + s;
                const int64_t t = tc.t0 + r;
                if (t < geo.T) {
                    const char* rows[4];
                    row_ptrs(r, rows);
                    const int64_t orow = tc.b * geo.T + t;
                    if constexpr (K == Kind::FwdPlain) {
                        acc a[VEC], b[VEC];
                        load_smem<Tin, VEC>(rows[0] + c * sizeof(Tin), a);
                        load_smem<Tin, VEC>(rows[1] + c * sizeof(Tin), b);
#pragma unroll
                        for (int i = 0; i < VEC; ++i) e[i] = a[i] * e[i] + b[i];
                        if (valid)
                            store_global<Te, VEC>(prm.out[0].p + (orow * prm.out[0].rs + tc.cb + c) * (int64_t)sizeof(Te), e);
                    } else if constexpr (K == Kind::FwdGated) {
#pragma unroll
                        for (int i = 0; i < VEC; ++i) e[i] = cache.c0[s][i] * e[i] + cache.c1[s][i];
                        if (valid)
                            store_global<Te, VEC>(prm.out[0].p + (orow * prm.out[0].rs + tc.cb + c) * (int64_t)sizeof(Te), e);
                    } else if constexpr (K == Kind::RevPlain) {
                        // e holds H_{t+1}; G_t = dE_t + H_{t+1}
                        acc a[VEC], ep[VEC], d[VEC], ga[VEC];
                        load_smem<Te, VEC>(rows[0] + c * sizeof(Te), a);
                        load_smem<Te, VEC>(rows[2] + c * sizeof(Te), d);
                        if (t > 0) {
                            load_smem<Te, VEC>(rows[1] + c * sizeof(Te), ep);
                        } else {
#pragma unroll
                            for (int i = 0; i < VEC; ++i) ep[i] = acc(0);
                            if (prm.e0 != nullptr && valid) {
                                const acc* e0 = static_cast<const acc*>(prm.e0) + tc.b * geo.hd + tc.cb + c;
#pragma unroll
                                for (int i = 0; i < VEC; ++i) ep[i] = e0[i];
                            }
                        }
#pragma unroll
                        for (int i = 0; i < VEC; ++i) {
                            const acc g = d[i] + e[i];
                            ga[i] = g * ep[i];
                            d[i] = g;  // dB
                            e[i] = a[i] * g;
                        }
                        if (valid) {
                            store_global<Te, VEC>(prm.out[0].p + (orow * prm.out[0].rs + tc.cb + c) * (int64_t)sizeof(Te), ga);
                            store_global<Te, VEC>(prm.out[1].p + (orow * prm.out[1].rs + tc.cb + c) * (int64_t)sizeof(Te), d);
                        }
                    } else {  // RevGated: outputs d gate_raw, d value_raw (Tin)
                        acc v[VEC], ep[VEC], d[VEC], dg[VEC], dv[VEC];
                        load_smem<Tin, VEC>(rows[1] + c * sizeof(Tin), v);
                        load_smem<Te, VEC>(rows[3] + c * sizeof(Te), d);
                        if (t > 0) {
                            load_smem<Te, VEC>(rows[2] + c * sizeof(Te), ep);
                        } else {
#pragma unroll
                            for (int i = 0; i < VEC; ++i) ep[i] = acc(0);
                            if (prm.e0 != nullptr && valid) {
                                const acc* e0 = static_cast<const acc*>(prm.e0) + tc.b * geo.hd + tc.cb + c;
#pragma unroll
                                for (int i = 0; i < VEC; ++i) ep[i] = e0[i];
                            }
                        }
                        const acc lo = prm.gmin, span = acc(prm.gmax) - acc(prm.gmin);
#pragma unroll
                        for (int i = 0; i < VEC; ++i) {
                            const acc sg = cache.c0[s][i];
                            const acc A = lo + span * sg;
                            const acc Ar = prm.round_ab ? round_to<Te>(A) : A;
                            const acc V = tanh_(v[i]);
                            const acc g = d[i] + e[i];
                            const acc dA = g * ep[i];
                            dg[i] = (dA - g * V) * span * sg * (acc(1) - sg);
                            dv[i] = g * (acc(1) - A) * (acc(1) - V * V);
                            e[i] = Ar * g;
                        }
                        if (valid) {
                            store_global<Tin, VEC>(prm.out[0].p + (orow * prm.out[0].rs + tc.cb + c) * (int64_t)sizeof(Tin), dg);
                            store_global<Tin, VEC>(prm.out[1].p + (orow * prm.out[1].rs + tc.cb + c) * (int64_t)sizeof(Tin), dv);
                        }
                    }
                }
            }
            // reverse: H_0 = A_0 G_0 is the gradient w.r.t. the initial state
            if (P::REV && prm.e_last != nullptr && tc.t0 == 0 && warp == 0 && valid) {
                acc* de0 = static_cast<acc*>(prm.e_last) + tc.b * geo.hd + tc.cb + c;
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
    // After a failed wait, give every copy still in flight one more bounded
    // wait, so that no bulk copy targets this CTA's shared memory after exit.
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
        if (outstanding & (1u << s2)) mbar_wait_bounded(&bars[s2], (phase_bits >> s2) & 1u);
}

// ---------------------------------------------------------------------------
// Fallback for shapes the bulk-copy path cannot stage (rows not 16-byte
// aligned): one thread per channel, sequential over T.  Same math.
// ---------------------------------------------------------------------------
template <Kind K, typename Tin, typename Te>
__global__ void sequential_scan_kernel(const Params<K, Tin, Te> prm) {
    using P = Policy<K, Tin, Te>;
    using acc = typename P::acc;
    const Geometry& geo = prm.geo;
    const int64_t ch = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= geo.nb * geo.hd) return;
    const int64_t b = ch / geo.hd, c = ch - b * geo.hd;
    const acc lo = prm.gmin, span = acc(prm.gmax) - acc(prm.gmin);
    auto ld = [&](int a, int64_t t, auto tag) -> acc {
        using T = decltype(tag);
        const T* p = reinterpret_cast<const T*>(prm.in[a].p) + (b * geo.T + t) * prm.in[a].rs + c;
        return static_cast<acc>(Elem<T>::to_acc(*p));
    };
    auto st = [&](int o, int64_t t, acc val, auto tag) {
        using T = decltype(tag);
        T* p = reinterpret_cast<T*>(prm.out[o].p) + (b * geo.T + t) * prm.out[o].rs + c;
        *p = Elem<T>::from_acc(static_cast<typename Elem<T>::acc>(val));
    };
    if constexpr (!P::REV) {
        acc e = prm.e0 ? static_cast<const acc*>(prm.e0)[ch] : acc(0);
        for (int64_t t = 0; t < geo.T; ++t) {
            acc a, bb;
            if constexpr (K == Kind::FwdPlain) {
                a = ld(0, t, Tin{});
                bb = ld(1, t, Tin{});
            } else {
                a = lo + span * sigmoid_(ld(0, t, Tin{}));
                bb = (acc(1) - a) * tanh_(ld(1, t, Tin{}));
                if (prm.round_ab) {
                    a = round_to<Te>(a);
                    bb = round_to<Te>(bb);
                }
            }
            e = a * e + bb;
            st(0, t, e, Te{});
        }
        if (prm.e_last) static_cast<acc*>(prm.e_last)[ch] = e;
    } else {
        acc h = acc(0);
        for (int64_t t = geo.T - 1; t >= 0; --t) {
            if constexpr (K == Kind::RevPlain) {
                const acc a = ld(0, t, Te{});
                const acc d = ld(2, t, Te{});
                const acc ep = t > 0 ? ld(1, t - 1, Te{}) : (prm.e0 ? static_cast<const acc*>(prm.e0)[ch] : acc(0));
                const acc g = d + h;
                st(0, t, g * ep, Te{});
                st(1, t, g, Te{});
                h = a * g;
            } else {
                const acc sg = sigmoid_(ld(0, t, Tin{}));
                const acc A = lo + span * sg;
                const acc Ar = prm.round_ab ? round_to<Te>(A) : A;
                const acc V = tanh_(ld(1, t, Tin{}));
                const acc d = ld(3, t, Te{});
                const acc ep = t > 0 ? ld(2, t - 1, Te{}) : (prm.e0 ? static_cast<const acc*>(prm.e0)[ch] : acc(0));
                const acc g = d + h;
                st(0, t, (g * ep - g * V) * span * sg * (acc(1) - sg), Tin{});
                st(1, t, g * (acc(1) - A) * (acc(1) - V * V), Tin{});
                h = Ar * g;
            }
        }
        if (prm.e_last) static_cast<acc*>(prm.e_last)[ch] = h;
    }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
int device_status(int device, int clear, unsigned* status) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned));
    if (e == cudaSuccess && clear) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned));
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("device status: ") + cudaGetErrorString(e));
    return ESA_OK;
}

// Steps per tile for a given compass: 16, 32 or 64 (nearest).  Kernels that
// stage four arrays (the fused reverse scan) cap it at 32 so that two stages
// fit in shared memory; the workspace is sized for the capped value, which is
// the larger tile count.
static int lt_for(int compass, int nin = 2) {
    int lt = compass <= 16 ? 16 : (compass <= 32 ? 32 : 64);
    if (nin >= 4 && lt > 32) lt = 32;
    return lt;
}

template <Kind K, typename Tin, typename Te>
static size_t smem_bytes_for(int nwarp) {
    using P = Policy<K, Tin, Te>;
    using acc = typename P::acc;
    const int lt = S * nwarp;
    size_t b = 2ull * lt * P::stage_row_bytes();
    b += (2ull * nwarp * P::WCH + P::WCH) * sizeof(acc);
    b += 2 * sizeof(uint64_t) + 3 * sizeof(int64_t);
    return b;
}

struct WsLayout {
    size_t flags_off, agg_a_off, agg_b_off, pref_off, total;
};

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static WsLayout ws_layout(int64_t ntiles, int wch, size_t acc_size) {
    WsLayout L;
    L.flags_off = 256;
    L.agg_a_off = round_up(L.flags_off + 4 * (size_t)ntiles, 256);
    const size_t d = round_up((size_t)ntiles * wch * acc_size, 256);
    L.agg_b_off = L.agg_a_off + d;
    L.pref_off = L.agg_b_off + d;
    L.total = L.pref_off + d;
    return L;
}

// Geometry for a call: tile sizes follow from the widest element size.
static Geometry make_geometry(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass,
                              int nin = 2) {
    Geometry g;
    const int vec = 16 / wide_es;
    const int wch = 32 * vec;
    const int lt = lt_for(compass, nin);
    g.nb = nb;
    g.T = T;
    g.hd = hd;
    g.ncpr = (hd + wch - 1) / wch;
    g.nct = nb * g.ncpr;
    g.G = (T + lt - 1) / lt;
    g.ntiles = g.G * g.nct;
    g.nwarp = lt / S;
    return g;
}

size_t scan_workspace_bytes(int64_t nb, int64_t T, int64_t hd, int wide_es, int compass) {
    // sized for the smallest tile any kernel uses at this compass (most tiles)
    const Geometry g = make_geometry(nb, T, hd, wide_es, compass, 4);
    const size_t acc_size = wide_es == 8 ? 8 : 4;
    return ws_layout(g.ntiles, 32 * (16 / wide_es), acc_size).total;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <Kind K, typename Tin, typename Te>
static int launch(Params<K, Tin, Te>& prm, void* workspace, size_t ws_bytes, cudaStream_t stream,
                  bool bulk_ok) {
    using P = Policy<K, Tin, Te>;
    using acc = typename P::acc;
    Geometry& geo = prm.geo;
    if (geo.nb == 0 || geo.T == 0 || geo.hd == 0) return ESA_OK;
    if (!bulk_ok) {
        const int threads = 256;
        const int64_t nch = geo.nb * geo.hd;
        const int64_t blocks = (nch + threads - 1) / threads;
        sequential_scan_kernel<K, Tin, Te><<<(unsigned)blocks, threads, 0, stream>>>(prm);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("sequential scan launch: ") + cudaGetErrorString(e));
        return ESA_OK;
    }
    const WsLayout L = ws_layout(geo.ntiles, P::WCH, sizeof(acc));
    if (workspace == nullptr || ws_bytes < L.total || !aligned16(workspace))
        return set_error(ESA_ERR_WORKSPACE, "workspace missing, misaligned or smaller than esa_scan_workspace_bytes()");
    char* ws = static_cast<char*>(workspace);
    prm.ws.ticket = reinterpret_cast<unsigned*>(ws);
    prm.ws.abort_flag = reinterpret_cast<unsigned*>(ws) + 1;
    prm.ws.flags = reinterpret_cast<unsigned*>(ws + L.flags_off);
    prm.ws.agg_a = ws + L.agg_a_off;
    prm.ws.agg_b = ws + L.agg_b_off;
    prm.ws.pref = ws + L.pref_off;
    cudaError_t e = cudaMemsetAsync(ws, 0, L.agg_a_off, stream);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("workspace reset: ") + cudaGetErrorString(e));

    const size_t smem = smem_bytes_for<K, Tin, Te>(geo.nwarp);
    if (smem > 232448)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "tile configuration exceeds shared memory");
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    // opt in to large dynamic shared memory (idempotent, cheap)
    e = cudaFuncSetAttribute(tiled_scan_kernel<K, Tin, Te>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("smem attribute: ") + cudaGetErrorString(e));
    (void)configured_dev;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiled_scan_kernel<K, Tin, Te>, 32 * geo.nwarp, smem);
    if (e != cudaSuccess || per_sm <= 0)
        return set_error(ESA_ERR_CUDA, "scan kernel cannot be resident (occupancy 0)");
    const int sms = device_sm_count(dev);
    int64_t grid = (int64_t)per_sm * sms;
    if (grid > geo.ntiles) grid = geo.ntiles;
    tiled_scan_kernel<K, Tin, Te><<<(unsigned)grid, 32 * geo.nwarp, smem, stream>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESA_ERR_CUDA, std::string("scan launch: ") + cudaGetErrorString(e));
    return ESA_OK;
}

// ---------------------------------------------------------------------------
// dtype dispatch
// ---------------------------------------------------------------------------
template <typename F>
static int dispatch1(int dtype, F&& f) {
    switch (dtype) {
        case ESA_DTYPE_F16: return f(__half{});
        case ESA_DTYPE_BF16: return f(__nv_bfloat16{});
        case ESA_DTYPE_F32: return f(float{});
        case ESA_DTYPE_F64: return f(double{});
        default: return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    }
}

static bool rows_aligned(const void* p, int64_t rs, int64_t hd, int es) {
    return aligned16(p) && ((rs * es) % 16 == 0) && ((hd * es) % 16 == 0);
}

static int check_dims(int64_t nb, int64_t T, int64_t hd, int compass) {
    if (nb < 0 || T < 0 || hd < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "negative dimension");
    if (compass <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "compass must be a positive integer");
    return ESA_OK;
}

int scan_fwd(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd, int dtype,
             int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    if (nb * T * hd > 0 && (!A || !B || !E)) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    return dispatch1(dtype, [&](auto tag) -> int {
        using T_ = decltype(tag);
        Params<Kind::FwdPlain, T_, T_> prm{};
        prm.in[0] = {static_cast<const char*>(A), hd};
        prm.in[1] = {static_cast<const char*>(B), hd};
        prm.out[0] = {static_cast<char*>(E), hd};
        prm.geo = make_geometry(nb, T, hd, sizeof(T_), compass);
        prm.e0 = e0;
        prm.e_last = e_last;
        const int es = sizeof(T_);
        const bool bulk = rows_aligned(A, hd, hd, es) && rows_aligned(B, hd, hd, es) && rows_aligned(E, hd, hd, es);
        return launch(prm, ws, ws_bytes, s, bulk);
    });
}

int scan_rev(const void* A, const void* E, const void* dE, void* dA, void* dB, int64_t nb, int64_t T,
             int64_t hd, int dtype, int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
             cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    if (nb * T * hd > 0 && (!A || !E || !dE || !dA || !dB))
        return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    return dispatch1(dtype, [&](auto tag) -> int {
        using T_ = decltype(tag);
        Params<Kind::RevPlain, T_, T_> prm{};
        prm.in[0] = {static_cast<const char*>(A), hd};
        prm.in[1] = {static_cast<const char*>(E), hd};
        prm.in[2] = {static_cast<const char*>(dE), hd};
        prm.out[0] = {static_cast<char*>(dA), hd};
        prm.out[1] = {static_cast<char*>(dB), hd};
        prm.geo = make_geometry(nb, T, hd, sizeof(T_), compass);
        prm.e0 = e0;
        prm.e_last = de0;
        const int es = sizeof(T_);
        const bool bulk = rows_aligned(A, hd, hd, es) && rows_aligned(E, hd, hd, es) &&
                          rows_aligned(dE, hd, hd, es) && rows_aligned(dA, hd, hd, es) &&
                          rows_aligned(dB, hd, hd, es);
        return launch(prm, ws, ws_bytes, s, bulk);
    });
}

int gated_scan_fwd(const void* g, const void* v, int64_t rrs, int raw_dtype, void* E, int e_dtype,
                   int64_t nb, int64_t T, int64_t hd, float gmin, float gmax, int round_ab,
                   int compass, const void* e0, void* e_last, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    if (nb * T * hd > 0 && (!g || !v || !E)) return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (rrs < hd) return set_error(ESA_ERR_INVALID_ARGUMENT, "raw_row_stride smaller than hd");
    return dispatch1(raw_dtype, [&](auto rtag) -> int {
        using Tr = decltype(rtag);
        return dispatch1(e_dtype, [&](auto etag) -> int {
            using Te_ = decltype(etag);
            Params<Kind::FwdGated, Tr, Te_> prm{};
            prm.in[0] = {static_cast<const char*>(g), rrs};
            prm.in[1] = {static_cast<const char*>(v), rrs};
            prm.out[0] = {static_cast<char*>(E), hd};
            const int wide = sizeof(Tr) > sizeof(Te_) ? sizeof(Tr) : sizeof(Te_);
            prm.geo = make_geometry(nb, T, hd, wide, compass);
            prm.e0 = e0;
            prm.e_last = e_last;
            prm.gmin = gmin;
            prm.gmax = gmax;
            prm.round_ab = round_ab;
            const bool bulk = rows_aligned(g, rrs, hd, sizeof(Tr)) && rows_aligned(v, rrs, hd, sizeof(Tr)) &&
                              rows_aligned(E, hd, hd, sizeof(Te_));
            return launch(prm, ws, ws_bytes, s, bulk);
        });
    });
}

int gated_scan_bwd(const void* g, const void* v, int64_t rrs, int raw_dtype, const void* E,
                   const void* dE, int e_dtype, void* dg, void* dv, int64_t drs, int draw_dtype,
                   int64_t nb, int64_t T, int64_t hd, float gmin, float gmax, int round_ab,
                   int compass, const void* e0, void* de0, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
    if (int rc = check_dims(nb, T, hd, compass)) return rc;
    if (nb * T * hd > 0 && (!g || !v || !E || !dE || !dg || !dv))
        return set_error(ESA_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (rrs < hd || drs < hd) return set_error(ESA_ERR_INVALID_ARGUMENT, "row stride smaller than hd");
    if (draw_dtype != raw_dtype)
        return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "d_gate_raw/d_value_raw must have the dtype of gate_raw/value_raw");
    return dispatch1(raw_dtype, [&](auto rtag) -> int {
        using Tr = decltype(rtag);
        return dispatch1(e_dtype, [&](auto etag) -> int {
            using Te_ = decltype(etag);
            Params<Kind::RevGated, Tr, Te_> prm{};
            prm.in[0] = {static_cast<const char*>(g), rrs};
            prm.in[1] = {static_cast<const char*>(v), rrs};
            prm.in[2] = {static_cast<const char*>(E), hd};
            prm.in[3] = {static_cast<const char*>(dE), hd};
            prm.out[0] = {static_cast<char*>(dg), drs};
            prm.out[1] = {static_cast<char*>(dv), drs};
            const int wide = sizeof(Tr) > sizeof(Te_) ? sizeof(Tr) : sizeof(Te_);
            prm.geo = make_geometry(nb, T, hd, wide, compass, 4);
            prm.e0 = e0;
            prm.e_last = de0;
            prm.gmin = gmin;
            prm.gmax = gmax;
            prm.round_ab = round_ab;
            const bool bulk = rows_aligned(g, rrs, hd, sizeof(Tr)) && rows_aligned(v, rrs, hd, sizeof(Tr)) &&
                              rows_aligned(E, hd, hd, sizeof(Te_)) && rows_aligned(dE, hd, hd, sizeof(Te_)) &&
                              rows_aligned(dg, drs, hd, sizeof(Tr)) && rows_aligned(dv, drs, hd, sizeof(Tr));
            return launch(prm, ws, ws_bytes, s, bulk);
        });
    });
}

}  // namespace esa
