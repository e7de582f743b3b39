// esa_tile.cuh -- row-tile scan of the ESA layer: one CTA tile is LT time
// steps x ALL C channels of one batch row, so the layer's RMS readout over C
// (esa/backends/thunder.py:304-311 of the reference normalises across every
// head) can be fused into the same pass as the gated recurrence.
//
// Forward (kind FWD), per tile:
//   phase 1  every consumer lane owns V channels and walks the tile's steps in
//            order: A = gmin + span*sigmoid(g), B = (1 - A) tanh(v), rounded
//            to the scan dtype (the reference's A.to(scan_dtype)), kept in
//            registers, and composed into the tile aggregate (prod A, state
//            from zero);
//   lookback decoupled look-back across the tiles of the same batch row
//            (Merrill & Garland 2016), one warp per 32*V-channel slice, with
//            the predecessors' aggregates loaded several at a time;
//   phase 3  the exact states E_t from the incoming carry, written once;
//   readout  (RO) per step the sum of E_t^2 over the warp (a butterfly
//            reduce-scatter: lane r ends with step r's sum), over the CTA
//            through shared memory and an mbarrier, rstd = 1/sqrt(mean + eps),
//            y = sigmoid(q) * E * rstd written once, rstd kept for the
//            backward.
// Backward (kind REV), tiles in descending time order:
//   readout  (RO) dq = dy n s(1-s) and dE = r (dy s - n mean_C(dy s n)),
//            s = sigmoid(q), n = E r, the mean again a CTA reduction;
//   phase 1  the reverse recurrence H_t = A_t (dE_t + H_{t+1}) aggregated
//            over the tile's steps, descending;
//   lookback as forward, in descending tile order;
//   phase 3  G_t = dE_t + H_{t+1}, dA = G_t E_{t-1}, and the gate chain rule
//            dg = (dA - G_t tanh v) span s_g (1 - s_g),
//            dv = G_t (1 - A)(1 - tanh^2 v), written once.
//
// CTA = NWC consumer warps (C = NWC*32*V channels) + one producer warp whose
// lane 0 takes tiles from an atomic ticket (time-chunk major, so every
// predecessor of a tile belongs to a CTA that is already running) and stages
// them with 3-D TMA loads (boxes of WB channels x the tile's rows, L2
// evict-first) into an NSTAGE ring; a stage holds one tile of every input.
// Every wait is bounded (one second): mbarrier waits, look-back flags and the
// cross-warp readout barrier (an mbarrier, not bar.sync, so a warp that gave
// up cannot strand the others).  On expiry the status word is raised and the
// launch's abort flag makes later waits give up at once.
#pragma once

#include <type_traits>

#include "esa_strip.cuh"

namespace esa {

constexpr unsigned TILE_AGG = 1, TILE_PFX = 2;

// Arguments of one row-tile launch (trivially copyable, passed by value).
struct TileArgs {
    // outputs, row-strided (element (row = b*T + t, c) at p + (row*rs + c)*es)
    char* out0;  // FWD: E (scan dtype);  REV: d gate_raw (raw dtype)
    char* out1;  // FWD RO: y (y dtype);  REV: d value_raw (raw dtype)
    char* out2;  // REV RO: d q (raw dtype)
    int64_t o0rs, o1rs, o2rs;
    void* rstd;      // RO: [nb*T] fp32 (FWD writes it, REV reads it)
    const void* e0;  // fp32 [nb*C] or null: FWD initial state; REV E_{-1}
    void* e_last;    // fp32 [nb*C] or null: FWD E_{T-1}; REV gradient w.r.t. e0
    int64_t nb, T, C, G, ntiles;
    int nwc;          // consumer warps
    int wb;           // channels per TMA box
    int nstage;
    int stage_bytes;
    int arr_off[5];   // byte offset of each staged array in a stage
    int arr_rows[5];  // rows of each staged array (LT, or LT + 1 for E in REV)
    double gmin, span, eps;
    unsigned* status;
    unsigned* ticket;
    unsigned* abort_flag;
    unsigned* flags;  // [ntiles * nwc]
    float* agg_a;     // [ntiles * C]
    float* agg_b;
    float* pref;
};

// Packed register copy of V values rounded to T (16-bit: two per word).
template <typename T, int V>
struct Packed {
    static constexpr bool HALF = sizeof(T) == 2;
    static constexpr int W = HALF ? V / 2 : V;
    typename std::conditional<HALF, uint32_t, float>::type w[W];

    __device__ __forceinline__ void set(const float (&x)[V]) {
        if constexpr (std::is_same<T, __half>::value) {
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
        } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
        } else {
#pragma unroll
            for (int i = 0; i < V; ++i) w[i] = x[i];
        }
    }
    __device__ __forceinline__ void get(float (&x)[V]) const {
        if constexpr (std::is_same<T, __half>::value) {
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
        } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < V; ++i) x[i] = w[i];
        }
    }
    // one vector store of the V packed values
    __device__ __forceinline__ void store(char* p) const {
        constexpr int BYTES = V * (int)sizeof(T);
        static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16, "lane vector of 4, 8 or 16 bytes");
        const uint32_t* u = reinterpret_cast<const uint32_t*>(w);
        if constexpr (BYTES == 16)
            *reinterpret_cast<uint4*>(p) = make_uint4(u[0], u[1], u[2], u[3]);
        else if constexpr (BYTES == 8)
            *reinterpret_cast<uint2*>(p) = make_uint2(u[0], u[1]);
        else
            *reinterpret_cast<uint32_t*>(p) = u[0];
    }
};

// V values of T from shared memory, widened to float.
template <typename T, int V>
__device__ __forceinline__ void lds_f(const char* p, float (&x)[V]) {
    load_smem<T, V>(p, x);
}

// Store V floats rounded to T with one vector store.
template <typename T, int V>
__device__ __forceinline__ void stg_f(char* p, const float (&x)[V]) {
    Packed<T, V> pk;
    pk.set(x);
    pk.store(p);
}

// Butterfly reduce-scatter over the warp: on entry every lane holds N partial
// sums x[0..N) (N = 8, 16 or 32); on exit lane l's x[0] holds the warp total
// of entry (l mod N).
template <int N>
__device__ __forceinline__ void warp_reduce_scatter(float (&x)[N], int lane) {
    static_assert(N == 8 || N == 16 || N == 32, "8, 16 or 32 rows");
    // offsets beyond N's index bits: plain pairwise sums first
#pragma unroll
    for (int o = 16; o >= N; o >>= 1) {
#pragma unroll
        for (int i = 0; i < N; ++i) x[i] += __shfl_xor_sync(0xffffffffu, x[i], o);
    }
    // then halve the live values at every offset: keep the half whose index
    // bit matches this lane's bit, add the partner's copy of that half
#pragma unroll
    for (int o = N / 2, n = N; o >= 1; o >>= 1, n >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float keep = upper ? x[i + n / 2] : x[i];
            const float send = upper ? x[i] : x[i + n / 2];
            x[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
}

__device__ __forceinline__ bool tile_aborted(const TileArgs& a) {
    return *(volatile unsigned*)a.abort_flag != 0u;
}

__device__ __forceinline__ void tile_give_up(const TileArgs& a, unsigned bit) {
    atomicOr(a.status, bit);
    atomicExch(a.abort_flag, 1u);
}

// Bounded wait on an mbarrier phase that also gives up at once when the
// launch is aborted.  Returns false on expiry (status raised).
__device__ __forceinline__ bool tile_mbar_wait(const TileArgs& a, uint64_t* bar, unsigned parity,
                                               unsigned bit) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned it = 0; it < kWaitMaxIters; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitBudgetNs || tile_aborted(a)) break;
    }
    tile_give_up(a, bit);
    return false;
}

// Decoupled look-back of one warp over its 32*V channels.  k: tile index
// (gproc * nb + b); predecessors in processing order are k - nb, k - 2 nb, ...
// Publishes the tile aggregate (ta, tb), resolves the incoming carry x (x0
// for the first tile of a row), publishes the inclusive prefix.
template <int V>
__device__ __forceinline__ void tile_lookback(const TileArgs& a, int64_t k, int64_t gproc, int w, int lane,
                                              const float (&ta)[V], const float (&tb)[V],
                                              const float (&x0)[V], float (&x)[V]) {
    const int64_t off = k * a.C + (int64_t)w * (32 * V) + lane * V;
    unsigned* myflag = a.flags + k * a.nwc + w;
    if (gproc == 0) {
#pragma unroll
        for (int i = 0; i < V; ++i) x[i] = x0[i];
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) {
            a.agg_a[off + i] = ta[i];
            a.agg_b[off + i] = tb[i];
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu(myflag, TILE_AGG);
        float ca[V], cb[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
            ca[i] = 1.0f;
            cb[i] = 0.0f;
        }
        int64_t consumed = 0;
        unsigned long long t_start = 0;
        unsigned spins = 0;
        while (true) {
            const int64_t j = consumed + lane + 1;  // predecessor distance polled by this lane
            unsigned f = 0;
            if (j <= gproc) f = ld_acquire_gpu(a.flags + (k - j * a.nb) * a.nwc + w);
            const unsigned nz = __ballot_sync(0xffffffffu, f != 0);
            const unsigned ip = __ballot_sync(0xffffffffu, f == TILE_PFX);
            __syncwarp();
            const int m = (nz == 0xffffffffu) ? 32 : (__ffs(~nz) - 1);
            const unsigned mm = (m >= 32) ? 0xffffffffu : ((1u << m) - 1u);
            const unsigned pm = ip & mm;
            const int p = pm ? (__ffs(pm) - 1) : -1;
            const int nagg = (p >= 0) ? p : m;
            // predecessors' aggregates in batches of LB independent loads
            constexpr int LB = 8 / V;
            for (int q0 = 0; q0 < nagg; q0 += LB) {
                float la[LB][V], lb[LB][V];
#pragma unroll
                for (int u = 0; u < LB; ++u) {
                    if (q0 + u < nagg) {
                        const int64_t jo =
                            (k - (consumed + q0 + u + 1) * a.nb) * a.C + (int64_t)w * (32 * V) + lane * V;
#pragma unroll
                        for (int i = 0; i < V; ++i) {
                            la[u][i] = __ldcg(a.agg_a + jo + i);
                            lb[u][i] = __ldcg(a.agg_b + jo + i);
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < LB; ++u) {
                    if (q0 + u < nagg) {
#pragma unroll
                        for (int i = 0; i < V; ++i) {
                            cb[i] = fmaf(ca[i], lb[u][i], cb[i]);
                            ca[i] = ca[i] * la[u][i];
                        }
                    }
                }
            }
            if (p >= 0) {
                const int64_t jo = (k - (consumed + p + 1) * a.nb) * a.C + (int64_t)w * (32 * V) + lane * V;
#pragma unroll
                for (int i = 0; i < V; ++i) x[i] = fmaf(ca[i], __ldcg(a.pref + jo + i), cb[i]);
                break;
            }
            consumed += m;
            if (m == 0) {
                if (spins == 0) t_start = globaltimer_ns();
                ++spins;
                __nanosleep(32);
                bool expired = (spins > kWaitMaxIters) || (globaltimer_ns() - t_start > kWaitBudgetNs) ||
                               tile_aborted(a);
                expired = __shfl_sync(0xffffffffu, expired, 0);
                if (expired) {
                    if (lane == 0) tile_give_up(a, ESA_STATUS_LOOKBACK_TIMEOUT);
#pragma unroll
                    for (int i = 0; i < V; ++i) x[i] = 0.0f;
                    break;
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) a.pref[off + i] = fmaf(ta[i], x[i], tb[i]);
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_gpu(myflag, TILE_PFX);
}

// At most 12 consumer warps: 13 warps put at most 4 on each of the SM's four
// schedulers, whose 16 K registers then allow 128 per thread (17 warps would
// cap them at 96 and spill the register tiles).
struct TileSmem {
    static constexpr int MAX_STAGES = 4;
    static constexpr int MAX_WARPS = 12;
};

template <bool REV, bool RO, typename Tr, typename Te, typename Ty, int V, int LT>
struct TileCfg {
    static constexpr int CW = 32 * V;  // channels per consumer warp
    // staged arrays: FWD {g, v, q}; REV {g, v, q, E (LT + 1 rows from t0 - 1), dY}
    static constexpr int NARR = REV ? 5 : 3;
    static __host__ __device__ constexpr bool HAS(int i) { return (i != 2 || RO); }
    static __host__ __device__ constexpr int es(int i) {
        return i < 3 ? (int)sizeof(Tr) : (i == 3 ? (int)sizeof(Te) : (RO ? (int)sizeof(Ty) : (int)sizeof(Te)));
    }
    static __host__ __device__ constexpr int rows(int i) { return (REV && i == 3) ? LT + 1 : LT; }
    // after the ring: full[4], empty[4], readout barrier, tile id per stage,
    // readout partials [2][MAX_WARPS][LT], alignment slack
    static size_t tail_bytes() {
        return (size_t)TileSmem::MAX_STAGES * 2 * 8 + 8 + TileSmem::MAX_STAGES * 8 +
               2 * TileSmem::MAX_WARPS * LT * sizeof(float) + 128;
    }
};

template <bool REV, bool RO, typename Tr, typename Te, typename Ty, int V, int LT>
__global__ void __launch_bounds__(32 * (TileSmem::MAX_WARPS + 1), 1)
    tile_layer_kernel(const TileArgs a, const __grid_constant__ CUtensorMap m0,
                      const __grid_constant__ CUtensorMap m1, const __grid_constant__ CUtensorMap m2,
                      const __grid_constant__ CUtensorMap m3, const __grid_constant__ CUtensorMap m4) {
    using Cfg = TileCfg<REV, RO, Tr, Te, Ty, V, LT>;
    constexpr int CW = Cfg::CW;
    constexpr int NARR = Cfg::NARR;
    constexpr bool FASTG = sizeof(Tr) == 2 && sizeof(Te) == 2;  // 16-bit gate math (gate_sigmoid)
    const int nwc = a.nwc;
    const int nstage = a.nstage;

    extern __shared__ __align__(128) char smem_raw[];
    char* smem = smem_raw + ((128u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 127u)) & 127u);
    char* tail = smem + (size_t)nstage * a.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(tail);
    uint64_t* empty = full + TileSmem::MAX_STAGES;
    uint64_t* redbar = empty + TileSmem::MAX_STAGES;
    int* tile_id = reinterpret_cast<int*>(redbar + 1);
    float* red = reinterpret_cast<float*>(tile_id + 2 * TileSmem::MAX_STAGES);  // [2][MAX_WARPS][LT]
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], nwc);
        }
        mbar_init(redbar, nwc);
        fence_mbarrier_init();
    }
    __syncthreads();

    if (warp == nwc) {
        // ---- producer: lane 0 takes tiles and fills the ring -----------------
        if (lane != 0) return;
        const CUtensorMap* maps[5] = {&m0, &m1, &m2, &m3, &m4};
        const uint64_t policy = policy_evict_first();
        int slot = 0;
        unsigned rnd = 0;
        uint64_t fills = 0;
        bool ok = true;
        while (true) {
            if (rnd > 0 && !tile_mbar_wait(a, &empty[slot], (rnd - 1) & 1u, ESA_STATUS_COPY_TIMEOUT)) {
                ok = false;
                break;
            }
            const unsigned k = atomicAdd(a.ticket, 1u);
            if ((int64_t)k >= a.ntiles) {
                tile_id[slot] = -1;
                mbar_arrive(&full[slot]);
                break;
            }
            tile_id[slot] = (int)k;
            const int64_t gproc = (int64_t)k / a.nb;
            const int64_t b = (int64_t)k - gproc * a.nb;
            const int64_t g = REV ? (a.G - 1 - gproc) : gproc;
            const int t0 = (int)(g * LT);
            char* stage = smem + (size_t)slot * a.stage_bytes;
            mbar_arrive_expect_tx(&full[slot], (unsigned)a.stage_bytes);
#pragma unroll
            for (int i = 0; i < NARR; ++i) {
                if (!Cfg::HAS(i)) continue;
                const int box_bytes = Cfg::rows(i) * a.wb * Cfg::es(i);
                const int y = (REV && i == 3) ? t0 - 1 : t0;
                for (int x = 0, j = 0; x < a.C; x += a.wb, ++j)
                    tma_load_3d(stage + a.arr_off[i] + j * box_bytes, maps[i], x, y, (int)b, &full[slot], policy);
            }
            ++fills;
            if (++slot == nstage) {
                slot = 0;
                ++rnd;
            }
        }
        if (!ok) {
            // consumers gone: let every copy still in flight land before exit
            const uint64_t first = fills > (uint64_t)nstage ? fills - nstage : 0;
            for (uint64_t u = first; u < fills; ++u)
                mbar_wait_bounded(&full[u % nstage], (unsigned)((u / nstage) & 1), a.status);
        }
        return;
    }

    // ---- consumers -------------------------------------------------------------
    const int c0 = warp * CW + lane * V;  // first channel of this lane
    const int boxj = c0 / a.wb, col = c0 - boxj * a.wb;
    int lo_off[NARR], rstride[NARR];  // this lane's byte offset in each array, bytes per row
#pragma unroll
    for (int i = 0; i < NARR; ++i) {
        rstride[i] = a.wb * Cfg::es(i);
        lo_off[i] = a.arr_off[i] + boxj * Cfg::rows(i) * rstride[i] + col * Cfg::es(i);
    }
    const float lo = (float)a.gmin, span = (float)a.span;
    int slot = 0;
    unsigned parity = 0, redpar = 0;
    while (true) {
        if (!__all_sync(0xffffffffu, tile_mbar_wait(a, &full[slot], parity, ESA_STATUS_COPY_TIMEOUT))) break;
        const int k = tile_id[slot];
        if (k < 0) break;
        const int64_t gproc = (int64_t)k / a.nb;
        const int64_t b = (int64_t)k - gproc * a.nb;
        const int64_t g = REV ? (a.G - 1 - gproc) : gproc;
        const int64_t t0 = g * LT;
        const int nrows = (int)(a.T - t0 < LT ? a.T - t0 : LT);
        const char* st = smem + (size_t)slot * a.stage_bytes;
        auto row_ptr = [&](int i, int r) -> const char* { return st + lo_off[i] + r * rstride[i]; };
        const int64_t row0 = b * a.T + t0;  // global row of the tile's first step
        bool ok = true;

        if constexpr (!REV) {
            // ---- forward: gates + aggregate ----------------------------------
            Packed<Te, V> ca[LT], cb[LT];
            float ta[V], tb[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                ta[i] = 1.0f;
                tb[i] = 0.0f;
            }
#pragma unroll
            for (int r = 0; r < LT; ++r) {
                if (r < nrows) {
                    float gv[V], vv[V], A[V], B[V];
                    lds_f<Tr, V>(row_ptr(0, r), gv);
                    lds_f<Tr, V>(row_ptr(1, r), vv);
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        A[i] = lo + span * gate_sigmoid<FASTG>(gv[i]);
                        B[i] = (1.0f - A[i]) * gate_tanh<FASTG>(vv[i]);
                    }
                    ca[r].set(A);  // rounded to the scan dtype, as the reference's A.to(scan_dtype)
                    cb[r].set(B);
                    ca[r].get(A);
                    cb[r].get(B);
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        tb[i] = fmaf(A[i], tb[i], B[i]);
                        ta[i] = ta[i] * A[i];
                    }
                }
            }
            float x0[V], x[V];
#pragma unroll
            for (int i = 0; i < V; ++i)
                x0[i] = (gproc == 0 && a.e0 != nullptr) ? static_cast<const float*>(a.e0)[b * a.C + c0 + i] : 0.0f;
            tile_lookback<V>(a, k, gproc, warp, lane, ta, tb, x0, x);
            // ---- forward: exact states, E written once ------------------------
            float ss[LT];
#pragma unroll
            for (int r = 0; r < LT; ++r) {
                ss[r] = 0.0f;
                if (r < nrows) {
                    float A[V], B[V];
                    ca[r].get(A);
                    cb[r].get(B);
#pragma unroll
                    for (int i = 0; i < V; ++i) x[i] = fmaf(A[i], x[i], B[i]);
                    Packed<Te, V> pe;
                    pe.set(x);
                    pe.store(a.out0 + ((row0 + r) * a.o0rs + c0) * (int64_t)sizeof(Te));
                    if constexpr (RO) {
                        float er[V];
                        pe.get(er);
                        ca[r] = pe;
#pragma unroll
                        for (int i = 0; i < V; ++i) ss[r] = fmaf(er[i], er[i], ss[r]);
                    }
                }
            }
            if (a.e_last != nullptr && t0 + nrows == a.T) {
#pragma unroll
                for (int i = 0; i < V; ++i) static_cast<float*>(a.e_last)[b * a.C + c0 + i] = x[i];
            }
            if constexpr (RO) {
                // ---- readout: RMS over all C channels of each step -----------
                warp_reduce_scatter<LT>(ss, lane);
                float* rbuf = red + redpar * TileSmem::MAX_WARPS * LT;
                if (lane < LT) rbuf[warp * LT + lane] = ss[0];
                __syncwarp();
                if (lane == 0) mbar_arrive(redbar);
                ok = __all_sync(0xffffffffu, tile_mbar_wait(a, redbar, redpar, ESA_STATUS_COPY_TIMEOUT));
                if (ok) {
                    const int r = lane % LT;
                    float tot = 0.0f;
                    for (int w2 = 0; w2 < nwc; ++w2) tot += rbuf[w2 * LT + r];
                    const float rs = 1.0f / sqrtf(tot * (1.0f / (float)a.C) + (float)a.eps);
                    if (warp == 0 && lane < nrows) static_cast<float*>(a.rstd)[row0 + lane] = rs;
#pragma unroll
                    for (int r2 = 0; r2 < LT; ++r2) {
                        const float rr = __shfl_sync(0xffffffffu, rs, r2);
                        if (r2 < nrows) {
                            float qv[V], er[V], yv[V];
                            lds_f<Tr, V>(row_ptr(2, r2), qv);
                            ca[r2].get(er);
#pragma unroll
                            for (int i = 0; i < V; ++i) yv[i] = gate_sigmoid<FASTG>(qv[i]) * (er[i] * rr);
                            stg_f<Ty, V>(a.out1 + ((row0 + r2) * a.o1rs + c0) * (int64_t)sizeof(Ty), yv);
                        }
                    }
                }
                redpar ^= 1u;
            }
        } else {
            // ---- backward ------------------------------------------------------
            float dE[LT][V];  // dE_t (readout backward output or staged input)
            float sg[LT][V];  // sigmoid(g_t); holds n_t during the readout backward
            if constexpr (RO) {
                const float rsv = lane < nrows ? static_cast<const float*>(a.rstd)[row0 + lane] : 0.0f;
                float p[LT];
#pragma unroll
                for (int r = 0; r < LT; ++r) {
                    p[r] = 0.0f;
                    const float rr = __shfl_sync(0xffffffffu, rsv, r);
                    if (r < nrows) {
                        float qv[V], ev[V], dy[V], dq[V];
                        lds_f<Tr, V>(row_ptr(2, r), qv);
                        lds_f<Te, V>(row_ptr(3, r + 1), ev);
                        lds_f<Ty, V>(row_ptr(4, r), dy);
#pragma unroll
                        for (int i = 0; i < V; ++i) {
                            const float s = gate_sigmoid<FASTG>(qv[i]);
                            const float n = ev[i] * rr;
                            const float t1 = dy[i] * s;
                            dq[i] = t1 * n * (1.0f - s);
                            dE[r][i] = t1;
                            sg[r][i] = n;
                            p[r] = fmaf(t1, n, p[r]);
                        }
                        stg_f<Tr, V>(a.out2 + ((row0 + r) * a.o2rs + c0) * (int64_t)sizeof(Tr), dq);
                    }
                }
                warp_reduce_scatter<LT>(p, lane);
                float* rbuf = red + redpar * TileSmem::MAX_WARPS * LT;
                if (lane < LT) rbuf[warp * LT + lane] = p[0];
                __syncwarp();
                if (lane == 0) mbar_arrive(redbar);
                ok = __all_sync(0xffffffffu, tile_mbar_wait(a, redbar, redpar, ESA_STATUS_COPY_TIMEOUT));
                redpar ^= 1u;
                float mean = 0.0f;
                if (ok) {
                    const int r = lane % LT;
                    float tot = 0.0f;
                    for (int w2 = 0; w2 < nwc; ++w2) tot += rbuf[w2 * LT + r];
                    mean = tot * (1.0f / (float)a.C);
                }
#pragma unroll
                for (int r = 0; r < LT; ++r) {
                    const float rr = __shfl_sync(0xffffffffu, rsv, r);
                    const float mm = __shfl_sync(0xffffffffu, mean, r);
#pragma unroll
                    for (int i = 0; i < V; ++i) dE[r][i] = rr * (dE[r][i] - sg[r][i] * mm);
                }
            } else {
#pragma unroll
                for (int r = 0; r < LT; ++r)
                    if (r < nrows) lds_f<Te, V>(row_ptr(4, r), dE[r]);
            }
            // ---- reverse aggregate (descending steps) -------------------------
            float ta[V], tb[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                ta[i] = 1.0f;
                tb[i] = 0.0f;
            }
#pragma unroll
            for (int rr = 0; rr < LT; ++rr) {
                const int r = LT - 1 - rr;
                if (r < nrows) {
                    float gv[V];
                    lds_f<Tr, V>(row_ptr(0, r), gv);
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        sg[r][i] = gate_sigmoid<FASTG>(gv[i]);
                        const float Ar = round_to<Te>(lo + span * sg[r][i]);
                        tb[i] = Ar * (dE[r][i] + tb[i]);
                        ta[i] = ta[i] * Ar;
                    }
                }
            }
            float zero[V], x[V];
#pragma unroll
            for (int i = 0; i < V; ++i) zero[i] = 0.0f;
            tile_lookback<V>(a, k, gproc, warp, lane, ta, tb, zero, x);
            // ---- gradients, descending steps ------------------------------------
#pragma unroll
            for (int rr = 0; rr < LT; ++rr) {
                const int r = LT - 1 - rr;
                if (r < nrows) {
                    float ep[V], vv[V], dg[V], dv[V];
                    lds_f<Te, V>(row_ptr(3, r), ep);  // E_{t-1} (zero-filled before t = 0)
                    if (t0 + r == 0 && a.e0 != nullptr) {
#pragma unroll
                        for (int i = 0; i < V; ++i) ep[i] = static_cast<const float*>(a.e0)[b * a.C + c0 + i];
                    }
                    lds_f<Tr, V>(row_ptr(1, r), vv);
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        const float s = sg[r][i];
                        const float A = lo + span * s;
                        const float Ar = round_to<Te>(A);
                        const float tv = gate_tanh<FASTG>(vv[i]);
                        const float G = dE[r][i] + x[i];
                        dg[i] = (G * ep[i] - G * tv) * span * s * (1.0f - s);
                        dv[i] = G * (1.0f - A) * (1.0f - tv * tv);
                        x[i] = Ar * G;
                    }
                    stg_f<Tr, V>(a.out0 + ((row0 + r) * a.o0rs + c0) * (int64_t)sizeof(Tr), dg);
                    stg_f<Tr, V>(a.out1 + ((row0 + r) * a.o1rs + c0) * (int64_t)sizeof(Tr), dv);
                }
            }
            if (a.e_last != nullptr && t0 == 0) {
#pragma unroll
                for (int i = 0; i < V; ++i) static_cast<float*>(a.e_last)[b * a.C + c0 + i] = x[i];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (!ok) break;
        if (++slot == nstage) {
            slot = 0;
            parity ^= 1u;
        }
    }
}

}  // namespace esa
